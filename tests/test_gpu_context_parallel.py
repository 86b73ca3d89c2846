"""Context-parallel prefill (evo2_flash_b200.context_parallel): one sequence
split into P contiguous slices, each run by its own mixer instance (own paged
state, shared weights) with the previous slice's last rows as halo; the LI
layer's slice states are combined after a gather.  Every slice's output must
match the single-pass prefill of the whole sequence, and the last slice's final
state must match the single-pass final state.  Ranks are emulated on one GPU
(both passes of every slice, the gather in between)."""

import pytest
import torch

from tests.helpers import REL_TOL, max_rel_err, prefill_meta, random_params

pytestmark = pytest.mark.gpu
DEV = "cuda"
H = 256


def _mixer(kind, k, params):
    from types import SimpleNamespace

    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    m = (HyenaIIRMixer(cfg, 0, prefix="cp", device=DEV) if kind == "hcl"
         else HyenaFIRMixer(cfg, 0, prefix="cp", k_inner=k, device=DEV))
    m.load_full_weights({kk: v.to(DEV) for kk, v in params.items()})
    m.allocate_state(2, DEV)
    return m


@pytest.mark.parametrize("kind,k", [("hcs", 7), ("hcm", 128), ("hcl", 16)])
@pytest.mark.parametrize("P", [2, 4])
def test_slices_match_single_pass(kind, k, P):
    from evo2_flash_b200 import set_forward_metadata
    from evo2_flash_b200.context_parallel import cp_prefill_start, halo_rows

    L = 600
    params = random_params(kind, H, k, seed=71)
    g = torch.Generator().manual_seed(72)
    x = (torch.randn(P * L, H, generator=g)).to(torch.bfloat16).to(DEV)
    full = _mixer(kind, k, params)
    with set_forward_metadata(prefill_meta([P * L], [1], [False], device=DEV)):
        ref = full(x)
    mixers = [_mixer(kind, k, params) for _ in range(P)]
    hr = halo_rows(mixers[0])
    starts = [cp_prefill_start(mixers[r], x[r * L:(r + 1) * L],
                               None if r == 0 else x[r * L - hr:r * L], r) for r in range(P)]
    if kind == "hcl":
        finals = torch.stack([s.local_final for s in starts])
        outs = [s.finish(finals) for s in starts]
    else:
        outs = starts
    torch.cuda.synchronize()
    for r in range(P):
        assert max_rel_err(outs[r], ref[r * L:(r + 1) * L]) < REL_TOL, r
    last = mixers[-1].kv_cache
    if kind == "hcl":
        assert max_rel_err(last[2][1], full.kv_cache[2][1]) < 1e-3
    else:
        assert torch.equal(last[1][1, : k - 1], full.kv_cache[1][1, : k - 1])
    assert torch.equal(last[0][1], full.kv_cache[0][1])
