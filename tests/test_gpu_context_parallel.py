"""Context-parallel prefill (evo2_flash_b200.context_parallel): one sequence
split into P contiguous slices, each run by its own mixer instance (own paged
state, shared weights) with the previous slice's last rows as halo; the LI
layer's slice states are combined after a gather.  Every slice's output must
match the single-pass prefill of the whole sequence, and the last slice's final
state must match the single-pass final state.  Ranks are emulated on one GPU
(both passes of every slice, the gather in between), and run as real ranks on
2 GPUs with the NCCL all-gather (skipped with fewer GPUs)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import REL_TOL, max_rel_err, prefill_meta, random_params

pytestmark = pytest.mark.gpu
DEV = "cuda"
H = 256


def _mixer(kind, k, params, dev=DEV):
    from types import SimpleNamespace

    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    m = (HyenaIIRMixer(cfg, 0, prefix="cp", device=dev) if kind == "hcl"
         else HyenaFIRMixer(cfg, 0, prefix="cp", k_inner=k, device=dev))
    m.load_full_weights({kk: v.to(dev) for kk, v in params.items()})
    m.allocate_state(2, dev)
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


def _sequence(n):
    g = torch.Generator().manual_seed(73)
    return torch.randn(n, H, generator=g).to(torch.bfloat16)


def _cp_worker(rank, world, kind, k, port, out_dir, lens):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta

    from evo2_flash_b200.context_parallel import cp_prefill, halo_rows

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        x = _sequence(sum(lens)).to(dev)
        m = _mixer(kind, k, random_params(kind, H, k, seed=71), dev)
        a, n = sum(lens[:rank]), lens[rank]
        halo = None if rank == 0 else x[a - halo_rows(m):a]
        out = cp_prefill(m, x[a:a + n], halo, rank)  # the LI layer all-gathers over NCCL
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "state": [s[1].cpu() for s in m.kv_cache]},
                   os.path.join(out_dir, f"cp{rank}.pt"))
        dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kind,k", [("hcm", 128), ("hcl", 16)])
def test_cp2_real_ranks_match_single_pass(kind, k, tmp_path):
    """Two ranks on two GPUs, slices of unequal length (each rank's token count
    travels with its final state in the one all-gather)."""
    from evo2_flash_b200 import set_forward_metadata

    lens = [700, 500]
    full = _mixer(kind, k, random_params(kind, H, k, seed=71))
    with set_forward_metadata(prefill_meta([sum(lens)], [1], [False], device=DEV)):
        ref = full(_sequence(sum(lens)).to(DEV)).cpu()
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_cp_worker, args=(r, 2, kind, k, port, str(tmp_path), lens))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        got = torch.load(tmp_path / f"cp{r}.pt")
        a = sum(lens[:r])
        assert max_rel_err(got["out"], ref[a:a + lens[r]]) < REL_TOL, r
    last = torch.load(tmp_path / "cp1.pt")["state"]
    if kind == "hcl":
        assert max_rel_err(last[2], full.kv_cache[2][1].cpu()) < 1e-3
    else:
        assert torch.equal(last[1][: k - 1], full.kv_cache[1][1, : k - 1].cpu())
    assert torch.equal(last[0], full.kv_cache[0][1].cpu())
