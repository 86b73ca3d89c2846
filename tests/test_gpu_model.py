"""Full-model parity: a random-init StripedHyena2 (7-block [HCS, HCM, HCL, MHA]
pattern, fp8 in_proj) scored with the B200 mixers must give the same mean
per-token NLL as the same model with every Hyena mixer computed by the CPU
oracle (the all-reference arm), within 1e-3 nats, on sequences from a seeded
order-3 Markov chain over ACGT.  Steps pack several sequences and split long ones
across steps, so prefill state continuation is part of what is compared."""

import math

import pytest
import torch

from tests.helpers import OracleMixer, max_rel_err

pytestmark = pytest.mark.gpu
NLL_TOL = 1e-3


def _pair(hidden, seed=11):
    from evo2_flash_b200.model import StripedHyena2, StripedHyena2Config

    cfg = StripedHyena2Config.small(hidden=hidden)
    gpu = StripedHyena2(cfg, device="cuda")
    ref = StripedHyena2(cfg, device="cpu", mixer_factory=OracleMixer)
    t = gpu.random_tensors(seed)
    gpu.load_tensors(t)
    ref.load_tensors(t)
    return gpu, ref


@pytest.mark.parametrize("hidden,budget", [(256, None), (256, 700), (512, 1024)])
def test_mean_nll_matches_reference_arm(hidden, budget):
    from evo2_flash_b200.synthetic import markov_acgt

    gpu, ref = _pair(hidden)
    seqs = markov_acgt([1200, 257, 640, 33, 900], seed=3)
    a = gpu.score(seqs, max_tokens_per_step=budget)
    b = ref.score(seqs, max_tokens_per_step=budget)
    assert all(math.isfinite(v) for v in a)
    mean_a, mean_b = sum(a) / len(a), sum(b) / len(b)
    assert abs(mean_a - mean_b) <= NLL_TOL, (a, b)
    for x, y in zip(a, b):
        assert abs(x - y) <= 2 * NLL_TOL, (a, b)


def test_final_hidden_states_match_reference_arm():
    from evo2_flash_b200.model import _prefill_meta
    from evo2_flash_b200.synthetic import markov_acgt

    gpu, ref = _pair(256)
    seqs = markov_acgt([500, 77, 300], seed=4)
    segs, a = [], 0
    for j, s in enumerate(seqs):
        segs.append((a, a + len(s), j, 0))
        a += len(s)
    ids = torch.cat(seqs)
    pos = torch.cat([torch.arange(len(s)) for s in seqs])
    outs = []
    for m, dev in ((gpu, "cuda"), (ref, "cpu")):
        m.allocate_state(len(seqs) + 1)
        outs.append(m(ids.to(dev), pos.to(dev), _prefill_meta(segs, dev), segs).float().cpu())
    # seven blocks of bf16 GEMMs on two devices: a few bf16 ulps of drift
    assert max_rel_err(outs[0], outs[1]) < 5e-2
