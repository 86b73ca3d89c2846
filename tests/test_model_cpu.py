"""The full-model harness on CPU with oracle-computed Hyena mixers: chunked
prefill (sequences split across steps, resumed from paged state) scores the same
as one-step prefill, and the Markov token source is seeded and well-formed."""

import math

import torch

from tests.helpers import OracleMixer


def _model(cfg, seed=5):
    from evo2_flash_b200.model import StripedHyena2

    m = StripedHyena2(cfg, device="cpu", mixer_factory=OracleMixer)
    m.load_tensors(m.random_tensors(seed))
    return m


def test_markov_sequences_are_seeded_acgt():
    from evo2_flash_b200.synthetic import ACGT, markov_acgt

    a = markov_acgt([50, 7, 0], seed=3)
    b = markov_acgt([50, 7, 0], seed=3)
    assert [x.tolist() for x in a] == [x.tolist() for x in b]
    assert [len(x) for x in a] == [50, 7, 0]
    assert set(torch.cat(a).tolist()) <= set(ACGT)
    # an order-3 chain with Dirichlet(1) rows is far from uniform: the empirical
    # next-letter entropy given 3 letters of context is well below 2 bits
    s = markov_acgt([20000], seed=3)[0]
    idx = torch.tensor([ACGT.index(v) for v in s.tolist()])
    ctx = idx[:-3] * 16 + idx[1:-2] * 4 + idx[2:-1]
    counts = torch.zeros(64, 4)
    counts.index_put_((ctx, idx[3:]), torch.ones(len(ctx)), accumulate=True)
    p = counts / counts.sum(1, keepdim=True).clamp_min(1)
    h = -(p * p.clamp_min(1e-12).log2()).sum(1)
    w = counts.sum(1) / counts.sum()
    assert float((w * h).sum()) < 1.9


def test_chunked_prefill_scores_like_one_step():
    from evo2_flash_b200.model import StripedHyena2Config
    from evo2_flash_b200.synthetic import markov_acgt

    cfg = StripedHyena2Config.small(hidden=128)
    m = _model(cfg)
    seqs = markov_acgt([300, 41, 170, 2], seed=3)
    one = m.score(seqs)
    chunked = m.score(seqs, max_tokens_per_step=128)
    assert all(math.isfinite(v) for v in one)
    for a, b in zip(one, chunked):
        assert abs(a - b) < 1e-3, (one, chunked)
    # a random-init byte model is near-uniform over the 512-token vocabulary
    assert abs(sum(one) / len(one) - math.log(512)) < 0.5
