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


def test_block_chain_keeps_the_reference_order_of_roundings():
    """Carrying each block's MLP output into the next block's pre-norm (the fused
    add-norm chain) gives bit for bit the reference's per-block order
    (model.py:189-198: pre-norm, mixer, post-norm of m + x, mlp(post) + x)."""
    from evo2_flash_b200.forward_context import set_forward_metadata
    from evo2_flash_b200.model import StripedHyena2Config, _prefill_meta
    from evo2_flash_b200.synthetic import markov_acgt

    cfg = StripedHyena2Config.small(hidden=128)
    m = _model(cfg)
    seqs = markov_acgt([90, 33], seed=4)
    segs, a = [], 0
    for j, s in enumerate(seqs):
        segs.append((a, a + len(s), j, 0))
        a += len(s)
    ids = torch.cat(seqs)
    pos = torch.cat([torch.arange(len(s)) for s in seqs])
    m.allocate_state(len(seqs) + 1)
    got = m(ids, pos, _prefill_meta(segs, "cpu"), segs)
    m.allocate_state(len(seqs) + 1)
    for layer in m.layers:
        if layer.kind == "attn":
            layer.mixer.kv.clear()
    x = m.embed[ids]
    with set_forward_metadata(_prefill_meta(segs, "cpu")):
        for layer in m.layers:
            pre = layer.pre_norm(x)
            mo = layer.mixer(pre, pos, segs) if layer.kind == "attn" else layer.mixer(pre)
            post, x = layer.post_norm(mo, x)
            x = layer.mlp(post) + x
    assert torch.equal(got, m.norm(x))


def test_add_norm_in_place_matches_the_two_output_form():
    from evo2_flash_b200.model import Evo2RMSNorm

    g = torch.Generator().manual_seed(0)
    norm = Evo2RMSNorm(64, 1e-6)
    norm.weight.copy_((1 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16))
    x = (torch.randn(5, 64, generator=g) * 3).to(torch.bfloat16)
    r = (torch.randn(5, 64, generator=g) * 1e6).to(torch.bfloat16)
    y_ref, s_ref = norm(x, r)
    r2 = r.clone()
    y = norm.add_norm_(x, r2)
    assert torch.equal(y, y_ref) and torch.equal(r2, s_ref)


def test_mixer_residual_needs_pre_norm():
    import pytest
    from types import SimpleNamespace

    from evo2_flash_b200 import HyenaFIRMixer

    cfg = SimpleNamespace(hidden_size=64, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    mixer = HyenaFIRMixer(cfg, 0, prefix="m", k_inner=7)
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        mixer(x, residual=x.clone())
