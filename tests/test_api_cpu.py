"""The engine-free Evo2 surface (evo2_flash_b200.api) on CPU, its Hyena layers
computed by the oracle: tokenizer and reverse complement semantics, scoring
reductions against the harness's per-token log-probabilities, forward logits
and embeddings against scoring, and generation (prefill, then one-token decode
steps on the paged state and the attention cache) against teacher-forced
scoring of the generated text."""

import math

import pytest
import torch

from tests.helpers import OracleMixer

ACGT = "ACGT"


@pytest.fixture(scope="module")
def evo():
    from evo2_flash_b200.api import Evo2
    from evo2_flash_b200.model import StripedHyena2, StripedHyena2Config

    m = StripedHyena2(StripedHyena2Config.small(hidden=128), device="cpu",
                      mixer_factory=OracleMixer)
    m.load_tensors(m.random_tensors(11))
    return Evo2(m)


def _dna(n, seed):
    g = torch.Generator().manual_seed(seed)
    return "".join(ACGT[i] for i in torch.randint(0, 4, (n,), generator=g).tolist())


def test_tokenizer_bytes_and_clamped_decoding():
    from evo2_flash_b200.api import CharLevelTokenizer

    tok = CharLevelTokenizer(512)
    assert tok.tokenize("ACGT") == [65, 67, 71, 84]
    assert tok.tokenize("é") == [0xC3, 0xA9]  # UTF-8 bytes
    assert tok.eod_id == tok.eos == 0 and tok.pad_id == 1 and tok.vocab_size == 512
    assert tok.detokenize([0, 1, 65, 700]) == "  A" + chr(512)
    assert tok.detokenize(torch.tensor([67, 71])) == "CG"
    assert tok.tokenize_batch(["A", "CG"]) == [[65], [67, 71]]
    assert tok.detokenize_batch([[65], [84]]) == ["A", "T"]


def test_reverse_complement_iupac_and_case():
    from evo2_flash_b200.api import reverse_complement

    assert reverse_complement("ACGTNacgtU-") == "-AacgtNACGT"
    assert reverse_complement("MRWSYKVHDBX") == "XVHDBMRSWYK"
    s = _dna(50, 1)
    assert reverse_complement(reverse_complement(s)) == s


def test_score_sequences_reductions(evo):
    seqs = [_dna(40, 2), _dna(17, 3)]
    ids = [torch.tensor(evo.tokenizer.tokenize(s)) for s in seqs]
    lps = evo.model.token_logprobs(ids)
    mean = evo.score_sequences(seqs)
    total = evo.score_sequences(seqs, reduce_method="sum")
    for s, lp, a, b in zip(seqs, lps, mean, total):
        assert lp.numel() == len(s) - 1
        assert a == pytest.approx(float(lp.mean()), abs=1e-9)
        assert b == pytest.approx(float(lp.sum()), abs=1e-9)
    nll = evo.model.score(ids)
    assert mean == pytest.approx([-v for v in nll], abs=1e-9)
    # a prepended EOD scores every original token
    with_bos = evo.score_sequences(seqs, prepend_bos=True, reduce_method="sum")
    bos_lps = evo.model.token_logprobs([torch.tensor([0] + x.tolist()) for x in ids])
    assert with_bos == pytest.approx([float(v.sum()) for v in bos_lps], abs=1e-9)
    assert all(v.numel() == len(s) for v, s in zip(bos_lps, seqs))


def test_score_sequences_reverse_complement_and_errors(evo):
    from evo2_flash_b200.api import reverse_complement

    s = _dna(33, 4)
    a, b = evo.score_sequences([s, reverse_complement(s)])
    assert evo.score_sequences(s, average_reverse_complement=True)[0] == pytest.approx(
        0.5 * (a + b), abs=1e-12)
    assert math.isnan(evo.score_sequences(["A"])[0])
    assert evo.score_sequences(["A"], reduce_method="sum") == [0.0]
    assert evo.score_sequences([]) == []
    with pytest.raises(ValueError, match="reduce_method"):
        evo.score_sequences([s], reduce_method="max")
    with pytest.raises(ValueError, match="empty"):
        evo.score_sequences([""])


def test_chunked_steps_score_like_one_step(evo):
    seqs = [_dna(90, 5), _dna(61, 6), _dna(8, 7)]
    one = evo.score_sequences(seqs)
    evo.max_tokens_per_step = 32
    try:
        chunked = evo.score_sequences(seqs)
    finally:
        evo.max_tokens_per_step = None
    assert chunked == pytest.approx(one, abs=1e-3)


def test_forward_logits_and_embeddings(evo):
    s = [_dna(30, 8), _dna(30, 9)]
    ids = torch.tensor([evo.tokenizer.tokenize(x) for x in s])
    logits, emb = evo(ids, return_embeddings=True, layer_names=["blocks.0", "blocks.3", "norm",
                                                                "unembed"])
    H = evo.model.cfg.hidden_size
    assert logits.shape == (2, 30, 512) and logits.dtype == torch.bfloat16
    assert emb["blocks.0"].shape == (2, 30, H) and emb["norm"].shape == (2, 30, H)
    assert emb["unembed"] is logits
    # the logits predict exactly what scoring scores
    lp = torch.log_softmax(logits.float(), -1)
    for r in range(2):
        want = evo.model.token_logprobs([ids[r]])[0]
        got = lp[r, :-1].gather(1, ids[r, 1:, None]).squeeze(1).double()
        assert torch.allclose(got, want, atol=1e-6)
    # 'norm' is the final-norm output the logits are made from
    assert torch.equal(torch.nn.functional.linear(emb["norm"], evo.model.embed), logits)
    assert evo.forward(ids)[1] is None
    with pytest.raises(ValueError, match="layer_names"):
        evo.forward(ids, return_embeddings=True)
    with pytest.raises(ValueError, match="not supported"):
        evo.forward(ids, return_embeddings=True, layer_names=["blocks.0.pre_norm"])
    with pytest.raises(ValueError, match="unsupported layer name"):
        evo.forward(ids, return_embeddings=True, layer_names=["blocks.0.bogus"])
    with pytest.raises(ValueError, match="attention block"):
        evo.forward(ids, return_embeddings=True, layer_names=["blocks.3.filter"])
    with pytest.raises(ValueError, match="Hyena block"):
        evo.forward(ids, return_embeddings=True, layer_names=["blocks.0.inner_mha_cls"])
    with pytest.raises(ValueError, match="out of range"):
        evo.forward(ids, return_embeddings=True, layer_names=["blocks.99"])
    with pytest.raises(ValueError, match="token ids"):
        evo.forward([[0, 600]])


def _incremental_vs_prefill(model, prompt, toks, zero_state=False):
    """max_rel_err of every step's hidden state, prompt prefill then one-token
    decode steps, against the same rows of one teacher-forced prefill."""
    from tests.helpers import max_rel_err

    full = torch.tensor(prompt + toks)
    (ref, _), = list(model.prefill_steps([full]))
    (h, _), = list(model.prefill_steps([torch.tensor(prompt)], keep_cache=True))
    if zero_state:
        model.allocate_state(2)
    got = [h[-1]]
    for s in range(len(toks) - 1):
        got.append(model.decode_step([toks[s]], [len(prompt) + s], [0])[0])
    model.release_all()
    n = len(prompt)
    return [max_rel_err(g.float(), ref[n - 1 + i].float()) for i, g in enumerate(got)]


def test_decode_steps_continue_the_prefill(evo):
    """Prefill of a prompt, then one-token decode steps (mixer decode rows on the
    paged state, attention on its key/value cache), must give each position's
    hidden state as one teacher-forced prefill does, within the path's bar (bf16
    roundings differ with the step's length: GEMM blocking, the oracle's FFT
    size); decoding from a zeroed mixer state must not."""
    from tests.helpers import REL_TOL

    p = evo.tokenizer.tokenize(_dna(23, 11))
    toks = evo.tokenizer.tokenize(_dna(12, 13))
    errs = _incremental_vs_prefill(evo.model, p, toks)
    assert max(errs) < REL_TOL, errs
    bad = _incremental_vs_prefill(evo.model, p, toks, zero_state=True)
    assert max(bad[1:]) > 5 * REL_TOL, bad


def test_generate_greedy_matches_teacher_forced_scoring(evo):
    """Greedy generation: deterministic, exactly n_tokens per prompt, and its
    logprobs_mean agrees with teacher-forced scoring of the generated text
    (the bf16 differences between step lengths move individual log-probs by a
    few 1e-3 in this random-init model)."""
    prompts = [_dna(37, 10), _dna(23, 11)]
    out = evo.generate(prompts, n_tokens=12, top_k=1, verbose=0)
    assert [len(t) for t in out.token_ids] == [12, 12]
    for p, toks, mean in zip(prompts, out.token_ids, out.logprobs_mean):
        full = torch.tensor(evo.tokenizer.tokenize(p) + toks)
        lp = evo.model.token_logprobs([full])[0]
        assert float(lp[len(p) - 1:].mean()) == pytest.approx(mean, abs=5e-3)
    again = evo.generate(prompts, n_tokens=12, top_k=1, verbose=0)
    assert again.token_ids == out.token_ids
    assert out.sequences == [evo.tokenizer.detokenize(t) for t in out.token_ids]
    # logits that predicted each generated token, vortex layout
    lg = out.logits
    assert len(lg) == 2 and lg[0].shape == (1, 12, 512)


def test_generate_seeded_sampling_and_errors(evo):
    p = [_dna(20, 12)] * 2
    a = evo.generate(p, n_tokens=8, top_k=4, temperature=1.0, seed=7, verbose=0)
    b = evo.generate(p, n_tokens=8, top_k=4, temperature=1.0, seed=7, verbose=0)
    assert a.token_ids == b.token_ids
    assert a.logits[0].shape == (2, 8, 512)  # equal prompt lengths: one stacked tensor
    with pytest.raises(ValueError, match="n_tokens"):
        evo.generate(p, n_tokens=0)
    with pytest.raises(ValueError, match="temperature"):
        evo.generate(p, n_tokens=1, temperature=-1.0)
    with pytest.raises(ValueError, match="top-p"):
        evo.generate(p, n_tokens=1, top_p=1.5)
    with pytest.raises(ValueError, match="empty prompt"):
        evo.generate([""], n_tokens=1)


def test_sample_token_filters():
    from evo2_flash_b200.api import sample_token

    logits = torch.tensor([0.0, 5.0, 4.0, 3.0, -1.0])
    assert sample_token(logits, 1.0, 1, 1.0) == 1
    assert sample_token(logits, 0.0, 4, 1.0) == 1
    g = torch.Generator().manual_seed(0)
    draws = {sample_token(logits, 1.0, 2, 1.0, g) for _ in range(200)}
    assert draws == {1, 2}  # top-2 only
    # top-p keeps the shortest prefix reaching the mass: p(1) ~ 0.66 < 0.7 <= p(1) + p(2)
    draws = {sample_token(logits, 1.0, 0, 0.7, g) for _ in range(200)}
    assert draws == {1, 2}
    draws = {sample_token(logits, 1.0, 0, 0.5, g) for _ in range(50)}
    assert draws == {1}


def test_chunked_prompts_generate_and_forward_like_one_step(evo):
    """Prompts longer than the step budget are prefilled over several steps
    (resumed from the paged state) before decoding; forward over chunked steps
    returns every position's logits."""
    prompts = [_dna(70, 14), _dna(45, 15)]
    one = evo.generate(prompts, n_tokens=6, top_k=1, verbose=0)
    ids = torch.tensor([evo.tokenizer.tokenize(_dna(60, 16))])
    lg_one, _ = evo.forward(ids)
    evo.max_tokens_per_step = 24
    try:
        chunked = evo.generate(prompts, n_tokens=6, top_k=1, verbose=0)
        lg_chunked, _ = evo.forward(ids)
    finally:
        evo.max_tokens_per_step = None
    assert [len(t) for t in chunked.token_ids] == [6, 6]
    assert chunked.logprobs_mean == pytest.approx(one.logprobs_mean, abs=5e-3)
    lp1 = torch.log_softmax(lg_one.float(), -1)
    lp2 = torch.log_softmax(lg_chunked.float(), -1)
    assert (lp1 - lp2).abs().max() < 5e-2


def test_forward_module_embeddings_by_vortex_name(evo):
    """Module outputs by the reference's vortex names, captured by forward hooks:
    the MLP and its l1..l3, the attention mixer and its o_proj, the embedding."""
    ids = torch.tensor([evo.tokenizer.tokenize(_dna(40, 17))])
    names = ["blocks.0.mlp", "blocks.0.mlp.l3", "blocks.1.mlp.l1", "blocks.3.inner_mha_cls",
             "blocks.3.inner_mha_cls.out_proj", "embedding_layer", "blocks.2"]
    logits, emb = evo(ids, return_embeddings=True, layer_names=names)
    cfg = evo.model.cfg
    assert list(emb) == names
    assert emb["blocks.1.mlp.l1"].shape == (1, 40, cfg.intermediate_size)
    assert torch.equal(emb["blocks.0.mlp"], emb["blocks.0.mlp.l3"])  # the MLP's output is l3's
    assert torch.equal(emb["blocks.3.inner_mha_cls"], emb["blocks.3.inner_mha_cls.out_proj"])
    assert torch.equal(emb["embedding_layer"], evo.model.embed[ids])
    # the same names over chunked steps give the same rows
    evo.max_tokens_per_step = 16
    try:
        _, emb2 = evo(ids, return_embeddings=True, layer_names=["blocks.0.mlp.l3"])
    finally:
        evo.max_tokens_per_step = None
    from tests.helpers import REL_TOL, max_rel_err

    assert max_rel_err(emb2["blocks.0.mlp.l3"].float(), emb["blocks.0.mlp.l3"].float()) < REL_TOL
    # Hyena-module names need the B200 mixers' in_proj / out_proj submodules
    with pytest.raises(ValueError, match="no module"):
        evo(ids, return_embeddings=True, layer_names=["blocks.0.projections"])
