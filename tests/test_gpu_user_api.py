"""The engine-free Evo2 surface (evo2_flash_b200.api) on the B200 mixers, bf16
projections: `score_sequences` against the all-reference arm (the same weights,
every Hyena mixer computed by the CPU oracle) within the path's NLL bar; the
decode steps' hidden states (prompt prefill, then one-token steps through the
decode kernels) against one teacher-forced prefill within the path's bar, with
a decode from a zeroed mixer state as the control that must miss it; and
`generate`'s logprobs_mean against teacher-forced scoring of its own text;
embeddings by vortex name, the Hyena projections' included."""

import math

import pytest
import torch

from tests.helpers import REL_TOL, OracleMixer
from tests.test_api_cpu import _dna, _incremental_vs_prefill

pytestmark = pytest.mark.gpu
NLL_TOL = 1e-3


def test_evo2_surface_on_the_b200_mixers():
    from evo2_flash_b200.api import Evo2
    from evo2_flash_b200.model import StripedHyena2, StripedHyena2Config

    cfg = StripedHyena2Config.small(hidden=256, use_fp8_input_projections=False)
    gpu = StripedHyena2(cfg, device="cuda")
    ref = StripedHyena2(cfg, device="cpu", mixer_factory=OracleMixer)
    t = gpu.random_tensors(17)
    gpu.load_tensors(t)
    ref.load_tensors(t)
    eg, er = Evo2(gpu), Evo2(ref)

    seqs = [_dna(600, 31), _dna(300, 32), _dna(120, 33)]
    a, b = eg.score_sequences(seqs), er.score_sequences(seqs)
    assert all(math.isfinite(v) for v in a)
    assert abs(sum(a) / len(a) - sum(b) / len(b)) <= NLL_TOL, (a, b)
    for x, y in zip(a, b):
        assert abs(x - y) <= 2 * NLL_TOL, (a, b)

    p = eg.tokenizer.tokenize(_dna(200, 21))
    toks = eg.tokenizer.tokenize(_dna(16, 22))
    errs = _incremental_vs_prefill(gpu, p, toks)
    assert max(errs) < REL_TOL, errs
    bad = _incremental_vs_prefill(gpu, p, toks, zero_state=True)
    assert min(bad[1:]) > 5 * REL_TOL, bad

    prompts = [_dna(50, 40), _dna(50, 41)]
    out = eg.generate(prompts, n_tokens=16, top_k=4, seed=3, verbose=0)
    assert [len(v) for v in out.token_ids] == [16, 16]
    for pr, tt, mean in zip(prompts, out.token_ids, out.logprobs_mean):
        full = torch.tensor(eg.tokenizer.tokenize(pr) + tt)
        lp = gpu.token_logprobs([full])[0][len(pr) - 1:]
        assert abs(float(lp.mean()) - mean) <= NLL_TOL, (float(lp.mean()), mean)

    ids = torch.tensor([eg.tokenizer.tokenize(_dna(64, 50))])
    lg, emb = eg(ids, return_embeddings=True,
                 layer_names=["blocks.2", "norm", "blocks.1.projections", "blocks.1.filter",
                              "blocks.1.out_filter_dense"])
    assert lg.shape == (1, 64, 512) and emb["blocks.2"].shape == (1, 64, 256)
    assert emb["blocks.1.projections"].shape == (1, 64, 768)  # the in_proj triple, 3H
    assert emb["blocks.1.filter"].shape == emb["blocks.1.out_filter_dense"].shape == (1, 64, 256)
    assert bool(torch.isfinite(lg.float()).all())
    # hooks on a layer's projections leave its output as it was
    lg0, _ = eg(ids)
    assert torch.equal(lg, lg0)
