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


def test_7b_shape_every_mixer_and_the_nll():
    """Config 4 at the full 7B shape (32 blocks, H = 4096, MLP 11008, fp8
    in_proj): three sequences, 512 tokens in steps of at most 256, so one
    sequence resumes from its paged state.

    Per layer: while the B200 model scores, every one of its 27 Hyena mixers is
    also computed by the CPU oracle on the very same input (teacher forcing,
    each oracle mixer keeping its own paged state); each output must match to
    the path's bar, per token row and per channel.

    End to end: the free-running all-reference arm (every Hyena mixer by the
    oracle, all else the same torch code on the GPU).  A random-init model this
    deep is chaotic under rounding: the e4m3 quantisation of each Hyena layer's
    input turns a last-bit difference upstream into a whole e4m3 step, and the
    cubic gates amplify it layer by layer.  The reference's own two numerics,
    exact fp32 accumulation (its Blackwell path) and the Hopper fast-accumulation
    model (its H100 path, fp8_emul.py), give mean NLLs 1.5e-2 apart on this very
    sample (7.0673 vs 7.0824; measured with the oracle), while the B200 arm sits
    1.3e-2 from the first.  So the 1e-3 bar of the reference's own test, which it
    applies to trained checkpoints (test_evo2.py:31), is held on the 7-block
    models above; here the free-running gap is held to that measured spread."""
    from evo2_flash_b200.model import StripedHyena2, StripedHyena2Config
    from evo2_flash_b200.synthetic import markov_acgt
    from tests.helpers import REL_TOL, max_slice_rel_err

    cfg = StripedHyena2Config.evo2_7b()
    gpu = StripedHyena2(cfg, device="cuda")
    ref = StripedHyena2(cfg, device="cuda", mixer_factory=OracleMixer)
    forced = StripedHyena2(cfg, device="cuda", mixer_factory=OracleMixer)
    t = gpu.random_tensors(17, gen_device="cuda")
    for m in (gpu, ref, forced):
        m.load_tensors(t)
    del t
    seqs = markov_acgt([300, 150, 62], seed=6)
    forced.allocate_state(len(seqs) + 1)
    errs, hooks = [], []
    for i, layer in enumerate(gpu.layers):
        if layer.kind == "attn":
            continue
        layer.mixer.fuses_pre_norm = False  # the oracle mixer takes the normed input

        def hook(mod, args, out, twin=forced.layers[i].mixer, i=i):
            errs.append((i, max_slice_rel_err(out.float().cpu(), twin(args[0]).float().cpu())))
        hooks.append(layer.mixer.register_forward_hook(hook))
    a = gpu.score(seqs, max_tokens_per_step=256)
    for h in hooks:
        h.remove()
    assert len(errs) == 2 * 27
    worst = max(errs, key=lambda e: e[1])
    assert worst[1] < REL_TOL, worst
    b = ref.score(seqs, max_tokens_per_step=256)
    assert all(math.isfinite(v) for v in a)
    mean_a, mean_b = sum(a) / len(a), sum(b) / len(b)
    assert abs(mean_a - mean_b) <= 1.5e-2, (a, b)


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
