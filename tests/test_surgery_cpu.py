"""FP8-surgery projection layers (mixers.py:681-800): construction, parameter
names and sharding rules, on CPU (no kernel calls)."""

from types import SimpleNamespace

import pytest
import torch


def _cfg(**kw):
    c = SimpleNamespace(hidden_size=64, short_filter_length=3, hcm_filter_length=128,
                        state_size=16, use_fp8_input_projections=False, vocab_size=512)
    c.__dict__.update(kw)
    return c


def test_surgery_layers_take_the_reference_projection_forms():
    from evo2_flash_b200.mixers import (Bf16Linear, HybridProjection, HyenaFIRMixer,
                                        HyenaIIRMixer, ProjectionTap)

    cfg = _cfg(hyena_token_table_layers=[0], hyena_fp8_emulated_layers=[1],
               hyena_fp8_emulated_channels={2: 5})
    table = HyenaFIRMixer(cfg, 0, prefix="l0", k_inner=7)
    assert isinstance(table.in_proj, ProjectionTap)
    assert tuple(table.in_proj_token_table.shape) == (512, 192)
    emul = HyenaFIRMixer(cfg, 1, prefix="l1", k_inner=128)
    assert isinstance(emul.in_proj, ProjectionTap) and emul.in_proj_token_table is None
    assert tuple(emul.in_proj_emul_weight_t.shape) == (64, 192)
    assert tuple(emul.in_proj_emul_scales.shape) == (2,)
    hyb = HyenaIIRMixer(cfg, 2, prefix="l2")
    assert isinstance(hyb.in_proj, HybridProjection)
    assert tuple(hyb.in_proj_emul_weight_t.shape) == (64, 5)
    assert hyb.in_proj_emul_cols.dtype == torch.int64
    plain = HyenaFIRMixer(cfg, 3, prefix="l3", k_inner=7)
    assert type(plain.in_proj) is Bf16Linear and plain.in_proj_emul_weight_t is None


def test_surgery_tensors_load_unsharded_and_refuse_sharding():
    from evo2_flash_b200.mixers import HyenaFIRMixer
    from evo2_flash_b200.parallel import shard_mixer_tensors

    cfg = _cfg(hyena_fp8_emulated_layers=[0])
    m = HyenaFIRMixer(cfg, 0, prefix="l0", k_inner=7)
    g = torch.Generator().manual_seed(0)
    t = {"in_proj_emul_weight_t": torch.randn(64, 192, generator=g).to(torch.bfloat16),
         "in_proj_emul_scales": torch.tensor([0.1, 0.02]),
         "short_filter": torch.randn(192, 1, 3, generator=g).to(torch.bfloat16),
         "conv": torch.randn(64, 1, 7, generator=g).to(torch.bfloat16),
         "out_proj.weight": torch.randn(64, 64, generator=g).to(torch.bfloat16),
         "out_proj.bias": torch.zeros(64, dtype=torch.bfloat16)}
    m.load_full_weights(t)
    assert torch.equal(m.in_proj_emul_weight_t, t["in_proj_emul_weight_t"])
    with pytest.raises(ValueError):
        shard_mixer_tensors(t, 0, 2, 64)
    with pytest.raises(ValueError):
        HyenaFIRMixer(cfg, 0, prefix="l0", k_inner=7, tp_rank=0, tp_size=2)


def _torch_ops(monkeypatch, calls):
    """CPU stand-ins for the three kernels the surgery projections call, so the
    host routing of mixer._project can be checked without a GPU."""
    from evo2_flash_b200 import ops

    def rms_norm(x, w, eps, residual=None, *, want_y=True, quant_scale=None, s_out=None):
        calls.append(("rms_norm", want_y, s_out is residual and residual is not None))
        s = x if residual is None else (x.float() + residual.float()).to(x.dtype)
        if s_out is not None:
            s_out.copy_(s)
        return (s * 0.5 if want_y else None), None

    def fp8_linear_emulated(x, w_t, scales):
        calls.append(("emulated", tuple(w_t.shape)))
        return torch.full((x.shape[0], w_t.shape[1]), 7.0, dtype=torch.bfloat16)

    def gemm_bf16(a, b, bias, out=None):
        calls.append(("gemm_bf16",))
        return (a.float() @ b.float().t()).to(torch.bfloat16)

    monkeypatch.setattr(ops, "rms_norm", rms_norm)
    monkeypatch.setattr(ops, "fp8_linear_emulated", fp8_linear_emulated)
    monkeypatch.setattr(ops, "gemm_bf16", gemm_bf16)


def test_project_routes_each_surgery_form(monkeypatch):
    """mixers.py:1076-1092: the token table needs token ids and returns the
    table rows; the emulated layer returns the emulation; the hybrid layer
    overwrites its emulated columns of the bf16 projection; with a pre-norm the
    residual add still happens (and a token-table layer asks for no normed
    output)."""
    from evo2_flash_b200.mixers import HyenaFIRMixer

    calls = []
    _torch_ops(monkeypatch, calls)
    g = torch.Generator().manual_seed(1)
    cfg = _cfg(hyena_token_table_layers=[0], hyena_fp8_emulated_layers=[1],
               hyena_fp8_emulated_channels={2: 3})
    x = torch.randn(5, 64, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 0, 511, 7, 7])
    norm = SimpleNamespace(weight=torch.ones(64, dtype=torch.bfloat16), eps=1e-6)

    table = HyenaFIRMixer(cfg, 0, prefix="r0", k_inner=7)
    with torch.no_grad():
        table.in_proj_token_table.copy_(torch.randn(512, 192, generator=g))
    assert torch.equal(table._project(x, ids), table.in_proj_token_table[ids])
    with pytest.raises(ValueError):
        table._project(x)
    res = torch.randn(5, 64, generator=g).to(torch.bfloat16)
    want = (x.float() + res.float()).to(torch.bfloat16)
    z = table._project(x, ids, pre_norm=norm, residual=res)
    assert torch.equal(z, table.in_proj_token_table[ids]) and torch.equal(res, want)
    assert calls[-1] == ("rms_norm", False, True)

    emul = HyenaFIRMixer(cfg, 1, prefix="r1", k_inner=7)
    z = emul._project(x)
    assert calls[-1] == ("emulated", (64, 192)) and torch.equal(z, torch.full_like(z, 7.0))

    hyb = HyenaFIRMixer(cfg, 2, prefix="r2", k_inner=7)
    with torch.no_grad():
        hyb.in_proj.weight.copy_(torch.randn(192, 64, generator=g))
        hyb.in_proj_emul_cols.copy_(torch.tensor([4, 100, 191]))
    z = hyb._project(x)
    plain = (x.float() @ hyb.in_proj.weight.float().t()).to(torch.bfloat16)
    keep = torch.ones(192, dtype=torch.bool)
    keep[[4, 100, 191]] = False
    assert torch.equal(z[:, ~keep], torch.full((5, 3), 7.0, dtype=torch.bfloat16))
    assert torch.equal(z[:, keep], plain[:, keep])
