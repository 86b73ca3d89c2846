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
