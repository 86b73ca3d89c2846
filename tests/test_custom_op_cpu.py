"""The mixer's custom-op boundary (mixers.py:807-829, 1404-1423), on CPU: the op
resolves the layer by name and mutates `output`; its fake implementation runs
nothing; an engine compilation config gets the layer registered (duplicate
names refused) and the op appended to its splitting ops."""

from types import SimpleNamespace

import pytest
import torch


class _Stub:
    def _forward_impl(self, hidden_states, token_ids=None):
        out = hidden_states * 2
        if token_ids is not None:
            out = out + token_ids[:, None].to(out.dtype)
        return out


def test_op_calls_the_named_layer_and_passes_opcheck():
    from evo2_flash_b200.custom_op import register_layer

    stub = _Stub()
    register_layer("stub.mixer", stub)
    x = torch.randn(6, 8)
    out = torch.empty_like(x)
    ids = torch.arange(6)
    torch.ops.evo2_b200.hyena_mixer(x, out, ids, "stub.mixer")
    assert torch.equal(out, x * 2 + ids[:, None].float())
    torch.library.opcheck(torch.ops.evo2_b200.hyena_mixer.default,
                          (x, torch.empty_like(x), None, "stub.mixer"))


def test_fake_implementation_runs_nothing():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(4, 8)
        out = torch.empty_like(x)
        # no layer of this name exists: only the fake implementation may run
        assert torch.ops.evo2_b200.hyena_mixer(x, out, None, "not.registered") is None


def test_engine_config_registration():
    from evo2_flash_b200.custom_op import HYENA_MIXER_OP
    from evo2_flash_b200.mixers import HyenaFIRMixer

    comp = SimpleNamespace(static_forward_context={}, splitting_ops=[])
    cfg = SimpleNamespace(hidden_size=64, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    m = HyenaFIRMixer(cfg, 0, prefix="model.layers.0.mixer", k_inner=7, compilation_config=comp)
    assert comp.static_forward_context["model.layers.0.mixer"] is m and m.use_custom_op
    assert comp.splitting_ops == [HYENA_MIXER_OP]
    with pytest.raises(ValueError):
        HyenaFIRMixer(cfg, 1, prefix="model.layers.0.mixer", k_inner=7, compilation_config=comp)


def test_engine_state_surface():
    """get_state_shape / get_state_dtype / mamba_type / get_attn_backend, the
    MambaBase surface vLLM builds the paged state from (mixers.py:832-917)."""
    from evo2_flash_b200.mixers import HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=64, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    m = HyenaIIRMixer(cfg, 0, prefix="surface.mixer", num_spec=3)
    assert m.get_state_shape() == ((2 + 3, 192), (127, 64), (64, 17))
    assert m.get_state_dtype() == (torch.bfloat16, torch.float32, torch.float32)
    try:
        from vllm.v1.attention.backends.mamba2_attn import Mamba2AttentionBackend
        from vllm.v1.attention.backends.registry import MambaAttentionBackendEnum
    except Exception:
        assert m.mamba_type == "mamba2"
        return
    assert m.mamba_type == MambaAttentionBackendEnum.MAMBA2
    assert m.get_attn_backend() is Mamba2AttentionBackend
    m.attn_backend = object
    assert m.get_attn_backend() is object
