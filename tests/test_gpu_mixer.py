"""The B200 mixer modules replay the reference's golden fixtures end to end:
in_proj (tcgen05 GEMM) -> fused core kernels -> out_proj (tcgen05 GEMM), with the
paged state, position stamps and speculative rollback handled by the module, and
every step's output compared with what the reference computed."""

from types import SimpleNamespace

import pytest
import torch

from tests.helpers import REL_TOL, load_fixture, max_rel_err, meta_from_dict

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = ["hcm_prefill", "hcs_mixed", "hcl_mixed", "hcm_decode", "hcm_spec", "hcl_spec", "hcs_spec"]


def build_mixer(fx, fp8=False):
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=fx["H"], short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=fp8)
    kw = dict(num_spec=fx["num_spec"], device=DEV)
    if fx["kind"] == "hcl":
        m = HyenaIIRMixer(cfg, 0, prefix=fx["name"], **kw)
    else:
        m = HyenaFIRMixer(cfg, 0, prefix=fx["name"], k_inner=fx["k_inner"], **kw)
    m.load_full_weights({k: v.to(DEV) for k, v in fx["params"].items()})
    m.allocate_state(fx["num_blocks"], DEV)
    return m


@pytest.mark.parametrize("name", CASES)
def test_mixer_replays_reference(name):
    from evo2_flash_b200 import set_forward_metadata

    fx = load_fixture(name)
    m = build_mixer(fx)
    seen = {}
    m.in_proj.register_forward_hook(lambda mod, a, o: seen.__setitem__("z", o[0]))
    m.out_proj.register_forward_hook(lambda mod, a, o: seen.__setitem__("g", a[0]))
    for i, step in enumerate(fx["steps"]):
        meta = meta_from_dict(step["meta"], DEV)
        with set_forward_metadata(meta):
            out = m(step["x"].to(DEV))
        torch.cuda.synchronize()
        assert max_rel_err(seen["z"].cpu(), step["z"]) < 1e-2, (name, i)
        assert max_rel_err(seen["g"].cpu(), step["g"]) < REL_TOL, (name, i)
        assert max_rel_err(out.cpu(), step["out"]) < REL_TOL, (name, i)
    ref = fx["final_states"]
    got = [s.cpu() for s in m.kv_cache]
    assert torch.equal(got[0][1:], ref[0][1:])
    if fx["kind"] == "hcl":
        # the fixture's prefill K=3 filter uses fp32 products (the reference's CPU
        # twin), this path bf16 ones (its GPU kernel): u differs in the last bit
        assert max_rel_err(got[2][1:, :, :16], ref[2][1:, :, :16]) < REL_TOL
    else:
        k = fx["k_inner"]
        assert max_rel_err(got[1][1:, : k - 1], ref[1][1:, : k - 1]) < REL_TOL
        if fx["num_spec"]:
            assert torch.equal(got[2][1:, 0, 16], ref[2][1:])


def test_profile_run_without_metadata():
    fx = load_fixture("hcm_prefill")
    m = build_mixer(fx)
    x = fx["steps"][0]["x"][:17].to(DEV)
    out = m(x)
    z = x.float() @ m.in_proj.weight.float().t()
    zb = z.to(torch.bfloat16)
    y = zb[:, 0::3] * zb[:, 1::3] * zb[:, 2::3]
    ref = y.float() @ m.out_proj.weight.float().t() + m.out_proj.bias.float()
    assert max_rel_err(out, ref) < REL_TOL


@pytest.mark.parametrize("name", ["hcm_prefill", "hcl_mixed"])
@pytest.mark.parametrize("fp8", [True, False])
def test_pre_norm_fused_into_the_in_proj_pass(name, fp8):
    """forward(add, pre_norm=norm, residual=x) == forward(norm(add + x)), with x
    updated to add + x in place, for the fp8 and the bf16 projection."""
    from evo2_flash_b200 import set_forward_metadata
    from evo2_flash_b200.model import Evo2RMSNorm

    fx = load_fixture(name)
    H = fx["H"]
    g = torch.Generator().manual_seed(3)
    norm = Evo2RMSNorm(H, 1e-6, DEV)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16))
    step = fx["steps"][0]
    add = step["x"].to(DEV)
    x0 = (torch.randn(add.shape, generator=g) * 3).to(torch.bfloat16).to(DEV)
    outs = []
    for fused in (True, False):
        m = build_mixer(fx, fp8=fp8)
        x = x0.clone()
        with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
            if fused:
                out = m(add, pre_norm=norm, residual=x)
            else:
                pre, x = norm(add, x)
                out = m(pre)
        torch.cuda.synchronize()
        outs.append((out.cpu(), x.cpu()))
    assert torch.equal(outs[0][1], (add.cpu().float() + x0.cpu().float()).to(torch.bfloat16))
    assert torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][0], outs[1][0])


def _surgery_mixer(fx, **flags):
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=fx["H"], short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False, vocab_size=512, **flags)
    kw = dict(num_spec=fx["num_spec"], device=DEV)
    if fx["kind"] == "hcl":
        return HyenaIIRMixer(cfg, 0, prefix=fx["name"] + "_s", **kw)
    return HyenaFIRMixer(cfg, 0, prefix=fx["name"] + "_s", k_inner=fx["k_inner"], **kw)


@pytest.mark.parametrize("name", ["hcs_mixed", "hcl_mixed"])
def test_token_table_layer(name):
    """FP8-surgery token table (mixers.py:1079-1084): z is the table row of each
    token, and the rest of the layer is the ordinary path (checked against the
    oracle's mixer core on the same z)."""
    from evo2_flash_b200 import set_forward_metadata
    from oracle import hyena_oracle as O
    from tests.helpers import empty_states, oracle_params

    fx = load_fixture(name)
    H = fx["H"]
    m = _surgery_mixer(fx, hyena_token_table_layers=[0])
    g = torch.Generator().manual_seed(8)
    table = (torch.randn(512, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
    params = {k: v for k, v in fx["params"].items() if k != "in_proj.weight"}
    params["in_proj_token_table"] = table
    m.load_full_weights({k: v.to(DEV) for k, v in params.items()})
    m.allocate_state(fx["num_blocks"], DEV)
    step = fx["steps"][0]
    T = step["x"].shape[0]
    ids = torch.randint(0, 512, (T,), generator=g)
    seen = {}
    m.in_proj.register_forward_hook(lambda mod, a, o: seen.__setitem__("z", o[0]))
    with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
        out = m(step["x"].to(DEV), ids.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(seen["z"].cpu(), table[ids])
    p = oracle_params(fx)
    ref = O.out_proj(O.mixer_core(table[ids], p, meta_from_dict(step["meta"]), empty_states(fx)), p)
    assert max_rel_err(out.cpu(), ref) < REL_TOL
    with pytest.raises(ValueError):
        with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
            m(step["x"].to(DEV))  # a token table needs the token ids


def test_emulated_and_hybrid_projections():
    """Fully emulated (mixers.py:1085-1089) and hybrid (mixers.py:691-702)
    FP8-surgery projections: z is the Hopper fast-accumulation model of the
    oracle, bit for bit, on the emulated columns; the hybrid's other columns are
    the bf16 projection."""
    from evo2_flash_b200 import ops, set_forward_metadata
    from oracle import hyena_oracle as O

    fx = load_fixture("hcs_mixed")
    H = fx["H"]
    g = torch.Generator().manual_seed(9)
    w8 = (torch.randn(3 * H, H, generator=g) * 60).clamp(-448, 448).to(torch.float8_e4m3fn)
    sx, sw = torch.tensor([0.02]), torch.tensor([0.004])
    step = fx["steps"][0]
    x = step["x"]
    z_emul = O.fp8_linear(x, w8, sx, sw, hopper=True)
    w_t = w8.float().t().contiguous().to(torch.bfloat16)
    scales = torch.cat([sx, sw])

    m = _surgery_mixer(fx, hyena_fp8_emulated_layers=[0])
    params = {k: v for k, v in fx["params"].items() if k != "in_proj.weight"}
    params.update(in_proj_emul_weight_t=w_t, in_proj_emul_scales=scales)
    m.load_full_weights({k: v.to(DEV) for k, v in params.items()})
    m.allocate_state(fx["num_blocks"], DEV)
    seen = {}
    m.in_proj.register_forward_hook(lambda mod, a, o: seen.__setitem__("z", o[0]))
    with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
        m(x.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(seen["z"].cpu(), z_emul)

    cols = torch.tensor([0, 5, 17, 3 * H - 1, 40, 41, 2, 99])
    m = _surgery_mixer(fx, hyena_fp8_emulated_channels={0: len(cols)})
    params = dict(fx["params"])
    params.update(in_proj_emul_weight_t=w_t[:, cols].contiguous(), in_proj_emul_scales=scales,
                  in_proj_emul_cols=cols)
    m.load_full_weights({k: v.to(DEV) for k, v in params.items()})
    m.allocate_state(fx["num_blocks"], DEV)
    seen = {}
    m.in_proj.register_forward_hook(lambda mod, a, o: seen.__setitem__("z", o[0]))
    with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
        m(x.to(DEV))
    torch.cuda.synchronize()
    z = seen["z"].cpu()
    assert torch.equal(z[:, cols], z_emul[:, cols])
    plain = ops.gemm_bf16(x.to(DEV), fx["params"]["in_proj.weight"].to(DEV), None).cpu()
    keep = torch.ones(3 * H, dtype=torch.bool)
    keep[cols] = False
    assert torch.equal(z[:, keep], plain[:, keep])


def test_forward_through_the_custom_op_matches_direct():
    """A mixer built with an engine compilation config runs forward() as
    torch.ops.evo2_b200.hyena_mixer; the result equals the direct call."""
    from evo2_flash_b200 import HyenaFIRMixer, set_forward_metadata

    fx = load_fixture("hcm_prefill")
    comp = SimpleNamespace(static_forward_context={}, splitting_ops=[])
    cfg = SimpleNamespace(hidden_size=fx["H"], short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    outs = []
    for i, cc in enumerate((comp, None)):
        m = HyenaFIRMixer(cfg, 0, prefix=f"op_test_{i}", k_inner=fx["k_inner"], device=DEV,
                          compilation_config=cc)
        m.load_full_weights({k: v.to(DEV) for k, v in fx["params"].items()})
        m.allocate_state(fx["num_blocks"], DEV)
        step = fx["steps"][0]
        with set_forward_metadata(meta_from_dict(step["meta"], DEV)):
            outs.append(m(step["x"].to(DEV)).cpu())
    assert torch.equal(outs[0], outs[1])
    assert max_rel_err(outs[0], fx["steps"][0]["out"]) < REL_TOL
