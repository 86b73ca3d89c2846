"""GPU parity of the sm_100a kernels, called through the C ABI (evo2_flash_b200.ops),
against the CPU oracle on the same seeded inputs.

Tolerance: the hot path's bar is max|a-b| / max|b| <= 2e-2 on bf16 outputs
(REL_TOL); integer-valued / copied state (windows of bf16 inputs) must match
bit for bit.
"""

import pytest
import torch

from oracle import hyena_oracle as O
from tests.helpers import (REL_TOL, decode_meta, max_rel_err, params_to_oracle, prefill_meta,
                           random_params)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _weights(p, kind):
    from evo2_flash_b200 import ops

    if kind == "hcl":
        return ops.layer_weights("iir", p["short_filter"], D=p["D"], log_poles=p["log_poles"],
                                 residues=p["residues"])
    return ops.layer_weights("fir", p["short_filter"], conv=p["conv"], D=p.get("D"))


def _random_states(H, num_blocks, W0, seed, spec_col=False):
    g = torch.Generator().manual_seed(seed)
    s0 = (torch.randn(num_blocks, W0, 3 * H, generator=g) * 0.3).to(torch.bfloat16)
    s1 = torch.randn(num_blocks, 127, H, generator=g) * 0.1
    s2 = torch.randn(num_blocks, H, 17 if spec_col else 16, generator=g)
    return [s0, s1, s2]


KINDS = [("hcs", 7), ("hcm", 128), ("hcl", 16)]


@pytest.mark.parametrize("kind,k", KINDS)
@pytest.mark.parametrize("layout", ["ragged", "long", "tiny"])
def test_prefill_matches_oracle(kind, k, layout):
    from evo2_flash_b200 import ops

    H = 256
    if layout == "ragged":
        lengths, init = [700, 5, 131, 1, 1290, 64], [False, True, True, True, False, True]
    elif layout == "long":
        lengths, init = [3000, 1700], [True, False]
    else:
        lengths, init = [1, 2, 3, 126, 127, 128], [True] * 6
    nb = len(lengths) + 2
    blocks = list(range(2, 2 + len(lengths)))
    p = random_params(kind, H, k, seed=11)
    po = params_to_oracle(p, kind, H, k)
    T = sum(lengths)
    g = torch.Generator().manual_seed(12)
    z = (torch.randn(T, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
    states = _random_states(H, nb, 2, seed=13)
    ref_states = [s.clone() for s in states]
    meta = prefill_meta(lengths, blocks, init)
    ref = O.mixer_core(z, po, meta, ref_states, None, bf16_products=True)

    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    dz = z.to(DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ds = [s.to(DEV) for s in states]
    inner = ds[2] if kind == "hcl" else ds[1]
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    dm = prefill_meta(lengths, blocks, init, device=DEV)
    ops.prefill(w, dz, out, dm.query_start_loc_p, dm.has_initial_states_p, dm.state_indices_tensor_p,
                ds[0], inner, error_flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    err = max_rel_err(out.cpu(), ref)
    assert err < REL_TOL, err
    assert torch.equal(ds[0].cpu(), ref_states[0])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu(), ref_states[2]) < 1e-4
    else:
        assert torch.equal(ds[1].cpu()[:, : k - 1], ref_states[1][:, : k - 1])
        assert torch.equal(ds[1].cpu()[:, k - 1:], states[1][:, k - 1:])


def test_hcl_prefill_against_float64_scan():
    """Long segment: the chunked scan agrees with an exact float64 recurrence."""
    from evo2_flash_b200 import ops

    H, L = 128, 5000
    p = random_params("hcl", H, 16, seed=21)
    g = torch.Generator().manual_seed(22)
    z = (torch.randn(L, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
    s_prev = torch.randn(H, 16, generator=g)
    states = [torch.zeros(2, 2, 3 * H, dtype=torch.bfloat16), torch.zeros(2, 127, H),
              torch.zeros(2, H, 16)]
    states[2][1] = s_prev
    meta = prefill_meta([L], [1], [True])
    # u and x2 from the oracle's short filter, the LI map from the float64 scan
    zf = O.short_fir_prefill(z, p["short_filter"].reshape(3 * H, 3), meta,
                             states[0].clone(), True)
    x2, x1, v = zf[:, 0::3], zf[:, 1::3], zf[:, 2::3]
    u = x1 * v
    y64, s64 = O.iir_segment_scan(u.float().t(), p["residues"], p["log_poles"][..., 0], s_prev)
    y = y64.t().to(torch.bfloat16)
    ref = (y + u * p["D"]) * x2

    w = _weights({kk: vv.to(DEV) for kk, vv in p.items()}, "hcl")
    out = torch.empty(L, H, dtype=torch.bfloat16, device=DEV)
    ds = [s.to(DEV) for s in states]
    dm = prefill_meta([L], [1], [True], device=DEV)
    ops.prefill(w, z.to(DEV), out, dm.query_start_loc_p, dm.has_initial_states_p,
                dm.state_indices_tensor_p, ds[0], ds[2])
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert max_rel_err(ds[2][1].cpu(), s64) < 1e-4


@pytest.mark.parametrize("kind,k", KINDS)
@pytest.mark.parametrize("layout", ["sd", "dim_first"])
def test_decode_matches_oracle(kind, k, layout):
    """Ordinary decode; the SD layout takes the vectorised q=1 kernels, the
    dim-first storage (channel stride != 1) the generic kernel."""
    from evo2_flash_b200 import ops

    H, B = 256, 5
    p = random_params(kind, H, k, seed=31)
    po = params_to_oracle(p, kind, H, k)
    states = _random_states(H, 8, 2, seed=32)
    slots = [3, 1, 6, 2, 7]
    g = torch.Generator().manual_seed(33)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    if layout == "sd":
        ds = [s.to(DEV) for s in states]
    else:  # same logical tensors, stored dim-first
        ds = [s.to(DEV).transpose(1, 2).contiguous().transpose(1, 2) for s in states]
    ref_states = [s.clone() for s in states]
    for step in range(3):
        z = (torch.randn(B, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
        meta = decode_meta(slots)
        ref = O.mixer_core(z, po, meta, ref_states, None, bf16_products=True)
        out = torch.empty(B, H, dtype=torch.bfloat16, device=DEV)
        idx = torch.tensor(slots, dtype=torch.int32, device=DEV)
        ops.decode(w, z.to(DEV), out, idx, idx, idx[:, None], idx[:, None], ds[0],
                   ds[2] if kind == "hcl" else ds[1], zero_null_rows=True)
        torch.cuda.synchronize()
        assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert torch.equal(ds[0].cpu(), ref_states[0])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu(), ref_states[2]) < 1e-5
    else:
        assert torch.equal(ds[1].cpu()[:, : k - 1], ref_states[1][:, : k - 1])


@pytest.mark.parametrize("kind,k", KINDS)
def test_verify_matches_oracle(kind, k):
    """Speculative verify: q=4, ragged lengths, accepted counts 1..4, snapshots."""
    from evo2_flash_b200 import ops

    H = 256
    p = random_params(kind, H, k, seed=41)
    po = params_to_oracle(p, kind, H, k)
    slots = [[1, 5, 6, 7], [2, 8, 9, 10], [3, 11, 12, 13]]
    lengths = [4, 2, 1]
    accepted = torch.tensor([1, 3, 4])
    states = _random_states(H, 14, 5, seed=42, spec_col=True)
    ref_states = [s.clone() for s in states]
    T = sum(lengths)
    g = torch.Generator().manual_seed(43)
    z = (torch.randn(T, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
    meta = decode_meta(slots, lengths, computed=[10, 20, 30])
    ref = O.mixer_core(z, po, meta, ref_states, accepted, bf16_products=True)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    ds = [s.to(DEV) for s in states]
    st = torch.tensor(slots, dtype=torch.int32, device=DEV)
    qs = torch.tensor([0, 4, 6, 7], dtype=torch.int32, device=DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.decode(w, z.to(DEV), out, st[:, 0], st[:, 0], st, st, ds[0],
               ds[2] if kind == "hcl" else ds[1], token_start=qs, accepted=accepted.to(DEV))
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert torch.equal(ds[0].cpu()[1:], ref_states[0][1:])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu()[1:, :, :16], ref_states[2][1:, :, :16]) < 1e-5
    else:
        assert torch.equal(ds[1].cpu()[1:, : k - 1], ref_states[1][1:, : k - 1])


@pytest.mark.parametrize("kind,k", KINDS)
def test_verify_many_requests_matches_oracle(kind, k):
    """Speculative verify over several channel and request groups of every
    kernel: 19 requests with ragged lengths 1..4 and accepted counts 1..4 on
    scrambled verifier slots (the accepted snapshot is often also a slot the
    step writes).  The position stamps (channel 0's last S2 column) stay as
    they were: only hyena_spec_record writes them."""
    from evo2_flash_b200 import ops

    H, B, q = 512, 19, 4
    p = random_params(kind, H, k, seed=44)
    po = params_to_oracle(p, kind, H, k)
    g = torch.Generator().manual_seed(45)
    nb = 1 + B * q
    order = (torch.randperm(nb - 1, generator=g) + 1).view(B, q)
    slots = order.tolist()
    lengths = torch.randint(1, q + 1, (B,), generator=g).tolist()
    accepted = torch.randint(1, q + 1, (B,), generator=g)
    states = _random_states(H, nb, 2 + q - 1, seed=46, spec_col=True)
    ref_states = [s.clone() for s in states]
    T = sum(lengths)
    z = (torch.randn(T, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
    meta = decode_meta(slots, lengths, computed=[100 + r for r in range(B)])
    ref = O.mixer_core(z, po, meta, ref_states, accepted, bf16_products=True)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    ds = [s.to(DEV) for s in states]
    stamps_before = ds[2][:, 0, 16].clone()
    st = torch.tensor(slots, dtype=torch.int32, device=DEV)
    qs = meta.query_start_loc_d.to(DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.decode(w, z.to(DEV), out, st[:, 0], st[:, 0], st, st, ds[0],
               ds[2] if kind == "hcl" else ds[1], token_start=qs, accepted=accepted.to(DEV))
    torch.cuda.synchronize()
    assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert torch.equal(ds[0].cpu()[1:], ref_states[0][1:])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu()[1:, :, :16], ref_states[2][1:, :, :16]) < 1e-5
        assert torch.equal(ds[2][:, 0, 16], stamps_before)
    else:
        assert torch.equal(ds[1].cpu()[1:, : k - 1], ref_states[1][1:, : k - 1])


@pytest.mark.parametrize("kind,k", [("hcm", 128), ("hcl", 16)])
def test_decode_null_block_row_is_zero_and_writes_nothing(kind, k):
    from evo2_flash_b200 import ops

    H = 128
    p = random_params(kind, H, k, seed=51)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    states = [s.to(DEV) for s in _random_states(H, 4, 2, seed=52)]
    inner = 2 if kind == "hcl" else 1
    before = [s.clone() for s in states]
    z = torch.randn(2, 3 * H, device=DEV).to(torch.bfloat16)
    out = torch.full((2, H), 7.0, dtype=torch.bfloat16, device=DEV)
    idx = torch.tensor([0, 2], dtype=torch.int32, device=DEV)
    ops.decode(w, z, out, idx, idx, idx[:, None], idx[:, None], states[0], states[inner],
               zero_null_rows=True)
    torch.cuda.synchronize()
    assert torch.all(out[0] == 0)
    assert torch.equal(states[0][0], before[0][0]) and torch.equal(states[inner][0], before[inner][0])
    assert not torch.equal(states[inner][2], before[inner][2])


@pytest.mark.parametrize("kind,k", KINDS)
def test_decode_many_requests_matches_oracle(kind, k):
    """Enough requests and channels that every kernel covers several request /
    channel groups, with the slots in scrambled order."""
    from evo2_flash_b200 import ops

    H, B = 512, 19
    p = random_params(kind, H, k, seed=34)
    po = params_to_oracle(p, kind, H, k)
    states = _random_states(H, 41, 2, seed=35)
    slots = torch.randperm(40, generator=torch.Generator().manual_seed(36))[:B].add(1).tolist()
    g = torch.Generator().manual_seed(37)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, kind)
    ds = [s.to(DEV) for s in states]
    ref_states = [s.clone() for s in states]
    for step in range(2):
        z = (torch.randn(B, 3 * H, generator=g) * 0.5).to(torch.bfloat16)
        ref = O.mixer_core(z, po, decode_meta(slots), ref_states, None, bf16_products=True)
        out = torch.empty(B, H, dtype=torch.bfloat16, device=DEV)
        idx = torch.tensor(slots, dtype=torch.int32, device=DEV)
        ops.decode(w, z.to(DEV), out, idx, idx, idx[:, None], idx[:, None], ds[0],
                   ds[2] if kind == "hcl" else ds[1], zero_null_rows=True)
        torch.cuda.synchronize()
        assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert torch.equal(ds[0].cpu(), ref_states[0])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu(), ref_states[2]) < 1e-5
    else:
        assert torch.equal(ds[1].cpu()[:, : k - 1], ref_states[1][:, : k - 1])


def test_out_of_range_block_sets_flag_without_fault():
    from evo2_flash_b200 import ops

    H = 128
    p = random_params("hcs", H, 7, seed=61)
    w = _weights({kk: v.to(DEV) for kk, v in p.items()}, "hcs")
    states = [s.to(DEV) for s in _random_states(H, 3, 2, seed=62)]
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    z = torch.randn(10, 3 * H, device=DEV).to(torch.bfloat16)
    out = torch.empty(10, H, dtype=torch.bfloat16, device=DEV)
    m = prefill_meta([10], [99], [True], device=DEV)
    ops.prefill(w, z, out, m.query_start_loc_p, m.has_initial_states_p, m.state_indices_tensor_p,
                states[0], states[1], error_flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) & 1


def test_quant_e4m3_exact():
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(71)
    x = (torch.randn(300, 512, generator=g) * 3).to(torch.bfloat16)
    x[0, :6] = torch.tensor([float("inf"), -float("inf"), float("nan"), 0.0, -0.0, 4.48])
    sx = torch.tensor([0.01], dtype=torch.float32)
    ref = O.quantize_input(x, sx)
    q = ops.quant_e4m3(x.to(DEV), sx.to(DEV))
    torch.cuda.synchronize()
    got = q.float().cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref))  # NaN stays NaN, as torch's clamp
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(ref))


def test_emulated_fp8_gemm_matches_reference_fixture():
    """The Hopper fast-accumulation model against the reference's own emulation
    output (fp8_emul.static_fp8_linear_emulated, golden fixture): bit for bit."""
    from evo2_flash_b200 import ops
    from tests.helpers import load_fixture

    fx = load_fixture("fp8_in_proj")
    w8 = fx["w8"].view(torch.float8_e4m3fn)
    w_t = w8.float().t().contiguous().to(torch.bfloat16)
    scales = torch.stack([fx["sx"].reshape(()), fx["sw"].reshape(())]).float()
    out = ops.fp8_linear_emulated(fx["x"].to(DEV), w_t.to(DEV), scales.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), fx["out_hopper"])


@pytest.mark.parametrize("N,K,M", [(200, 512, 384), (1, 4096, 128), (37, 96, 70)])
def test_emulated_fp8_gemm_matches_oracle(N, K, M):
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(N + K + M)
    x = (torch.randn(N, K, generator=g) * torch.logspace(-2, 2, K)).to(torch.bfloat16)
    x[0, :5] = 0.0
    w8 = (torch.randn(M, K, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    sx, sw = torch.tensor([0.05]), torch.tensor([0.01])
    ref = O.fp8_linear(x, w8, sx, sw, hopper=True)
    w_t = w8.float().t().contiguous().to(torch.bfloat16)
    out = ops.fp8_linear_emulated(x.to(DEV), w_t.to(DEV), torch.cat([sx, sw]).to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), ref)


def _all_finite_bf16(cols=512):
    """Every finite bf16 value once, as (rows, cols) rows (zero padded)."""
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    x = x[torch.isfinite(x)]
    pad = (-x.numel()) % cols
    return torch.cat([x, torch.zeros(pad, dtype=torch.bfloat16)]).view(-1, cols)


@pytest.mark.parametrize("sx", [0.01, 4.0 / 448.0, 1.0 / 3.0, 0.1, 2.0 ** -5, 3.3e-3, 1e-39,
                                7.5e30])
def test_quant_e4m3_every_bf16_value(sx):
    """The quantiser divides by a reciprocal multiply and falls back to the
    correctly rounded division near rounding ties: every finite bf16 value must
    give the byte of the oracle's division (1e-39 is an fp32 subnormal scale,
    which takes the division everywhere)."""
    from evo2_flash_b200 import ops

    x = _all_finite_bf16()
    s = torch.tensor([sx], dtype=torch.float32)
    ref = O.quantize_input(x, s).to(torch.float8_e4m3fn).view(torch.uint8)
    q = ops.quant_e4m3(x.to(DEV), s.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.uint8).cpu(), ref)


def _grid_rows(rows, h, seed, lim=16):
    """Multiples of 1/4 in [-lim/4, lim/4]: a row's sum of squares is exact in fp32
    in any order (up to h = 16384), so the kernel's n equals the oracle's."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(-lim, lim + 1, (rows, h), generator=g).float() / 4).to(torch.bfloat16)


def test_rms_norm_matches_reference_fixture():
    from evo2_flash_b200 import ops
    from tests.helpers import load_fixture

    fx = load_fixture("rms_norm")
    x, r, w = fx["x"].to(DEV), fx["r"].to(DEV), fx["weight"].to(DEV)
    sx = fx["sx"].reshape(1).float().to(DEV)
    y, _ = ops.rms_norm(x, w, fx["eps"])
    s = torch.empty_like(x)
    y2, q2 = ops.rms_norm(x, w, fx["eps"], r, quant_scale=sx, s_out=s)
    torch.cuda.synchronize()
    y, y2, s, q2 = y.cpu(), y2.cpu(), s.cpu(), q2.float().cpu()
    assert torch.equal(s, fx["s_add"])
    # rows 0-15: sums of squares exact in any order -> bit for bit
    assert torch.equal(y[:16], fx["y"][:16]) and torch.equal(y2[:16], fx["y_add"][:16])
    assert torch.equal(q2[:16], fx["q_add"][:16])
    # other rows: n may differ in its last bf16 bit from the reference's order
    for got, ref in ((y, fx["y"]), (y2, fx["y_add"])):
        assert max_rel_err(got, ref) < 1e-2
        assert (got == ref).float().mean() > 0.99
    same = (y2 == fx["y_add"]).all(dim=1)
    assert torch.equal(q2[same], fx["q_add"][same])


@pytest.mark.parametrize("h", [4096, 8192, 1000, 12288])
def test_rms_norm_exact_rows_with_residual_and_quant(h):
    from evo2_flash_b200 import ops

    x = _grid_rows(700, h, seed=h)
    r = _grid_rows(700, h, seed=h + 1, lim=4)
    g = torch.Generator().manual_seed(5)
    w = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)
    sx = torch.tensor([6.0 / 448.0])
    ref_y = O.rms_norm(x, w, 1e-6)
    ref_y2, ref_s = O.rms_norm(x, w, 1e-6, r)
    ref_q = O.quantize_input(ref_y2, sx)
    xd, rd, wd = x.to(DEV), r.to(DEV), w.to(DEV)
    y, none = ops.rms_norm(xd, wd, 1e-6)
    assert none is None
    # in place into the residual (vLLM's fused add-norm), y not materialised
    none, q = ops.rms_norm(xd, wd, 1e-6, rd, want_y=False, quant_scale=sx.to(DEV), s_out=rd)
    assert none is None
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), ref_y)
    assert torch.equal(rd.cpu(), ref_s)
    assert torch.equal(q.float().cpu(), ref_q)
    # in place into x, bf16 output this time
    xd2 = x.to(DEV)
    y3, _ = ops.rms_norm(xd2, wd, 1e-6, r.to(DEV), s_out=xd2)
    torch.cuda.synchronize()
    assert torch.equal(xd2.cpu(), ref_s) and torch.equal(y3.cpu(), ref_y2)


def test_rms_norm_random_rows_within_tolerance():
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(9)
    x = (torch.randn(3000, 4096, generator=g) * torch.logspace(-3, 9, 3000)[:, None]).to(
        torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    ref = O.rms_norm(x, w, 1e-6)
    y, _ = ops.rms_norm(x.to(DEV), w.to(DEV), 1e-6)
    torch.cuda.synchronize()
    y = y.cpu()
    assert max_rel_err(y, ref) < 1e-2
    assert (y == ref).float().mean() > 0.99


def test_rms_norm_rejects_bad_arguments():
    from evo2_flash_b200 import ops

    x = torch.zeros(4, 4096, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(4096, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        ops.rms_norm(x, w[:100], 1e-6)
    with pytest.raises(ValueError):
        ops.rms_norm(x, w, 1e-6, want_y=False)
    with pytest.raises(ValueError):  # H above the kernel's 16384
        ops.rms_norm(torch.zeros(2, 16392, dtype=torch.bfloat16, device=DEV),
                     torch.ones(16392, dtype=torch.bfloat16, device=DEV), 1e-6)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 384, 512), (1000, 768, 256),
                                   (4096, 12288, 4096), (128, 12288, 4096), (1024, 4096, 4096),
                                   (7, 4096, 256), (512, 12288, 4096), (500, 12288, 1024),
                                   (4224, 776, 256), (8192, 12288, 512)])
def test_gemm_e4m3(M, N, K):
    """(512 | 500, 12288): 192-wide persistent tiles (the q = 4 verify in_proj);
    M >= 4096: 256 x 256 tiles on SM pairs, with row and column tails (4224 x 776)."""
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(M + N)
    a = (torch.randn(M, K, generator=g) * 4).to(torch.float8_e4m3fn)
    b = (torch.randn(N, K, generator=g) * 4).to(torch.float8_e4m3fn)
    sa = torch.tensor([0.02], dtype=torch.float32)
    sb = torch.tensor([0.003], dtype=torch.float32)
    da, db = a.to(DEV), b.to(DEV)
    out = ops.gemm_e4m3(da, db, sa.to(DEV), sb.to(DEV))
    ref = ((da.float() @ db.float().t()) * sa.to(DEV) * sb.to(DEV)).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert max_rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 384, 512), (1000, 776, 192),
                                   (4096, 4096, 4096), (128, 4096, 4096), (256, 4096, 4096),
                                   (5, 4104, 128), (4200, 4104, 128)])
def test_gemm_bf16_bias(M, N, K):
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(M * 3 + N)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    b = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    bias = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV)
    out = ops.gemm_bf16(a, b, bias)
    ref = (a.float() @ b.float().t() + bias.float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert max_rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("fp8", [True, False])
@pytest.mark.parametrize("M", [128, 61, 300])
def test_small_m_gemm_cluster_split_k_is_deterministic(fp8, M):
    """Decode-sized GEMMs split K over the CTAs of a cluster and sum the slices
    over DSMEM in a fixed order: they need no workspace, match torch, and two
    calls give bitwise-identical results."""
    from evo2_flash_b200 import _lib, ops

    N, K = (12288, 4096) if fp8 else (4096, 4096)
    g = torch.Generator().manual_seed(81 + M)
    if fp8:
        a = (torch.randn(M, K, generator=g) * 4).to(torch.float8_e4m3fn).to(DEV)
        b = (torch.randn(N, K, generator=g) * 4).to(torch.float8_e4m3fn).to(DEV)
        sa = torch.tensor([0.02], device=DEV)
        sb = torch.tensor([0.003], device=DEV)
        ref = ((a.float() @ b.float().t()) * sa * sb).to(torch.bfloat16)
        run = lambda: ops.gemm_e4m3(a, b, sa, sb)  # noqa: E731
    else:
        a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
        b = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
        bias = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV)
        ref = (a.float() @ b.float().t() + bias.float()).to(torch.bfloat16)
        run = lambda: ops.gemm_bf16(a, b, bias)  # noqa: E731
    assert _lib.load().hyena_gemm_workspace_size(M, N, K, int(fp8)) == 0
    first, second = run(), run()
    torch.cuda.synchronize()
    assert max_rel_err(first, ref) < 1e-2
    assert torch.equal(first, second)


def test_gemm_barrier_waits_never_expired():
    """The GEMMs bound every shared-memory barrier wait and count expiries in a
    device counter; after every GEMM above (and one more of each kind here) the
    counter, read back through hyena_gemm_wait_timeouts, is zero."""
    from evo2_flash_b200 import ops

    a = torch.randn(512, 1024, device=DEV).to(torch.bfloat16)
    b = torch.randn(768, 1024, device=DEV).to(torch.bfloat16)
    ops.gemm_bf16(a, b)
    sc = torch.ones(1, device=DEV)
    ops.gemm_e4m3(a.to(torch.float8_e4m3fn), b.to(torch.float8_e4m3fn), sc, sc)
    torch.cuda.synchronize()
    assert ops.gemm_wait_timeouts() == 0
    ops.check_gemm_waits()


def test_spec_bookkeeping_matches_the_stamp_rules():
    """hyena_spec_accepted / hyena_spec_record against the reference's torch
    rules (mixers.py:962-984, 1040-1062) on random stamps: accepted = clamp(
    computed - stamp(first slot), 0, num_spec) + 1; stamps of the active verifier
    slots = computed + p + 1; a mismatching non-null stamp sets the flag."""
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(91)
    nb, R, q, ns = 64, 9, 4, 3
    s2 = torch.zeros(nb, 8, 17)
    s2[:, 0, 16] = torch.randint(0, 1000, (nb,), generator=g).float()
    slots = torch.randperm(nb - 1, generator=g)[: R * q].add(1).view(R, q).int()
    slots[2, 0] = 0  # a null first slot
    stamp_first = s2[slots[:, 0].long(), 0, 16]
    offs = torch.randint(0, ns + 1, (R,), generator=g)
    computed = (stamp_first + offs).int()
    ds2 = s2.to(DEV)
    stamps = ds2[:, 0, 16]
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    acc = ops.spec_accepted(slots.to(DEV), computed.to(DEV), stamps, ns, error_flags=flags)
    want = (computed.long() - stamp_first.long()).clamp(0, ns) + 1
    torch.cuda.synchronize()
    assert torch.equal(acc.cpu().long(), want)
    assert int(flags.item()) == 0
    bad = computed.clone()
    bad[0] += 50  # offset beyond num_spec on a non-null slot
    ops.spec_accepted(slots.to(DEV), bad.to(DEV), stamps, ns, error_flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) & 4

    lens = torch.tensor([4, 2, 1, 3, 4, 1, 2, 4, 3])
    starts = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)]).int()
    ops.spec_record(slots.to(DEV), starts.to(DEV), computed.to(DEV), stamps)
    ref = s2[:, 0, 16].clone()
    for r in range(R):
        for p in range(int(lens[r])):
            b = int(slots[r, p])
            if b:
                ref[b] = float(int(computed[r]) + p + 1)
    torch.cuda.synchronize()
    got = ds2[:, 0, 16].cpu()
    assert torch.equal(got[1:], ref[1:])


def test_state_repair_copies_stale_prefill_blocks():
    """hyena_state_repair against the rule of mixers.py:1001-1037, restated on
    the host: a resumed prefill row whose block is not stamped with its
    computed-token count takes every state slice of its source block when
    that one is; fresh rows, null blocks and consistent rows are untouched.
    hyena_spec_record_prefill then stamps the prefill blocks."""
    from evo2_flash_b200 import ops

    g = torch.Generator().manual_seed(93)
    nb, H, W0 = 24, 128, 5
    states = [torch.randn(nb, W0, 3 * H, generator=g).to(torch.bfloat16),
              torch.randn(nb, 127, H, generator=g), torch.randn(nb, H, 17, generator=g)]
    states[2][:, 0, 16] = torch.randint(0, 50, (nb,), generator=g).float()
    stamps = states[2][:, 0, 16]
    dst = torch.tensor([3, 4, 5, 6, 7, 0, 8], dtype=torch.int32)
    src = torch.tensor([10, 11, 12, 0, 13, 14, 15], dtype=torch.int32)
    init = torch.tensor([True, True, False, True, True, True, True])
    computed = stamps[src.long()].int().clone()
    computed[1] = int(stamps[11]) + 1          # source stamp wrong: no copy
    stamps[8] = float(computed[6])             # destination already right: no copy
    want = [s.clone() for s in states]
    bad = (init & (stamps[dst.long()] != computed.float()) & (stamps[src.long()] == computed.float())
           & (src != 0) & (dst != 0))
    for j in range(len(dst)):
        if bad[j]:
            for w in want:
                w[dst[j]] = w[src[j]]
    assert bad.tolist() == [True, False, False, False, True, False, False]
    ds = [s.to(DEV) for s in states]
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    take = ops.state_repair(dst.to(DEV), src.to(DEV), computed.to(DEV), init.to(DEV),
                            ds[2][:, 0, 16], ds, error_flags=flags)
    torch.cuda.synchronize()
    assert take.cpu().tolist() == [10, -1, -1, -1, 13, -1, -1]
    for a, b in zip(ds, want):
        assert torch.equal(a.cpu(), b)
    lens = torch.tensor([60, 61, 62, 63, 64, 65, 66], dtype=torch.int32)
    ops.spec_record_prefill(dst.to(DEV), lens.to(DEV), ds[2][:, 0, 16], error_flags=flags)
    torch.cuda.synchronize()
    got = ds[2][:, 0, 16].cpu()
    for j in range(len(dst)):
        if int(dst[j]):
            assert got[int(dst[j])] == float(lens[j])
    assert int(flags.item()) == 0
