"""Torch-facing launchers of the sm_100a Hyena kernels.

Each function validates shapes and dtypes on the host (ValueError, as the
reference's launchers do, mixers.py:479-509), builds the C-ABI argument structs
from tensor pointers and strides, and launches on the current CUDA stream.
Nothing here synchronises with the device, so all of it is CUDA-graph capturable
given fixed shapes (the HCL prefill workspace is the one allocation, made through
torch's caching allocator).

Kernel-side layouts:
  conv_state   (blocks, W0, 3H) bf16 view in vLLM's SD orientation (any strides)
  inner_state  FIR: (blocks, >=K-1, H) fp32 view; IIR: (blocks, H, >=16) fp32
  weights      LayerWeights, built once per layer by `layer_weights`
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DecodeArgs, LayerParams, PrefillArgs, StateView

BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _require(cond, msg):
    if not cond:
        raise ValueError(msg)


def _cuda(t, name):
    _require(t.is_cuda, f"{name} must be a CUDA tensor")


@dataclass
class LayerWeights:
    """Device tensors of one Hyena layer in the layout the kernels read.

    kind: "fir" or "iir". short_w (3H, 3) bf16 contiguous. FIR: inner_w_t (K, H)
    bf16 contiguous (the (H, K) taps transposed, so a warp reads consecutive
    channels of one tap). IIR: log_poles / residues (H, 16) fp32. D (H,) bf16 or None.
    """

    kind: str
    H: int
    K: int
    short_w: torch.Tensor
    inner_w_t: torch.Tensor | None = None
    log_poles: torch.Tensor | None = None
    residues: torch.Tensor | None = None
    D: torch.Tensor | None = None

    def params(self) -> LayerParams:
        p = LayerParams()
        p.kind = _lib.HYENA_KIND_FIR if self.kind == "fir" else _lib.HYENA_KIND_IIR
        p.H, p.K = self.H, self.K
        p.short_w = self.short_w.data_ptr()
        if self.kind == "fir":
            p.inner_w = self.inner_w_t.data_ptr()
            p.inner_w_stride_h = self.inner_w_t.stride(1)
            p.inner_w_stride_k = self.inner_w_t.stride(0)
        else:
            p.log_poles = self.log_poles.data_ptr()
            p.lp_stride_h, p.lp_stride_s = self.log_poles.stride()
            p.residues = self.residues.data_ptr()
            p.res_stride_h, p.res_stride_s = self.residues.stride()
        p.D = None if self.D is None else self.D.data_ptr()
        return p


def layer_weights(kind, short_filter, conv=None, D=None, log_poles=None, residues=None):
    """LayerWeights from checkpoint-layout parameters (mixers.py:805, 1247-1250,
    1323-1325): short_filter (3H,1,3), conv (H,1,K), D (H,), log_poles (H,S,1),
    residues (H,S)."""
    H = short_filter.shape[0] // 3
    short_w = short_filter.detach().reshape(3 * H, 3).to(BF16).contiguous()
    Dd = None if D is None else D.detach().to(BF16).contiguous()
    if kind == "fir":
        K = conv.shape[-1]
        inner = conv.detach().reshape(H, K).to(BF16).t().contiguous()
        return LayerWeights("fir", H, K, short_w, inner_w_t=inner, D=Dd)
    lp = log_poles.detach().reshape(H, -1).float().contiguous()
    res = residues.detach().reshape(H, -1).float().contiguous()
    return LayerWeights("iir", H, lp.shape[1], short_w, log_poles=lp, residues=res, D=Dd)


def state_view(t, cols_dim, chan_dim, cols=None) -> StateView:
    """A hyena_state_view over a (blocks, ...) tensor: `cols_dim` indexes window
    columns (or modes), `chan_dim` channels."""
    v = StateView()
    v.data = t.data_ptr()
    v.block_stride = t.stride(0)
    v.col_stride = t.stride(cols_dim)
    v.dim_stride = t.stride(chan_dim)
    v.cols = t.shape[cols_dim] if cols is None else cols
    v.num_blocks = t.shape[0]
    return v


def _check_states(w, conv_state, inner_state):
    _require(conv_state.dtype == BF16 and conv_state.dim() == 3 and conv_state.shape[2] == 3 * w.H,
             f"conv_state must be (blocks, W0, 3H) bf16, got {tuple(conv_state.shape)} {conv_state.dtype}")
    _require(conv_state.shape[1] >= 2, "conv_state needs at least 2 window columns")
    _require(inner_state.dtype == torch.float32 and inner_state.dim() == 3,
             "inner_state must be a 3-D fp32 tensor")
    if w.kind == "fir":
        _require(inner_state.shape[2] == w.H and inner_state.shape[1] >= w.K - 1,
                 f"FIR inner_state must be (blocks, >={w.K - 1}, H), got {tuple(inner_state.shape)}")
    else:
        _require(inner_state.shape[1] == w.H and inner_state.shape[2] >= w.K,
                 f"LI state must be (blocks, H, >={w.K}), got {tuple(inner_state.shape)}")


def _inner_view(w, inner_state):
    if w.kind == "fir":
        return state_view(inner_state, 1, 2, cols=w.K - 1)
    return state_view(inner_state, 2, 1, cols=w.K)


def _i32(t, name):
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    _cuda(t, name)
    return t


def prefill(w: LayerWeights, z, out, query_start_loc, has_initial_state, state_indices,
            conv_state, inner_state, error_flags=None):
    """Fused prefill core over packed rows: z (T, 3H) bf16 -> out (T, H) bf16.

    query_start_loc (n+1,) int32 segment offsets relative to z's first row;
    has_initial_state (n,) bool or None; state_indices (n,) int (any stride).
    """
    _require(z.dim() == 2 and z.shape[1] == 3 * w.H and z.dtype == BF16 and z.stride(1) == 1,
             f"z must be (T, 3H) bf16 with unit column stride, got {tuple(z.shape)}")
    _require(out.dim() == 2 and out.shape[1] == w.H and out.dtype == BF16 and out.stride(1) == 1,
             "out must be (T, H) bf16 with unit column stride")
    _require(out.shape[0] >= z.shape[0], "out has fewer rows than z")
    _cuda(z, "z")
    _check_states(w, conv_state, inner_state)
    n = state_indices.shape[0]
    _require(query_start_loc.numel() >= n + 1, "query_start_loc too short")
    qsl = _i32(query_start_loc[: n + 1].contiguous(), "query_start_loc")
    idx = _i32(state_indices, "state_indices")
    flags = None
    if has_initial_state is not None:
        flags = has_initial_state[:n]
        flags = (flags if flags.dtype == torch.bool else flags != 0).contiguous().view(torch.uint8)
    a = PrefillArgs()
    a.z, a.ldz = z.data_ptr(), z.stride(0)
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.T = z.shape[0]
    a.num_segments = n
    a.query_start_loc = qsl.data_ptr()
    a.has_initial_state = None if flags is None else flags.data_ptr()
    a.state_indices = idx.data_ptr()
    a.state_indices_stride = idx.stride(0) if idx.dim() else 1
    a.conv_state = state_view(conv_state, 1, 2)
    a.inner_state = _inner_view(w, inner_state)
    a.error_flags = None if error_flags is None else error_flags.data_ptr()
    lib = _lib.load()
    p = w.params()
    ws_bytes = lib.hyena_prefill_workspace_size(C.byref(p), a.T, n)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=z.device) if ws_bytes else None
    # keep the temporaries alive until the launch returned
    _keep = (qsl, idx, flags, ws)
    _lib.check(lib.hyena_prefill(C.byref(p), C.byref(a), _ptr(ws), C.c_size_t(ws_bytes), _stream()),
               "hyena_prefill")
    del _keep
    return out


def decode(w: LayerWeights, z, out, conv_in_block, conv_out_block, in_slots, out_slots,
           conv_state, inner_state, token_start=None, accepted=None, zero_null_rows=False,
           skip_null_writes=True, null_block=0, error_flags=None):
    """Fused decode / speculative verify: z (tokens, 3H) -> out (tokens, H).

    conv_in_block / conv_out_block (B,) int; in_slots / out_slots (B, q) int
    (q = 1 for ordinary decode); token_start (B+1,) int or None (one token per
    request); accepted (B,) int (a count below 1 reads as 1) or None.
    """
    B = conv_in_block.shape[0]
    _require(z.dim() == 2 and z.shape[1] == 3 * w.H and z.dtype == BF16 and z.stride(1) == 1,
             "z must be (tokens, 3H) bf16")
    _require(out.dim() == 2 and out.shape[1] == w.H and out.dtype == BF16 and out.stride(1) == 1,
             "out must be (tokens, H) bf16")
    _check_states(w, conv_state, inner_state)
    _require(in_slots.dim() == 2 and out_slots.dim() == 2 and in_slots.shape[0] >= B
             and out_slots.shape[0] >= B, "slot tables must be (B, q)")
    q = out_slots.shape[1]
    _require(1 <= q <= 8, f"at most 8 positions per request, got {q}")
    if B == 0:
        return out
    cin = _i32(conv_in_block, "conv_in_block")
    cout = _i32(conv_out_block, "conv_out_block")
    if cin.dim() != 1 or cin.stride(0) < 1:
        cin = cin.contiguous().view(-1)
    if cout.dim() != 1 or cout.stride(0) < 1:
        cout = cout.contiguous().view(-1)
    ins = _i32(in_slots, "in_slots")
    outs = _i32(out_slots, "out_slots")
    ts = None if token_start is None else _i32(token_start[: B + 1], "token_start").contiguous()
    acc = None if accepted is None else _i32(accepted[:B], "accepted").contiguous()
    a = DecodeArgs()
    a.z, a.ldz = z.data_ptr(), z.stride(0)
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.num_reqs, a.q = B, q
    a.token_start = None if ts is None else ts.data_ptr()
    a.accepted = None if acc is None else acc.data_ptr()
    a.conv_in_block, a.conv_out_block = cin.data_ptr(), cout.data_ptr()
    a.conv_in_stride, a.conv_out_stride = cin.stride(0), cout.stride(0)
    a.in_slots, a.in_stride0, a.in_stride1 = ins.data_ptr(), ins.stride(0), ins.stride(1)
    a.out_slots, a.out_stride0, a.out_stride1 = outs.data_ptr(), outs.stride(0), outs.stride(1)
    a.zero_null_rows = int(bool(zero_null_rows))
    a.skip_null_writes = int(bool(skip_null_writes))
    a.null_block = int(null_block)
    a.conv_state = state_view(conv_state, 1, 2)
    a.inner_state = _inner_view(w, inner_state)
    a.error_flags = None if error_flags is None else error_flags.data_ptr()
    lib = _lib.load()
    p = w.params()
    _keep = (cin, cout, ins, outs, ts, acc)
    _lib.check(lib.hyena_decode(C.byref(p), C.byref(a), _stream()), "hyena_decode")
    del _keep
    return out


def quant_e4m3(x, input_scale, out=None):
    """q = e4m3(clamp(x / sx, +-448)) (fp8_emul.py:76-78). x (M, K) bf16 -> (M, K) e4m3."""
    _require(x.dim() == 2 and x.dtype == BF16 and x.stride(1) == 1, "x must be (M, K) bf16")
    _require(input_scale.dtype == torch.float32 and input_scale.numel() == 1,
             "input_scale must be one fp32 element")
    M, K = x.shape
    if out is None:
        out = torch.empty(M, K, dtype=E4M3, device=x.device)
    lib = _lib.load()
    _lib.check(lib.hyena_quant_e4m3(_ptr(x), x.stride(0), _ptr(out), out.stride(0), M, K,
                                    _ptr(input_scale), _stream()), "hyena_quant_e4m3")
    return out


def gemm_fp8_emulated(a, w_t, scale_a, scale_b, out=None):
    """out (N, M) bf16 = Hopper fast-accumulation model of a (N, K) e4m3 . w_t (K, M)
    (bf16 holding E4M3 values), scaled by sa then sb (fp8_emul.py:45-88)."""
    _cuda(a, "a")
    _require(a.dtype == E4M3 and a.dim() == 2 and a.stride(1) == 1, "a must be (N, K) e4m3 rows")
    _require(w_t.dtype == BF16 and w_t.dim() == 2 and w_t.stride(1) == 1 and
             w_t.shape[0] == a.shape[1], "w_t must be (K, M) bf16 rows")
    N, K = a.shape
    M = w_t.shape[1]
    if out is None:
        out = torch.empty(N, M, dtype=BF16, device=a.device)
    lib = _lib.load()
    _lib.check(lib.hyena_gemm_fp8_emulated(_ptr(a), a.stride(0), _ptr(w_t), w_t.stride(0),
                                           _ptr(out), out.stride(0), N, M, K, _ptr(scale_a),
                                           _ptr(scale_b), _stream()), "hyena_gemm_fp8_emulated")
    return out


def fp8_linear_emulated(x, w_t, scales):
    """The FP8-surgery projection without FP8 hardware (mixers.py:701-705,
    fp8_emul_triton.py:181-191): q(x) with the static input scale scales[0],
    then the fast-accumulation model against w_t (K, M), times scales[0] * scales[1]."""
    _require(scales.dtype == torch.float32 and scales.numel() == 2, "scales must be 2 fp32")
    sx, sw = scales[0:1], scales[1:2]
    x2 = x.reshape(-1, x.shape[-1])
    q = quant_e4m3(x2.contiguous(), sx)
    return gemm_fp8_emulated(q, w_t, sx, sw).reshape(*x.shape[:-1], w_t.shape[1])


def rms_norm(x, weight, eps, residual=None, *, want_y=True, quant_scale=None, s_out=None):
    """Evo2RMSNorm of the decoder layer (model.py:47-76 Evo2RMSNorm.forward;
    triton_norm.py:127-156 rms_norm), one pass over the rows of x (M, H) bf16:

      s = x + residual (bf16), written to s_out (which may be x or residual:
          vLLM's in-place fused add-norm);
      y = weight * s / (||s||_2 * H^-0.5 + eps) with torch's bf16 roundings;
      q = e4m3(clamp(y / quant_scale, +-448)) when quant_scale is given.

    Returns (y or None, q or None).  want_y=False with quant_scale skips the
    bf16 output entirely (the in_proj input of a Hyena layer)."""
    _cuda(x, "x")
    _require(x.dim() == 2 and x.dtype == BF16 and x.stride(1) == 1, "x must be (M, H) bf16 rows")
    M, H = x.shape
    _require(weight.dtype == BF16 and weight.numel() == H and weight.is_contiguous(),
             "weight must be (H,) bf16")
    if residual is not None:
        _require(residual.shape == x.shape and residual.dtype == BF16 and residual.stride(1) == 1,
                 "residual must match x")
    if s_out is not None:
        _require(s_out.shape == x.shape and s_out.dtype == BF16 and s_out.stride(1) == 1,
                 "s_out must match x")
    if quant_scale is not None:
        _require(quant_scale.dtype == torch.float32 and quant_scale.numel() == 1,
                 "quant_scale must be one fp32 element")
    _require(want_y or quant_scale is not None or s_out is not None, "no output requested")
    y = torch.empty(M, H, dtype=BF16, device=x.device) if want_y else None
    q = torch.empty(M, H, dtype=E4M3, device=x.device) if quant_scale is not None else None
    lib = _lib.load()
    ld = lambda t: t.stride(0) if t is not None else 0  # noqa: E731
    _lib.check(lib.hyena_rms_norm(
        _ptr(x), x.stride(0), _ptr(residual), ld(residual), _ptr(weight), float(eps),
        _ptr(s_out), ld(s_out), _ptr(y), ld(y), _ptr(q), ld(q), _ptr(quant_scale), M, H,
        _stream()), "hyena_rms_norm")
    return y, q


def gemm_e4m3(a, b, scale_a, scale_b, out=None):
    """out (M, N) bf16 = (a (M,K) e4m3 . b (N,K) e4m3^T) * sa * sb (tcgen05)."""
    _require(a.dtype == E4M3 and b.dtype == E4M3, "e4m3 operands expected")
    _require(a.dim() == 2 and b.dim() == 2 and a.shape[1] == b.shape[1], "shape mismatch")
    _require(a.stride(1) == 1 and b.stride(1) == 1, "operands must be K-contiguous")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=BF16, device=a.device)
    lib = _lib.load()
    ws = _gemm_workspace(lib, M, N, K, True, a.device)
    _lib.check(lib.hyena_gemm_e4m3(_ptr(a), a.stride(0), _ptr(b), b.stride(0), _ptr(out),
                                   out.stride(0), M, N, K, _ptr(scale_a), _ptr(scale_b),
                                   _ptr(ws), C.c_size_t(0 if ws is None else ws.numel() * 4),
                                   _stream()), "hyena_gemm_e4m3")
    return out


def gemm_wait_timeouts(reset: bool = False) -> int:
    """Expired shared-memory barrier waits in the GEMMs on the current device
    since the last reset (hyena_gemm_wait_timeouts; synchronous).  Non-zero
    means some GEMM output was written from an incomplete tile."""
    n = C.c_int32(0)
    _lib.check(_lib.load().hyena_gemm_wait_timeouts(C.byref(n), int(bool(reset))),
               "hyena_gemm_wait_timeouts")
    return int(n.value)


def check_gemm_waits() -> None:
    """Raises RuntimeError when any GEMM wait expired on the current device."""
    n = gemm_wait_timeouts()
    if n:
        raise RuntimeError(f"{n} GEMM shared-memory barrier wait(s) expired: "
                           "GEMM outputs of this process are unreliable")


def set_gemm_max_ctas(n: int) -> None:
    """Caps the CTAs of the large-M GEMMs (0: one per SM) so that collectives
    running on another stream find free SMs (hyena_set_gemm_max_ctas)."""
    _lib.load().hyena_set_gemm_max_ctas(int(n))


def _stamp_view(stamps):
    """(base pointer, element stride) of a 1-D fp32 stamp view (one per block)."""
    _require(stamps.dim() == 1 and stamps.dtype == torch.float32, "stamps must be a 1-D fp32 view")
    return stamps.data_ptr(), stamps.stride(0)


def spec_accepted(slots, computed, stamps, num_spec, out=None, error_flags=None):
    """accepted (R,) int32 = clamp(computed - stamp(slots[:, 0]), 0, num_spec) + 1
    (hyena_spec_accepted; mixers.py:962-984).  slots (R,) or (R, S) int32."""
    lib = _lib.load()
    first = slots if slots.dim() == 1 else slots[:, 0]
    first = _i32(first, "slots")
    comp = _i32(computed[: first.shape[0]].contiguous(), "computed")
    R = first.shape[0]
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=first.device)
    base, stride = _stamp_view(stamps)
    _lib.check(lib.hyena_spec_accepted(first.data_ptr(), first.stride(0) if R else 1, R,
                                       comp.data_ptr(), base, stride, stamps.shape[0], int(num_spec),
                                       out.data_ptr(), _ptr(error_flags), _stream()),
               "hyena_spec_accepted")
    return out


def spec_record(out_slots, starts, computed, stamps, error_flags=None):
    """stamp(out_slots[r, p]) = computed[r] + p + 1 for the active positions p of
    each request (hyena_spec_record; mixers.py:1040-1062)."""
    lib = _lib.load()
    slots = _i32(out_slots if out_slots.dim() == 2 else out_slots[:, None], "out_slots")
    R, q = slots.shape
    st = _i32(starts[: R + 1].contiguous(), "starts")
    comp = _i32(computed[:R].contiguous(), "computed")
    base, stride = _stamp_view(stamps)
    _lib.check(lib.hyena_spec_record(slots.data_ptr(), slots.stride(0), slots.stride(1), R, q,
                                     st.data_ptr(), comp.data_ptr(), base, stride, stamps.shape[0],
                                     _ptr(error_flags), _stream()), "hyena_spec_record")


def spec_record_prefill(blocks, seq_lens, stamps, error_flags=None):
    """stamp(blocks[j]) = seq_lens[j] (hyena_spec_record_prefill;
    mixers.py:1070-1074).  blocks (n,) int (any stride), seq_lens (n,) int."""
    n = blocks.shape[0]
    if n == 0:
        return
    b = _i32(blocks, "blocks")
    lens = _i32(seq_lens[:n].contiguous(), "seq_lens")
    base, stride = _stamp_view(stamps)
    _lib.check(_lib.load().hyena_spec_record_prefill(
        b.data_ptr(), b.stride(0), n, lens.data_ptr(), base, stride, stamps.shape[0],
        _ptr(error_flags), _stream()), "hyena_spec_record_prefill")


def _block_slice(t):
    """A StateBlock over a paged (blocks, ...) tensor whose blocks are contiguous."""
    from ._lib import StateBlock

    inner = t[0] if t.shape[0] else t
    _require(inner.is_contiguous(), "state blocks must be contiguous within a block")
    sb = StateBlock()
    sb.data = t.data_ptr()
    sb.block_stride_bytes = t.stride(0) * t.element_size()
    sb.block_bytes = inner.numel() * t.element_size()
    return sb


def state_repair(dst_blocks, src_blocks, computed, has_init, stamps, states, error_flags=None):
    """Prefix-caching repair of resumed prefill rows (hyena_state_repair;
    mixers.py:1001-1037): where a row's destination block is not stamped with
    its computed-token count but its source block is, the source block's whole
    state (every tensor of `states`, each (blocks, ...)) is copied over the
    destination.  Returns the (n,) int32 decision (source block or -1)."""
    from ._lib import StateBlock

    n = dst_blocks.shape[0]
    take = torch.empty(max(n, 1), dtype=torch.int32, device=stamps.device)
    if n == 0:
        return take[:0]
    dst = _i32(dst_blocks, "dst_blocks")
    src = _i32(src_blocks[:n].contiguous(), "src_blocks")
    comp = _i32(computed[:n].contiguous(), "computed")
    init = has_init[:n]
    init = (init if init.dtype == torch.bool else init != 0).contiguous().view(torch.uint8)
    arr = (StateBlock * len(states))(*[_block_slice(t) for t in states])
    base, stride = _stamp_view(stamps)
    _lib.check(_lib.load().hyena_state_repair(
        n, dst.data_ptr(), dst.stride(0), src.data_ptr(), comp.data_ptr(), init.data_ptr(), base,
        stride, stamps.shape[0], arr, len(states), take.data_ptr(), _ptr(error_flags), _stream()),
        "hyena_state_repair")
    return take[:n]


def set_launch_chaining(enable: bool) -> None:
    """Programmatic dependent launch between this library's kernels on/off
    (hyena_set_launch_chaining; on by default)."""
    _lib.load().hyena_set_launch_chaining(int(bool(enable)))


def _gemm_workspace(lib, M, N, K, fp8, device):
    """Workspace the library asks for at this shape (none at present: small-M
    GEMMs reduce their K slices inside a thread-block cluster)."""
    n = lib.hyena_gemm_workspace_size(M, N, K, int(fp8))
    return torch.empty(n // 4, dtype=torch.float32, device=device) if n else None


def gemm_bf16(a, b, bias=None, out=None):
    """out (M, N) bf16 = a (M,K) bf16 . b (N,K) bf16^T [+ bias] (tcgen05)."""
    _require(a.dtype == BF16 and b.dtype == BF16, "bf16 operands expected")
    _require(a.dim() == 2 and b.dim() == 2 and a.shape[1] == b.shape[1], "shape mismatch")
    _require(a.stride(1) == 1 and b.stride(1) == 1, "operands must be K-contiguous")
    _require(bias is None or (bias.dtype == BF16 and bias.numel() == b.shape[0]), "bias must be (N,) bf16")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=BF16, device=a.device)
    lib = _lib.load()
    ws = _gemm_workspace(lib, M, N, K, False, a.device)
    _lib.check(lib.hyena_gemm_bf16(_ptr(a), a.stride(0), _ptr(b), b.stride(0), _ptr(out),
                                   out.stride(0), M, N, K, _ptr(bias), _ptr(ws),
                                   C.c_size_t(0 if ws is None else ws.numel() * 4), _stream()),
               "hyena_gemm_bf16")
    return out
