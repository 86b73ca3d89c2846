"""CPU restatement of the evo2_flash Hyena-mixer hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker the GPU kernels are compared against. It is imported
only by `tests/`, `__graft_entry__.smoke()` and the CPU-baseline legs of
`bench.py`; the product path (`evo2_flash_b200`) never calls it.

Every function restates the reference algorithm on CPU tensors, citing the
reference file:line it follows (paths relative to the evo2_flash project):

  short K=3 FIR, prefill ........ vLLM causal_conv1d_fn; torch twin mixers.py:350-383
  short K=3 FIR, decode/verify .. vLLM causal_conv1d_update (window convention
                                  mixers.py:227-237; rounding triton_decode.py:43-53)
  inner FIR prefill ............. mixers.py:350-383 (+ gate order 1293-1302)
  LI segment .................... mixers.py:144-210 (+ gate order 1356-1397)
  decode / verify snapshots ..... mixers.py:555-663
  fp8 projection ................ fp8_emul.py:45-88
  decoder-layer norm ............ model.py:47-76 (Evo2RMSNorm, + residual add)
  mixer forward ................. mixers.py:1277-1305 (FIR), 1327-1401 (LI)

Pinning: `tests/golden/make_golden.py` runs the reference itself (its own CPU
torch paths, with vLLM's Triton-only K=3 decode update replaced by
`conv_update` below) and `tests/test_oracle_golden.py` checks this module
against those fixtures.

State layout (vLLM's SD orientation, mixers.py:940-949): conv state
(blocks, W0, 3H) bf16; inner FIR state (blocks, 127, H) fp32; LI state
(blocks, H, 16[+1]) fp32.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

E4M3 = torch.float8_e4m3fn
FP8_MAX = 448.0


def _bf(x):
    return x.to(torch.bfloat16).float()


# ---------------------------------------------------------------- segments
def segments(meta):
    """(start, end, has_initial_state, block) per prefill segment, host ints."""
    qsl = meta.query_start_loc_p.tolist()
    flags = meta.has_initial_states_p
    flags = [False] * meta.num_prefills if flags is None else [bool(f) for f in flags.tolist()]
    blocks = meta.state_indices_tensor_p
    blocks = blocks.tolist()
    return [(qsl[j], qsl[j + 1], flags[j], int(blocks[j])) for j in range(meta.num_prefills)]


# ---------------------------------------------------------------- short K=3 FIR
def short_fir_prefill(z_p, w, meta, conv_state, bf16_products=True):
    """K=3 causal cross-correlation per prefill segment with cached left context.

    z_p (T, 3H) bf16, w (3H, 3) bf16, conv_state (blocks, W0, 3H) bf16.  The left
    context is window columns 0..1 and the last two inputs are written back there
    (mixers.py:374, 382: the first K_short-1 columns of the dim-first view); any
    speculative columns 2..W0-1 are left untouched.  With the ordinary W0 = 2 this
    is exactly vLLM causal_conv1d_fn's update.
    bf16_products: round each tap product to bf16 before the fp32 sum, as the
    GPU kernel the reference runs does (triton_decode.py:10-12).
    """
    T, C = z_p.shape
    out = torch.empty_like(z_p)
    wf = w.float()
    for a, b, init, blk in segments(meta):
        if b <= a:
            continue
        seq = z_p[a:b].float()                                   # (L, C)
        hist = conv_state[blk, :2].float() if init else torch.zeros(2, C)
        ext = torch.cat([hist, seq], 0)                          # (2 + L, C)
        x0, x1, x2 = ext[:-2], ext[1:-1], ext[2:]
        if bf16_products:
            acc = torch.zeros_like(seq)
            acc = acc + _bf(x0 * wf[:, 0])
            acc = acc + _bf(x1 * wf[:, 1])
            acc = acc + _bf(x2 * wf[:, 2])
        else:
            acc = x0 * wf[:, 0] + x1 * wf[:, 1] + x2 * wf[:, 2]
        out[a:b] = acc.to(z_p.dtype)
        conv_state[blk, :2] = ext[-2:].to(conv_state.dtype)
    return out


def conv_update(z_d, w, conv_state, meta, accepted=None, bf16_products=True):
    """vLLM causal_conv1d_update for K=3, ordinary or speculative.

    Request r reads its window from block state_indices_tensor_d[r, 0] at column
    offset accepted[r]-1, runs its tokens [qsl_d[r], qsl_d[r+1]) through the
    filter, and stores [window[off+1 : off+1+W0-n], x_0 .. x_{n-1}] back
    (window convention restated in mixers.py:227-237).  Columns past the window
    read as zero.  Returns (tokens, 3H) bf16.
    """
    slots = meta.state_indices_tensor_d
    if slots.dim() == 1:
        slots = slots[:, None]
    nreq = int(meta.num_decodes)
    qsl = getattr(meta, "query_start_loc_d", None)
    starts = list(range(nreq + 1)) if qsl is None else qsl[: nreq + 1].tolist()
    acc_list = [1] * nreq if accepted is None else accepted[:nreq].tolist()
    W0 = conv_state.shape[1]
    wf = w.float()
    out = torch.zeros_like(z_d)
    for r in range(nreq):
        t0, t1 = starts[r], starts[r + 1]
        n = t1 - t0
        if n <= 0:
            continue
        blk = int(slots[r, 0])
        off = int(acc_list[r]) - 1
        win = conv_state[blk].float()                            # (W0, C)
        pad = torch.cat([win, torch.zeros(W0 + 8, win.shape[1])], 0)
        c0, c1 = pad[off], pad[off + 1]
        xs = z_d[t0:t1].float()
        for p in range(n):
            x = xs[p]
            if bf16_products:
                acc = _bf(c0 * wf[:, 0]) + _bf(c1 * wf[:, 1])
                acc = acc + _bf(x * wf[:, 2])
            else:
                acc = c0 * wf[:, 0] + c1 * wf[:, 1] + x * wf[:, 2]
            out[t0 + p] = acc.to(z_d.dtype)
            c0, c1 = c1, x
        keep = W0 - n
        new = torch.empty_like(win)
        for i in range(W0):
            new[i] = pad[off + 1 + i] if i < keep else xs[i - keep]
        conv_state[blk] = new.to(conv_state.dtype)
    return out


# ---------------------------------------------------------------- inner FIR
def inner_fir_prefill(u_p, w, meta, state, k):
    """Depthwise causal FIR per segment, left context = cached (k-1)-window or zeros.

    u_p (T, H) bf16, w (H, k) cross-correlation order (w[:, -1] pairs with the
    current sample), state (blocks, 127, H) fp32 whose first k-1 columns are
    updated in place (mixers.py:350-383).
    """
    T, H = u_p.shape
    out = torch.empty_like(u_p)
    wt = w.float().unsqueeze(1)
    for a, b, init, blk in segments(meta):
        if b <= a:
            continue
        seq = u_p[a:b].transpose(0, 1).float()                   # (H, L)
        prev = state[blk, : k - 1].transpose(0, 1).float() if init else torch.zeros(H, k - 1)
        seq_in = torch.cat([prev, seq], -1)
        y = F.conv1d(seq_in.unsqueeze(0), wt, padding=0, groups=H)
        out[a:b] = y[0].transpose(0, 1).to(out.dtype)
        state[blk, : k - 1] = seq_in[:, -(k - 1):].transpose(0, 1).to(state.dtype)
    return out


# ---------------------------------------------------------------- LI segment
def modal_filter(res, lp, t):
    """h[d, l] = sum_s res[d, s] exp(lp[d, s] t[l])  (triton_hcl.py:77-85)."""
    h = torch.zeros(res.shape[0], t.shape[0], dtype=torch.float32)
    for s in range(res.shape[1]):
        h += res[:, s : s + 1].float() * torch.exp(lp[:, s : s + 1].float() * t.float())
    return h


def iir_segment(seq, res, lp, s_prev):
    """One LI prefill segment (mixers.py:144-210): FFT long conv with the modal
    filter, closed-form final state, and the s_prev continuation terms.

    seq (H, L) fp32, res/lp (H, S), s_prev (H, S) or None -> (y (H, L), s_last (H, S)).
    """
    H, L = seq.shape
    t = torch.arange(L, dtype=torch.float32)
    h = modal_filter(res, lp, t)
    lag = t.flip(0)
    st = (seq.unsqueeze(1) * torch.exp(lp.unsqueeze(-1) * lag)).sum(-1)
    n = 2 * L
    y = torch.fft.irfft(torch.fft.rfft(seq, n=n) * (torch.fft.rfft(h, n=n) / n), n=n,
                        norm="forward")[..., :L]
    if s_prev is not None:
        st = st + torch.exp(lp * L) * s_prev
        y = y + modal_filter(res * s_prev, lp, t + 1.0)
    return y, st


def iir_segment_scan(seq, res, lp, s_prev):
    """The same map as `iir_segment` as the explicit recurrence s = s*p + x,
    y = sum_s R_s s_s, in float64 (an exactness reference for long segments)."""
    p = torch.exp(lp.double())
    s = torch.zeros_like(p) if s_prev is None else s_prev.double().clone()
    ys = torch.empty(seq.shape, dtype=torch.float64)
    x = seq.double()
    for i in range(seq.shape[1]):
        s = s * p + x[:, i : i + 1]
        ys[:, i] = (res.double() * s).sum(-1)
    return ys.float(), s.float()


# ---------------------------------------------------------------- decode / verify
def accepted_for(meta, accepted):
    nreq = int(meta.num_decodes)
    if accepted is not None:
        return accepted[:nreq].long()
    a = getattr(meta, "num_accepted_tokens", None)
    if a is None:
        return torch.ones(nreq, dtype=torch.long)
    return a[:nreq].long().clamp_min(1)


def decode_tables(meta, accepted):
    """(in_slots, out_slots, starts, ends, accepted) as `_decode_tensors` builds them
    without prefix caching (mixers.py:459-524)."""
    slots = meta.state_indices_tensor_d
    if slots.dim() == 1:
        slots = slots[:, None]
    nreq = int(meta.num_decodes)
    qsl = getattr(meta, "query_start_loc_d", None)
    starts = torch.arange(nreq + 1) if qsl is None else qsl[: nreq + 1].long()
    return slots[:nreq].long(), slots[:nreq].long(), starts[:-1], starts[1:], accepted_for(meta, accepted)


def fir_snapshots(x, w, state, tables, k):
    """mixers.py:578-628 on the SD (blocks, 127, H) state: one full (k-1)-window
    snapshot per verified position; y in x's dtype."""
    ins, outs, starts, ends, accepted = tables
    out = torch.zeros_like(x)
    wf = w.float()
    source = ins.gather(1, (accepted - 1)[:, None]).squeeze(1)
    st = state[source, : k - 1].float()                          # (B, k-1, H)
    lengths = ends - starts
    for pos in range(outs.shape[1]):
        active = pos < lengths
        tok = (starts + pos).clamp_max(x.shape[0] - 1)
        xt = x[tok].float()
        yt = (st.transpose(1, 2) * wf[None, :, :-1]).sum(-1) + wf[None, :, -1] * xt
        nxt = torch.cat([st[:, 1:], xt[:, None]], 1)
        st = torch.where(active[:, None, None], nxt, st)
        for r in range(len(active)):
            if bool(active[r]) and int(outs[r, pos]) != 0:
                state[int(outs[r, pos]), : k - 1] = st[r].to(state.dtype)
        out.index_add_(0, tok, yt.to(out.dtype) * active[:, None])
    return out


def iir_snapshots(x, poles, res, state, tables):
    """mixers.py:631-663: diagonal recurrence with a snapshot after each token."""
    ins, outs, starts, ends, accepted = tables
    out = torch.zeros_like(x)
    source = ins.gather(1, (accepted - 1)[:, None]).squeeze(1)
    S = poles.shape[1]
    st = state[source, :, :S].float()
    lengths = ends - starts
    for pos in range(outs.shape[1]):
        active = pos < lengths
        tok = (starts + pos).clamp_max(x.shape[0] - 1)
        xt = x[tok].float()
        nxt = st * poles[None] + xt[..., None]
        st = torch.where(active[:, None, None], nxt, st)
        for r in range(len(active)):
            if bool(active[r]) and int(outs[r, pos]) != 0:
                state[int(outs[r, pos]), :, :S] = st[r]
        yt = (res[None] * st).sum(-1)
        out.index_add_(0, tok, yt.to(out.dtype) * active[:, None])
    return out


# ---------------------------------------------------------------- decoder-layer norm
def rms_norm(x, weight, eps, residual=None):
    """Evo2RMSNorm (model.py:47-76): s = x (+ residual), y = weight * s /
    (||s||_2 * H^-0.5 + eps), every op a bf16 torch op (eps outside the sqrt).
    Returns y, or (y, s) with a residual, as the reference's forward does."""
    if residual is not None:
        s = x + residual
        return rms_norm(s, weight, eps), s
    h = x.shape[-1]
    y = x / (x.norm(2, dim=-1, keepdim=True) * h ** -0.5 + eps)
    return weight * y


# ---------------------------------------------------------------- fp8 projection
def quantize_input(x, input_scale):
    """Static per-tensor E4M3 quantisation as fp32 values (fp8_emul.py:76-78)."""
    return (x.float() / input_scale).clamp(-FP8_MAX, FP8_MAX).to(E4M3).float()


def _pow2_floor(x):
    _, e = torch.frexp(x)
    return torch.where(x == 0, torch.zeros_like(x), torch.ldexp(torch.ones_like(x), e - 1))


def fast_accum_mm(a, b_t, group=32, frac_bits=13, chunk_rows=256):
    """Hopper fp8 fast-accumulation model (fp8_emul.py:45-73): 32-k groups,
    13 fraction bits, truncation toward zero.  Returns the fp32 accumulator."""
    a = a.float()
    b = b_t.float().t().contiguous()
    N, K = a.shape
    M = b.shape[1]
    pb = _pow2_floor(b.abs())
    out = torch.empty(N, M)
    two_f = 2.0 ** -frac_bits

    def trunc_to(v, ulp):
        return torch.trunc(v / ulp) * ulp

    for r0 in range(0, N, chunk_rows):
        ar = a[r0:r0 + chunk_rows]
        pa = _pow2_floor(ar.abs())
        acc = torch.zeros(ar.shape[0], M)
        for k0 in range(0, K, group):
            ag, bg = ar[:, k0:k0 + group], b[k0:k0 + group]
            mx = (pa[:, k0:k0 + group, None] * pb[None, k0:k0 + group]).amax(1)
            mx = torch.maximum(mx, _pow2_floor(acc.abs()))
            ulp = torch.where(mx == 0, torch.ones_like(mx), mx * two_f)
            s = trunc_to(ag[:, :, None] * bg[None], ulp[:, None, :]).sum(1)
            acc = trunc_to(acc, ulp) + s
            u2 = _pow2_floor(acc.abs()) * two_f
            acc = torch.where(u2 == 0, acc, trunc_to(acc, torch.where(u2 == 0, torch.ones_like(u2), u2)))
        out[r0:r0 + chunk_rows] = acc
    return out


def fp8_linear(x, w8, input_scale, weight_scale, hopper=False):
    """z = bf16((q(x) . W8^T) * sx * sw) (fp8_emul.py:81-88).  hopper=False uses an
    exact fp32 accumulation (Blackwell's tcgen05 accumulates in fp32)."""
    sx = torch.as_tensor(input_scale, dtype=torch.float32).reshape(1)
    sw = torch.as_tensor(weight_scale, dtype=torch.float32).reshape(1)
    xq = quantize_input(x, sx).reshape(-1, x.shape[-1])
    wf = w8.float()
    acc = fast_accum_mm(xq, wf) if hopper else (xq.double() @ wf.double().t()).float()
    out = (acc * sx * sw).to(x.dtype)
    return out.reshape(*x.shape[:-1], w8.shape[0])


# ---------------------------------------------------------------- mixer forward
class MixerParams:
    """Weights of one Hyena layer in checkpoint layout (mixers.py:801-805, 1247-1250,
    1323-1325): short_filter (3H,1,3), conv (H,1,K), D (H,), log_poles (H,S,1),
    residues (H,S), in_proj W (3H,H) [+ fp8 scales], out_proj W (H,H) + bias."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def _decode_rows_first(meta):
    return int(meta.num_decode_tokens), int(meta.num_prefill_tokens)


def mixer_core(z, p, meta, states, accepted=None, bf16_products=True):
    """in_proj output z (T, 3H) -> out_proj input g (T, H), states updated in place.

    bf16_products: bool, or a (prefill, decode) pair, for the K=3 filter rounding.

    Decode rows first, then prefill rows (mixers.py:29-36).  FIR: mixers.py:1277-1305;
    LI: mixers.py:1327-1401.  `states` = [conv (blocks, W0, 3H), inner
    (blocks, 127, H), li (blocks, H, 16[+1])].
    """
    conv_state, inner_state, li_state = states
    H = p.H
    w_short = p.short_filter.reshape(3 * H, 3)
    nd, npt = _decode_rows_first(meta)
    z_d, z_p = z[:nd], z[nd:nd + npt]
    bp_pre, bp_dec = bf16_products if isinstance(bf16_products, tuple) else (bf16_products,) * 2
    parts = []
    if npt:
        parts.append(short_fir_prefill(z_p, w_short, meta, conv_state, bp_pre))
    if nd:
        parts.insert(0, conv_update(z_d, w_short, conv_state, meta, accepted, bp_dec))
    zf = torch.cat(parts, 0) if len(parts) > 1 else parts[0]
    x2, x1, v = zf[:, 0::3], zf[:, 1::3], zf[:, 2::3]
    u = x1 * v
    if p.kind == "fir":
        k = p.k_inner
        w = p.conv.reshape(H, k)
        ys = []
        if npt:
            ys.append(inner_fir_prefill(u[nd:], w, meta, inner_state, k))
        if nd:
            tabs = decode_tables(meta, accepted)
            ys.insert(0, fir_snapshots(u[:nd], w, inner_state, tabs, k))
        y = torch.cat(ys, 0) if len(ys) > 1 else ys[0]
        if p.D is not None:
            y = y + p.D.to(y.dtype) * u
        return x2 * y
    S = p.residues.shape[1]
    lp = p.log_poles[..., 0].float()
    res = p.residues.float()
    y = torch.empty_like(u)
    if nd:
        tabs = decode_tables(meta, accepted)
        y[:nd] = iir_snapshots(u[:nd].float(), lp.exp(), res, li_state, tabs).to(y.dtype)
    for a, b, init, blk in segments(meta):
        if b <= a:
            continue
        seq = u[nd + a:nd + b].float().transpose(0, 1)
        s_prev = li_state[blk, :, :S].float() if init else None
        conv, st = iir_segment(seq, res, lp, s_prev)
        y[nd + a:nd + b] = conv.transpose(0, 1).to(y.dtype)
        li_state[blk, :, :S] = st
    return (y + u * p.D.to(y.dtype)) * x2


def in_proj(x, p, hopper=False):
    """fp8 static W8A8 (fp8_emul.py:81-88) or, for bf16 weights, the reference's
    CPU projection: F.linear in the activation dtype (ReplicatedLinear)."""
    if getattr(p, "in_proj_scales", None) is not None:
        sx, sw = p.in_proj_scales
        return fp8_linear(x, p.in_proj_weight, sx, sw, hopper=hopper)
    return F.linear(x, p.in_proj_weight.to(x.dtype))


def out_proj(g, p):
    """out_proj with bias (mixers.py:801-803): F.linear in the activation dtype."""
    b = None if p.out_proj_bias is None else p.out_proj_bias.to(g.dtype)
    return F.linear(g, p.out_proj_weight.to(g.dtype), b)


def mixer_forward(x, p, meta, states, accepted=None, bf16_products=True, hopper=False):
    """hidden (T, H) bf16 -> mixer output (T, H) bf16 (mixers.py:1277-1305 / 1327-1401)."""
    z = in_proj(x, p, hopper=hopper)
    g = mixer_core(z, p, meta, states, accepted, bf16_products)
    return out_proj(g, p)
