"""Hyena mixers for Evo 2 on B200: the drop-in for evo2_flash/mixers.py.

Same constructor signatures, parameter names and shapes, paged-state contract
and metadata fields as the reference's `HyenaFIRMixer` / `HyenaIIRMixer`
(mixers.py:711-1401); `in_proj` and `out_proj` stay hookable submodules that
return `(y, None)` like vLLM's ReplicatedLinear (api.py:185-188 hooks them).

Per step, between the two GEMMs, a layer issues at most two kernel launches
(one decode/verify launch for the decode rows, one prefill launch for the prefill
rows) instead of the reference's chain of Triton kernels, torch elementwise ops
and, for LI prefill, a Python loop over segments with an FFT each.

    in_proj   fp8: quant_e4m3 + tcgen05 e4m3 GEMM; bf16: tcgen05 bf16 GEMM
    decode    ops.decode   (K=3 update + gate + inner FIR/LI + D + x2, snapshots)
    prefill   ops.prefill  (same chain over packed varlen segments)
    out_proj  tcgen05 bf16 GEMM + bias   [+ NCCL all-reduce when channel-sharded]

Paged state (vLLM's SD layout, mixers.py:6-17, 892-904):
    kv_cache[0]  (blocks, K_short-1 [+num_spec], 3H) bf16   short-filter window
    kv_cache[1]  (blocks, 127, H) fp32                     inner FIR window
    kv_cache[2]  (blocks, H, 16 [+1 stamp]) fp32           LI modal state

Channel sharding (tp_size > 1): rank r owns channels [r H/P, (r+1) H/P); in_proj
keeps the matching rows of the interleaved (3H, H) weight (whole (x2, x1, v)
triples), out_proj the matching columns, and one all-reduce per layer sums the
partial outputs before the bias.  State shapes shrink to the local H.
"""

from __future__ import annotations

import torch
from torch import nn

from . import ops
from .custom_op import HYENA_MIXER_OP, register_layer
from .forward_context import lookup
from .parallel import PendingReduce, all_reduce_partial, all_reduce_partial_async, shard_mixer_tensors


# ---------------------------------------------------------------- projections
class Fp8InProj(nn.Module):
    """Static W8A8 e4m3 projection (the checkpoints' `vllm_fp8_static_w8a8_v1`
    contract, config.py:134-146): params `weight` (N, K) e4m3, `weight_scale`,
    `input_scale` (dequantisation scales).  forward -> (y, None)."""

    def __init__(self, in_features, out_features, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.float8_e4m3fn,
                                               device=device), requires_grad=False)
        self.weight_scale = nn.Parameter(torch.ones(1, dtype=torch.float32, device=device),
                                         requires_grad=False)
        self.input_scale = nn.Parameter(torch.ones(1, dtype=torch.float32, device=device),
                                        requires_grad=False)

    def forward(self, x):
        xq = ops.quant_e4m3(x, self.input_scale)
        return ops.gemm_e4m3(xq, self.weight, self.input_scale, self.weight_scale), None


class Bf16Linear(nn.Module):
    """bf16 nn.Linear on the tcgen05 GEMM.  forward -> (y, None)."""

    def __init__(self, in_features, out_features, bias=False, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.bfloat16,
                                               device=device), requires_grad=False)
        self.bias = (nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device),
                                  requires_grad=False) if bias else None)
        self.skip_bias = False  # the row-parallel out_proj adds it after the all-reduce

    def forward(self, x):
        bias = None if self.skip_bias else self.bias
        return ops.gemm_bf16(x, self.weight, bias), None


class ProjectionTap(nn.Module):
    """Parameter-free stand-in for in_proj in FP8-surgery layers whose projection
    is a token table or the fully emulated GEMM (mixers.py:681-688): forward(z)
    -> (z, None), so a hook on in_proj still sees the projection output."""

    def forward(self, z):
        return z, None


class HybridProjection(Bf16Linear):
    """bf16 in_proj whose calibrated worst output channels are recomputed by the
    emulated FP8 GEMM inside the module (mixers.py:691-702), so hooks see the
    final projection.  `emulate(x) -> (cols, values)` is attached by the mixer."""

    emulate = None

    def forward(self, x):
        z, _ = super().forward(x)
        cols, emul = self.emulate(x)
        return z.index_copy(-1, cols, emul), None


# ---------------------------------------------------------------- helpers
def _cache_safe_state_indices(indices, state):
    """vLLM's undersized profiling cache: use null block 0 (mixers.py:527-540)."""
    if indices.dim() == 2 and state.shape[0] < indices.numel():
        return torch.zeros_like(indices)
    return indices


def _accepted_tokens(m, num_reqs, device):
    a = getattr(m, "num_accepted_tokens", None)
    if a is None:
        return torch.ones(num_reqs, device=device, dtype=torch.long)
    if a.numel() < num_reqs:
        raise ValueError(f"num_accepted_tokens is too short: shape={tuple(a.shape)}, "
                         f"num_decodes={num_reqs}")
    return a[:num_reqs].to(torch.long).clamp_min(1)


def _decode_tensors(m, num_tokens, max_positions=None, accepted=None):
    """(in_slots, out_slots, starts, accepted) on device (mixers.py:459-524),
    including the prefix-caching ("all" mode) slot gathers (mixers.py:443-456).
    accepted=False skips the accepted counts (returned as None)."""
    slots = m.state_indices_tensor_d
    if slots.dim() == 1:
        slots = slots[:, None]
    if slots.dim() != 2:
        raise ValueError(f"state_indices_tensor_d must be rank 1 or 2, got shape={tuple(slots.shape)}")
    num_reqs = int(m.num_decodes)
    if slots.shape[0] < num_reqs:
        raise ValueError(f"decode state rows={slots.shape[0]} smaller than num_decodes={num_reqs}")
    starts = getattr(m, "query_start_loc_d", None)
    if starts is None:
        if num_tokens != num_reqs:
            raise ValueError("packed multi-token decode requires query_start_loc_d: "
                             f"num_decode_tokens={num_tokens}, num_decodes={num_reqs}")
        starts = torch.arange(num_reqs + 1, device=slots.device, dtype=torch.int32)
    else:
        if starts.numel() < num_reqs + 1:
            raise ValueError(f"query_start_loc_d is too short: shape={tuple(starts.shape)}, "
                             f"num_decodes={num_reqs}")
        starts = starts[: num_reqs + 1]
    if accepted is False:  # the caller needs the slots only
        accepted = None
    elif accepted is None:
        accepted = _accepted_tokens(m, num_reqs, slots.device)
    else:
        accepted = accepted[:num_reqs]
    slots = slots[:num_reqs]
    previous = getattr(m, "block_idx_last_scheduled_token_prev_step", None)
    scheduled = getattr(m, "block_idx_last_scheduled_token", None)
    ins = outs = slots
    if previous is not None and scheduled is not None:
        width = slots.shape[1] if max_positions is None else min(slots.shape[1], max_positions)
        off = torch.arange(width, device=slots.device, dtype=torch.long)
        ins = slots.gather(1, previous[:num_reqs, None].long() + off)
        outs = slots.gather(1, scheduled[:num_reqs, None].long() + off)
    elif max_positions is not None:
        ins = outs = slots[:, :max_positions]
    return ins, outs, starts, accepted


class HyenaMixerBase(nn.Module):
    """Shared front half: in_proj -> stateful K=3 FIR -> de-interleave -> gate."""

    kind = "fir"
    fuses_pre_norm = True  # forward() takes pre_norm= / residual=

    def __init__(self, config, layer_idx: int, model_config=None, cache_config=None,
                 prefix: str = "", quant_config=None, *, num_spec: int | None = None,
                 tp_rank: int = 0, tp_size: int = 1, tp_group=None, device=None,
                 compilation_config=None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.prefix = prefix
        self.model_config = model_config
        self.cache_config = cache_config
        h = config.hidden_size
        if h % tp_size:
            raise ValueError(f"hidden size {h} does not split over {tp_size} ranks")
        self.hidden_full = h
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        self.hidden = h // tp_size
        hl = self.hidden
        self.k_short = config.short_filter_length
        if self.k_short != 3:
            raise ValueError("the short filter kernels implement K_short = 3")
        self.num_spec = int(num_spec or 0)
        self.use_fp8 = bool(getattr(config, "use_fp8_input_projections", False))
        # FP8-surgery layers (mixers.py:758-800): a per-token table, the fully
        # emulated Hopper GEMM, or a bf16 projection with emulated channels.
        self.in_proj_token_table = None
        self.in_proj_emul_weight_t = None
        self.in_proj_emul_scales = None
        self.in_proj_emul_cols = None
        chan = getattr(config, "hyena_fp8_emulated_channels", None) or {}
        n_emul = int(chan.get(layer_idx, 0)) if isinstance(chan, dict) else 0
        token_layers = tuple(getattr(config, "hyena_token_table_layers", None) or ())
        emul_layers = tuple(getattr(config, "hyena_fp8_emulated_layers", None) or ())
        surgery = layer_idx in token_layers or layer_idx in emul_layers or n_emul > 0
        if surgery and tp_size != 1:
            raise ValueError(f"{prefix}: FP8-surgery layers are not channel-sharded (tp_size must be 1)")
        bf16 = dict(dtype=torch.bfloat16, device=device)
        if layer_idx in token_layers:
            self.in_proj = ProjectionTap()
            self.in_proj_token_table = nn.Parameter(
                torch.empty(config.vocab_size, 3 * h, **bf16), requires_grad=False)
        elif layer_idx in emul_layers:
            self.in_proj = ProjectionTap()
            self.in_proj_emul_weight_t = nn.Parameter(torch.empty(h, 3 * h, **bf16),
                                                      requires_grad=False)
            self.in_proj_emul_scales = nn.Parameter(
                torch.empty(2, dtype=torch.float32, device=device), requires_grad=False)
        elif n_emul:
            self.in_proj = HybridProjection(h, 3 * h, bias=False, device=device)
            self.in_proj_emul_weight_t = nn.Parameter(torch.empty(h, n_emul, **bf16),
                                                      requires_grad=False)
            self.in_proj_emul_scales = nn.Parameter(
                torch.empty(2, dtype=torch.float32, device=device), requires_grad=False)
            self.in_proj_emul_cols = nn.Parameter(
                torch.empty(n_emul, dtype=torch.int64, device=device), requires_grad=False)
            self.in_proj.emulate = lambda x: (
                self.in_proj_emul_cols,
                ops.fp8_linear_emulated(x, self.in_proj_emul_weight_t, self.in_proj_emul_scales))
        elif self.use_fp8:
            self.in_proj = Fp8InProj(h, 3 * hl, device=device)
        else:
            self.in_proj = Bf16Linear(h, 3 * hl, bias=False, device=device)
        self.out_proj = Bf16Linear(hl, h, bias=True, device=device)
        self.out_proj.skip_bias = tp_size > 1
        self.short_filter = nn.Parameter(torch.empty(3 * hl, 1, self.k_short, dtype=torch.bfloat16,
                                                     device=device), requires_grad=False)
        self.kv_cache = (torch.tensor([]), torch.tensor([]), torch.tensor([]))
        self._weights = None
        self._weights_key = None
        # With an engine's compilation config the layer registers under its
        # prefix and forward() runs as the opaque custom op (mixers.py:807-829).
        register_layer(prefix, self, compilation_config)
        self.use_custom_op = compilation_config is not None

    # ---- kernel-side weights --------------------------------------------------
    def _kernel_weights(self) -> ops.LayerWeights:
        params = [p for p in self._inner_params() if p is not None] + [self.short_filter]
        key = tuple((p.data_ptr(), p._version) for p in params)
        if self._weights is None or key != self._weights_key:
            self._weights = self._build_weights()
            self._weights_key = key
        return self._weights

    # ---- state spec (mixers.py:858-917) ---------------------------------------
    @staticmethod
    def unified_state_shape(hidden, k_short, k_inner_max, state_size, num_spec=0):
        return ((k_short - 1 + num_spec, 3 * hidden), (k_inner_max - 1, hidden),
                (hidden, state_size + (1 if num_spec else 0)))

    @staticmethod
    def unified_state_dtype(model_dtype=torch.bfloat16):
        return (model_dtype, torch.float32, torch.float32)

    def get_state_shape(self):
        c = self.config
        return self.unified_state_shape(self.hidden, c.short_filter_length, c.hcm_filter_length,
                                        c.state_size, self.num_spec)

    def get_state_dtype(self):
        dt = getattr(self.model_config, "dtype", torch.bfloat16) if self.model_config else torch.bfloat16
        return self.unified_state_dtype(dt)

    def allocate_state(self, num_blocks, device=None):
        """Zeroed paged state with this layer's spec (for engine-free use)."""
        shapes, dtypes = self.get_state_shape(), self.get_state_dtype()
        self.kv_cache = tuple(torch.zeros(num_blocks, *s, dtype=d, device=device)
                              for s, d in zip(shapes, dtypes))
        return self.kv_cache

    # ---- engine surface (vLLM MambaBase; mixers.py:832-850) -------------------
    attn_backend = None  # the engine's metadata backend class; None: vLLM's stock Mamba2

    @property
    def mamba_type(self):
        """MAMBA2: the metadata builder that passes accepted-token counts
        (mixers.py:833-840); the string "mamba2" without vLLM."""
        try:
            from vllm.v1.attention.backends.registry import MambaAttentionBackendEnum
        except Exception:  # vLLM absent: engine-free use
            return "mamba2"
        return MambaAttentionBackendEnum.MAMBA2

    def get_attn_backend(self):
        """The metadata backend (mixers.py:842-850): `attn_backend` when set (with
        speculation the engine's Hyena builder, which adds num_computed_tokens_d;
        the mixers read the same field names), else vLLM's stock Mamba2 one."""
        if self.attn_backend is not None:
            return self.attn_backend
        from vllm.v1.attention.backends.mamba2_attn import Mamba2AttentionBackend

        return Mamba2AttentionBackend

    @staticmethod
    def decode_state_indices(m):
        idx = m.state_indices_tensor_d
        return idx[:, 0] if idx.dim() > 1 else idx

    @staticmethod
    def is_speculative_decode(m) -> bool:
        idx = m.state_indices_tensor_d
        return ((idx.dim() > 1 and idx.shape[1] > 1)
                or getattr(m, "num_accepted_tokens", None) is not None
                or int(m.num_decode_tokens) != int(m.num_decodes))

    def _meta(self):
        return lookup(self.prefix)

    # ---- position stamps (mixers.py:952-1074) ---------------------------------
    def _position_stamps(self):
        return self.kv_cache[2][:, 0, -1]

    def _spec_accepted(self, m):
        """Accepted tokens per request from the position stamps (mixers.py:962-984),
        in one kernel (hyena_spec_accepted).  A mismatching stamp, where the
        reference's device assert fires, is clamped and reported through the
        kernel's error word instead."""
        nd = int(m.num_decodes)
        computed = getattr(m, "num_computed_tokens_d", None)
        if computed is None:
            raise RuntimeError("speculative Hyena decode needs num_computed_tokens_d "
                               "(HyenaMamba2Backend metadata)")
        slots = m.state_indices_tensor_d[:nd]
        if slots.dim() == 1:
            slots = slots[:, None]
        slots = _cache_safe_state_indices(slots, self.kv_cache[2])
        return ops.spec_accepted(slots, computed[:nd], self._position_stamps(), self.num_spec)

    def _repair_resumed_prefill_state(self, m):
        if not self.num_spec or not int(m.num_prefills):
            return
        computed = getattr(m, "computed_before_p", None)
        src = getattr(m, "state_src_block_p", None)
        has_init = getattr(m, "has_initial_states_p", None)
        if computed is None or src is None or has_init is None:
            return
        npf = int(m.num_prefills)
        dst = m.state_indices_tensor_p[:npf].long()
        src = src[:npf].long()
        computed = computed[:npf].to(torch.float32)
        stamps = self._position_stamps()
        bad = (has_init[:npf].bool() & (stamps[dst] != computed) & (stamps[src] == computed)
               & (src != 0) & (dst != 0))
        take = torch.where(bad, src, dst)
        for state in self.kv_cache:
            state[dst] = state[take]

    def _resolve_accepted(self, m):
        if self.num_spec and int(m.num_decodes) and self.is_speculative_decode(m):
            return self._spec_accepted(m)
        return None

    def _record_stamps(self, m):
        """Stamps of the slots written this step (mixers.py:1040-1074): verifier
        slots in one kernel (hyena_spec_record), prefill blocks in torch."""
        if not self.num_spec:
            return
        stamps = self._position_stamps()
        nd = int(m.num_decodes)
        if nd and self.is_speculative_decode(m):
            _, outs, starts, _ = _decode_tensors(m, int(m.num_decode_tokens), 1 + self.num_spec,
                                                 accepted=False)
            outs = _cache_safe_state_indices(outs, self.kv_cache[2])
            ops.spec_record(outs, starts, m.num_computed_tokens_d[:nd], stamps)
        npf = int(m.num_prefills)
        if npf:
            stamps[m.state_indices_tensor_p[:npf].long()] = m.seq_lens[nd:nd + npf].to(stamps.dtype)

    # ---- forward ----------------------------------------------------------------
    def _project(self, hidden_states, token_ids=None, pre_norm=None, residual=None):
        """in_proj, or for FP8-surgery layers the token table / the emulated GEMM,
        always returned through self.in_proj (mixers.py:1076-1092)."""
        if isinstance(self.in_proj, ProjectionTap):
            if pre_norm is not None and self.in_proj_token_table is None:
                hidden_states, _ = ops.rms_norm(hidden_states, pre_norm.weight, pre_norm.eps,
                                                residual, s_out=residual)
            elif pre_norm is not None and residual is not None:
                # the table ignores the normed input; the residual add still happens
                ops.rms_norm(hidden_states, pre_norm.weight, pre_norm.eps, residual, want_y=False,
                             s_out=residual)
            if self.in_proj_token_table is not None:
                if token_ids is None:
                    raise ValueError(
                        f"{self.prefix}: token-table projection needs input_ids "
                        "(inputs_embeds are unsupported for FP8-surgery checkpoints)")
                z, _ = self.in_proj(self.in_proj_token_table[token_ids[: hidden_states.shape[0]]])
                return z
            z, _ = self.in_proj(ops.fp8_linear_emulated(hidden_states, self.in_proj_emul_weight_t,
                                                        self.in_proj_emul_scales))
            return z
        if pre_norm is not None:
            # The decoder layer's pre-norm (and residual add) in the in_proj's input
            # pass: with the fp8 projection and no hook on it, the normed input
            # only ever exists as e4m3 (ops.rms_norm).
            ip = self.in_proj
            fused = isinstance(ip, Fp8InProj) and not (ip._forward_hooks or ip._forward_pre_hooks)
            y, q = ops.rms_norm(hidden_states, pre_norm.weight, pre_norm.eps, residual,
                                want_y=not fused, quant_scale=ip.input_scale if fused else None,
                                s_out=residual)
            if fused:
                return ops.gemm_e4m3(q, ip.weight, ip.input_scale, ip.weight_scale)
            hidden_states = y
        z, _ = self.in_proj(hidden_states)
        return z

    def _states_for_kernels(self):
        """(conv (blocks, W0, 3H), inner) views in the kernels' orientation."""
        s0 = self.kv_cache[0]
        if s0.shape[-1] != 3 * self.hidden:  # dim-first orientation -> SD view
            s0 = s0.transpose(-1, -2)
        return s0, self._inner_state_view()

    def _run_core(self, z, m, accepted):
        """g (T, H) = the mixer core on z (T, 3H); decode rows first, then prefill."""
        w = self._kernel_weights()
        nd, npt = int(m.num_decode_tokens), int(m.num_prefill_tokens)
        g = torch.empty(nd + npt, self.hidden, dtype=torch.bfloat16, device=z.device)
        conv, inner = self._states_for_kernels()
        if nd:
            if self.is_speculative_decode(m):
                ins, outs, starts, acc = _decode_tensors(m, nd, 1 + self.num_spec, accepted)
                ins = _cache_safe_state_indices(ins, inner)
                outs = _cache_safe_state_indices(outs, inner)
                slots = m.state_indices_tensor_d[: int(m.num_decodes)]
                slots = slots[:, None] if slots.dim() == 1 else slots
                slots = _cache_safe_state_indices(slots, conv)
                sched = getattr(m, "block_idx_last_scheduled_token", None)
                comp = getattr(m, "block_idx_last_computed_token", None)
                nreq = slots.shape[0]
                cin = slots.gather(1, comp[:nreq, None].long()).squeeze(1) if comp is not None else slots[:, 0]
                cout = slots.gather(1, sched[:nreq, None].long()).squeeze(1) if sched is not None else slots[:, 0]
                ops.decode(w, z[:nd], g[:nd], cin, cout, ins, outs, conv, inner,
                           token_start=starts, accepted=acc, zero_null_rows=False,
                           skip_null_writes=True)
            else:
                idx = self.decode_state_indices(m)[: int(m.num_decodes)]
                ops.decode(w, z[:nd], g[:nd], idx, idx, idx[:, None], idx[:, None], conv, inner,
                           zero_null_rows=True, skip_null_writes=True)
        if npt:
            ops.prefill(w, z[nd:nd + npt], g[nd:], m.query_start_loc_p,
                        getattr(m, "has_initial_states_p", None),
                        m.state_indices_tensor_p[: int(m.num_prefills)], conv, inner)
        return g

    def _out_proj(self, g, async_reduce=False, finish=None):
        out, _ = self.out_proj(g)
        if self.tp_size > 1:
            if async_reduce:
                return all_reduce_partial_async(out, self.out_proj.bias, self.tp_group, finish)
            out = all_reduce_partial(out, self.out_proj.bias, self.tp_group)
        if async_reduce:
            return PendingReduce(out, None, None, finish)
        return out

    def _forward_impl(self, hidden_states, token_ids=None, async_reduce=False, pre_norm=None,
                      residual=None):
        if residual is not None and pre_norm is None:
            raise ValueError("residual is added inside the pre-norm: pass pre_norm too")
        m = self._meta()
        if m is None:
            out = self._profile_run(hidden_states, token_ids, pre_norm, residual)
            return PendingReduce(out, None, None) if async_reduce else out
        self._repair_resumed_prefill_state(m)
        accepted = self._resolve_accepted(m)  # before any state is written
        nd, npt = int(m.num_decode_tokens), int(m.num_prefill_tokens)
        z = self._project(hidden_states[: nd + npt], token_ids, pre_norm,
                          None if residual is None else residual[: nd + npt])
        g = self._run_core(z, m, accepted)
        self._record_stamps(m)
        finish = lambda out: self._unpad(out, hidden_states, nd + npt)  # noqa: E731
        if async_reduce:
            return self._out_proj(g, True, finish)
        return finish(self._out_proj(g))

    def forward(self, hidden_states, token_ids=None, *, pre_norm=None, residual=None):
        """(T, H) bf16 -> (T, H) bf16 (mixers.py:823-829).

        With `pre_norm` (the decoder layer's Evo2RMSNorm: `.weight`, `.eps`) the
        mixer's input is pre_norm(hidden_states + residual) -- hidden_states
        alone without a residual -- computed in the in_proj's input pass; the
        sum is written back into `residual`, as vLLM's fused add-RMSNorm does.
        A layer built with a compilation config runs the plain form through the
        custom op torch.ops.evo2_b200.hyena_mixer."""
        if self.use_custom_op and pre_norm is None:
            output = torch.empty_like(hidden_states)
            torch.ops.evo2_b200.hyena_mixer(hidden_states, output, token_ids, self.prefix)
            return output
        return self._forward_impl(hidden_states, token_ids, pre_norm=pre_norm, residual=residual)

    def forward_async(self, hidden_states, token_ids=None, *, pre_norm=None,
                      residual=None) -> PendingReduce:
        """forward() with the channel-sharded all-reduce left in flight: returns a
        PendingReduce whose wait() yields the output.  Lets a caller overlap one
        step's (or chunk's) all-reduce with the next one's kernels; with
        tp_size == 1 the result is complete already."""
        return self._forward_impl(hidden_states, token_ids, async_reduce=True, pre_norm=pre_norm,
                                  residual=residual)

    @staticmethod
    def _unpad(out, hidden_states, n_actual):
        if out.shape[0] == hidden_states.shape[0]:
            return out
        full = torch.zeros_like(hidden_states)
        full[:n_actual] = out
        return full

    def _profile_run(self, hidden_states, token_ids=None, pre_norm=None, residual=None):
        """attn_metadata is None during a memory-profiling pass (mixers.py:1230-1235)."""
        z = self._project(hidden_states, token_ids, pre_norm, residual)
        y = z[:, 0::3] * z[:, 1::3] * z[:, 2::3]
        return self._out_proj(y.contiguous())

    # ---- weights ------------------------------------------------------------------
    def load_full_weights(self, tensors: dict):
        """Copies unsharded checkpoint tensors (names as in the reference) into this
        rank's shard (evo2_flash_b200.parallel.shard_mixer_tensors)."""
        shard = shard_mixer_tensors(tensors, self.tp_rank, self.tp_size, self.hidden_full)
        params = dict(self.named_parameters())
        with torch.no_grad():
            for name, t in shard.items():
                if name not in params:
                    raise KeyError(f"unexpected tensor {name!r} for {type(self).__name__}")
                dst = params[name]
                dst.copy_(t.reshape(dst.shape))
        self._weights = None


class HyenaFIRMixer(HyenaMixerBase):
    """Hyena-SE (K=7) and Hyena-MR (K=128): explicit depthwise causal conv
    (mixers.py:1238-1305)."""

    kind = "fir"

    def __init__(self, config, layer_idx, model_config=None, cache_config=None, prefix="",
                 k_inner=128, quant_config=None, **kw):
        super().__init__(config, layer_idx, model_config, cache_config, prefix, quant_config, **kw)
        hl = self.hidden
        self.k_inner = k_inner
        dev = kw.get("device")
        self.conv = nn.Parameter(torch.empty(hl, 1, k_inner, dtype=torch.bfloat16, device=dev),
                                 requires_grad=False)
        self.has_D = k_inner >= 128
        self.D = (nn.Parameter(torch.empty(hl, dtype=torch.bfloat16, device=dev), requires_grad=False)
                  if self.has_D else None)

    def _inner_params(self):
        return [self.conv, self.D]

    def _build_weights(self):
        return ops.layer_weights("fir", self.short_filter, conv=self.conv, D=self.D)

    def _inner_state_view(self):
        s1 = self.kv_cache[1]
        if s1.shape[-1] != self.hidden:
            s1 = s1.transpose(-1, -2)
        return s1



class HyenaIIRMixer(HyenaMixerBase):
    """Hyena-LI: diagonal LTI SSM s_t = p s_{t-1} + x_t (mixers.py:1308-1401)."""

    kind = "iir"

    def __init__(self, config, layer_idx, model_config=None, cache_config=None, prefix="",
                 quant_config=None, **kw):
        super().__init__(config, layer_idx, model_config, cache_config, prefix, quant_config, **kw)
        hl, s = self.hidden, config.state_size
        dev = kw.get("device")
        self.state_size = s
        self.log_poles = nn.Parameter(torch.empty(hl, s, 1, dtype=torch.float32, device=dev),
                                      requires_grad=False)
        self.residues = nn.Parameter(torch.empty(hl, s, dtype=torch.float32, device=dev),
                                     requires_grad=False)
        self.D = nn.Parameter(torch.empty(hl, dtype=torch.bfloat16, device=dev), requires_grad=False)

    def _inner_params(self):
        return [self.log_poles, self.residues, self.D]

    def _build_weights(self):
        return ops.layer_weights("iir", self.short_filter, D=self.D, log_poles=self.log_poles,
                                 residues=self.residues)

    def _inner_state_view(self):
        s2 = self.kv_cache[2]
        expected = (self.hidden, self.state_size + (1 if self.num_spec else 0))
        if tuple(s2.shape[-2:]) != expected:
            raise RuntimeError(f"temporal state cache has wrong trailing shape: expected {expected}, "
                               f"got {tuple(s2.shape[-2:])}")
        return s2

