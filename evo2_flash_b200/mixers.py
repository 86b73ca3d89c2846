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

from dataclasses import dataclass

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
    """bf16 nn.Linear on the tcgen05 GEMM.  forward(x[, out=]) -> (y, None);
    `out` (rows of x, N) receives the result in place of a new tensor."""

    def __init__(self, in_features, out_features, bias=False, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.bfloat16,
                                               device=device), requires_grad=False)
        self.bias = (nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device),
                                  requires_grad=False) if bias else None)
        # A row-parallel out_proj adds its bias on one rank only (in that rank's
        # GEMM epilogue), so the all-reduce of the partials counts it once.
        self.skip_bias = False

    def forward(self, x, out=None):
        bias = None if self.skip_bias else self.bias
        return ops.gemm_bf16(x, self.weight, bias, out=out), None


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


# ---------------------------------------------------------------- decode plan
@dataclass
class DecodePlan:
    """Where the decode rows of one step read and write their state, resolved
    on the device from the engine's metadata without a host synchronisation.

    table     (reqs, cols) block table of the decode requests (a 1-D table is
              one column); in the speculative layout column p is the snapshot
              slot of verifier position p
    in_slots  (reqs, q) blocks the inner state is read from, indexed by the
              accepted count - 1
    out_slots (reqs, q) blocks the state after token p is written to
    starts    (reqs + 1,) token offsets of the requests, or None (one each)
    conv_in / conv_out  (reqs,) blocks of the short-filter window
    engine_accepted     the engine's own accepted counts (the kernels read a
                        count below 1 as 1), or None when it sent none (every
                        count then reads as 1)
    """

    reqs: int
    table: torch.Tensor
    in_slots: torch.Tensor
    out_slots: torch.Tensor
    starts: torch.Tensor | None
    conv_in: torch.Tensor
    conv_out: torch.Tensor
    engine_accepted: torch.Tensor | None


def _profiling_table(table, num_blocks):
    """vLLM's memory-profiling pass sizes the state cache for one block per
    request while a speculative block table names one block per verifier
    position; a table that cannot fit the cache is that pass (its results are
    discarded), and it is pointed at the null block 0 instead.  Decided on
    shapes alone, so it costs no synchronisation and is fixed under capture
    (the reference's rule, mixers.py:527-540)."""
    if table.dim() == 2 and table.numel() > num_blocks:
        return table.new_zeros(table.shape)
    return table


def _pick_columns(table, first_col, width):
    """(reqs, width) columns of `table` starting at each request's first_col."""
    cols = first_col[:, None].long() + torch.arange(width, device=table.device)
    return table.gather(1, cols)


def plan_decode(m, positions, num_blocks):
    """DecodePlan of a step's decode rows (mixers.py:443-524 resolve the same
    slots).  positions: verifier positions per request (1 + num_spec).
    num_blocks: blocks of the smallest state slice (for the profiling rule).
    Shape errors raise ValueError before anything is indexed; value ranges are
    the engine's (out-of-range blocks are reported by the kernels' error word)."""
    reqs = int(m.num_decodes)
    tokens = int(m.num_decode_tokens)
    table = m.state_indices_tensor_d
    if table.dim() not in (1, 2):
        raise ValueError(f"decode block table must be 1-D or 2-D, got {table.dim()}-D "
                         f"{tuple(table.shape)}")
    if table.dim() == 1:
        table = table.unsqueeze(1)
    if table.shape[0] < reqs:
        raise ValueError(f"decode block table has {table.shape[0]} rows for {reqs} requests")
    table = table[:reqs]
    starts = getattr(m, "query_start_loc_d", None)
    if starts is not None:
        if starts.numel() <= reqs:
            raise ValueError(f"query_start_loc_d holds {starts.numel()} offsets, "
                             f"{reqs + 1} needed")
        starts = starts[: reqs + 1]
    elif tokens != reqs:
        raise ValueError(f"{tokens} decode tokens over {reqs} requests need query_start_loc_d "
                         "(the per-request token offsets)")
    engine = getattr(m, "num_accepted_tokens", None)
    if engine is not None:
        if engine.numel() < reqs:
            raise ValueError(f"num_accepted_tokens holds {engine.numel()} counts for "
                             f"{reqs} requests")
        engine = engine[:reqs]  # counts below 1 read as 1 in the kernels
    width = min(table.shape[1], positions)
    prev = getattr(m, "block_idx_last_scheduled_token_prev_step", None)
    sched = getattr(m, "block_idx_last_scheduled_token", None)
    if prev is not None and sched is not None:
        # prefix caching ("all" mode): the live window moves along the table
        in_slots = _pick_columns(table, prev[:reqs], width)
        out_slots = _pick_columns(table, sched[:reqs], width)
    else:
        in_slots = out_slots = table[:, :width]
    conv_table = _profiling_table(table, num_blocks)
    comp = getattr(m, "block_idx_last_computed_token", None)
    conv_in = (_pick_columns(conv_table, comp[:reqs], 1)[:, 0] if comp is not None
               else conv_table[:, 0])
    conv_out = (_pick_columns(conv_table, sched[:reqs], 1)[:, 0] if sched is not None
                else conv_table[:, 0])
    return DecodePlan(reqs, conv_table, _profiling_table(in_slots, num_blocks),
                      _profiling_table(out_slots, num_blocks), starts, conv_in, conv_out, engine)


class HyenaMixerBase(nn.Module):
    """Shared front half: in_proj -> stateful K=3 FIR -> de-interleave -> gate."""

    kind = "fir"
    fuses_pre_norm = True  # forward() takes pre_norm= / residual=

    def __init__(self, config, layer_idx: int, model_config=None, cache_config=None,
                 prefix: str = "", quant_config=None, *, num_spec: int | None = None,
                 tp_rank: int = 0, tp_size: int = 1, tp_group=None, device=None,
                 compilation_config=None, tp_collective: str = "auto"):
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
        # the row-parallel out_proj's all-reduce: "nvls" (in-switch, our kernel),
        # "nccl", or "auto" (nvls where the GPUs have NVLink multicast)
        if tp_collective not in ("auto", "nvls", "nccl"):
            raise ValueError(f"tp_collective must be auto, nvls or nccl, got {tp_collective!r}")
        self.tp_collective = tp_collective
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
        self.out_proj.skip_bias = tp_size > 1 and tp_rank != 0
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
    # One fp32 per state block (S2's last column of channel 0) records how many
    # tokens the block's snapshot represents; speculative rollback and the
    # prefix-cache repair are decided from it on the device, in small kernels
    # (csrc/spec.cu), so no step ever synchronises with the host.
    def _position_stamps(self):
        return self.kv_cache[2][:, 0, -1]

    def _num_blocks(self):
        return min(int(t.shape[0]) for t in self.kv_cache)

    def _decode_plan(self, m):
        return plan_decode(m, 1 + self.num_spec, self._num_blocks())

    def _accepted_from_stamps(self, m, plan):
        """Tokens accepted at the previous verify step, per request: the gap
        between the request's computed-token count and the stamp of its first
        block, clamped to [0, num_spec], plus one (hyena_spec_accepted; the
        reference derives it at mixers.py:962-984 and asserts on a mismatch,
        which here sets HYENA_FLAG_STAMP in the kernel's error word)."""
        computed = getattr(m, "num_computed_tokens_d", None)
        if computed is None:
            raise RuntimeError(f"{self.prefix}: speculative decode needs num_computed_tokens_d "
                               "in the step metadata (the engine's Hyena metadata builder)")
        return ops.spec_accepted(plan.table, computed[: plan.reqs], self._position_stamps(),
                                 self.num_spec)

    def _repair_prefill_blocks(self, m):
        """Prefix caching can hand a resumed prefill row a block whose snapshot
        is not the one at its computed-token count (the reference documents the
        case at mixers.py:1001-1037); hyena_state_repair copies the block of the
        row's last computed token over it when that one carries the right stamp."""
        npf = int(m.num_prefills)
        fields = [getattr(m, f, None) for f in ("computed_before_p", "state_src_block_p",
                                                 "has_initial_states_p")]
        if not self.num_spec or npf == 0 or any(f is None for f in fields):
            return
        computed, src, has_init = fields
        ops.state_repair(m.state_indices_tensor_p[:npf], src, computed, has_init,
                         self._position_stamps(), list(self.kv_cache))

    def _stamp_written_blocks(self, m, plan):
        """After the step: every verifier slot written gets computed + p + 1
        (hyena_spec_record) and every prefill block its sequence length
        (hyena_spec_record_prefill), as mixers.py:1040-1074 requires."""
        if not self.num_spec:
            return
        stamps = self._position_stamps()
        if plan is not None and self.is_speculative_decode(m):
            starts = plan.starts
            if starts is None:
                starts = torch.arange(plan.reqs + 1, device=plan.table.device, dtype=torch.int32)
            ops.spec_record(plan.out_slots, starts, m.num_computed_tokens_d[: plan.reqs], stamps)
        npf, nd = int(m.num_prefills), int(m.num_decodes)
        if npf:
            ops.spec_record_prefill(m.state_indices_tensor_p[:npf], m.seq_lens[nd:nd + npf], stamps)

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

    def _run_core(self, z, m, accepted, plan=None):
        """g (T, H) = the mixer core on z (T, 3H); decode rows first, then prefill.
        plan: the step's DecodePlan (built here when the step has decode rows
        and none is given); accepted: stamp-derived counts or None."""
        w = self._kernel_weights()
        nd, npt = int(m.num_decode_tokens), int(m.num_prefill_tokens)
        g = torch.empty(nd + npt, self.hidden, dtype=torch.bfloat16, device=z.device)
        conv, inner = self._states_for_kernels()
        if nd:
            if self.is_speculative_decode(m):
                plan = plan or self._decode_plan(m)
                ops.decode(w, z[:nd], g[:nd], plan.conv_in, plan.conv_out, plan.in_slots,
                           plan.out_slots, conv, inner, token_start=plan.starts,
                           accepted=accepted if accepted is not None else plan.engine_accepted,
                           zero_null_rows=False, skip_null_writes=True)
            else:
                # one token per request, state read and written in place; rows
                # on the null block are CUDA-graph padding (zero output, no write)
                blk = self.decode_state_indices(m)[: int(m.num_decodes)]
                col = blk.unsqueeze(1)
                ops.decode(w, z[:nd], g[:nd], blk, blk, col, col, conv, inner,
                           zero_null_rows=True, skip_null_writes=True)
        if npt:
            ops.prefill(w, z[nd:nd + npt], g[nd:], m.query_start_loc_p,
                        getattr(m, "has_initial_states_p", None),
                        m.state_indices_tensor_p[: int(m.num_prefills)], conv, inner)
        return g

    def _out_proj(self, g, async_reduce=False, out=None):
        """out_proj of g; with `out` (at least g's rows) the result is written
        into its first rows.  Channel-sharded: the partial sums (rank 0's with the
        bias from its GEMM epilogue) are all-reduced, left in flight when
        async_reduce.  With the in-switch collective the GEMM writes the partial
        into the group reducer's buffer ring and the result is a view into that
        ring, valid until 32 further channel-sharded out_projs of the group have
        been started (every caller here consumes it before then)."""
        if self.tp_size > 1 and out is None and self.tp_collective != "nccl":
            from .parallel import nvls_reducer

            red = nvls_reducer(self.tp_group, g.shape[0] * self.hidden_full, g.device)
            if red is None and self.tp_collective == "nvls":
                raise RuntimeError("tp_collective='nvls' but the GPUs have no NVLink multicast")
            if red is not None:
                k, buf = red.buffer(g.shape[0], self.hidden_full)
                self.out_proj(g, out=buf)
                pend = red.reduce_async(k, buf)
                return pend if async_reduce else pend.wait()
        y, _ = self.out_proj(g, out=None if out is None else out[: g.shape[0]])
        full = y if out is None else out
        if self.tp_size > 1:
            if async_reduce:
                return all_reduce_partial_async(full, None, self.tp_group)
            return all_reduce_partial(full, None, self.tp_group)
        return PendingReduce(full, None, None) if async_reduce else full

    def _output_buffer(self, hidden_states, rows):
        """None when the mixer computes every row; else a (padded rows, H) tensor
        whose rows past `rows` are zero.  Under CUDA graphs vLLM pads the token
        count to a captured size and the decoder layer's residual add needs an
        output of the padded length (mixers.py:1214-1228): the GEMM writes the
        real rows into it directly, no copy."""
        if rows == hidden_states.shape[0]:
            return None
        buf = torch.empty_like(hidden_states)
        buf[rows:].zero_()
        return buf

    def _forward_impl(self, hidden_states, token_ids=None, async_reduce=False, pre_norm=None,
                      residual=None):
        if residual is not None and pre_norm is None:
            raise ValueError("residual is added inside the pre-norm: pass pre_norm too")
        m = self._meta()
        if m is None:
            out = self._profile_run(hidden_states, token_ids, pre_norm, residual)
            return PendingReduce(out, None, None) if async_reduce else out
        self._repair_prefill_blocks(m)
        nd, npt = int(m.num_decode_tokens), int(m.num_prefill_tokens)
        plan = self._decode_plan(m) if int(m.num_decodes) and self.is_speculative_decode(m) else None
        # accepted counts come from the stamps before this layer writes any state
        accepted = (self._accepted_from_stamps(m, plan)
                    if plan is not None and self.num_spec else None)
        z = self._project(hidden_states[: nd + npt], token_ids, pre_norm,
                          None if residual is None else residual[: nd + npt])
        g = self._run_core(z, m, accepted, plan)
        self._stamp_written_blocks(m, plan)
        out = self._output_buffer(hidden_states, nd + npt)
        res = self._out_proj(g, async_reduce, out)
        return res

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

    def _profile_run(self, hidden_states, token_ids=None, pre_norm=None, residual=None):
        """vLLM's memory-profiling pass runs without metadata (mixers.py:1230-1235):
        no state is touched; the triple product of the in_proj channels stands
        in for the mixer so that both projections allocate what a step does."""
        z = self._project(hidden_states, token_ids, pre_norm, residual)
        x2, x1, v = z.unflatten(-1, (self.hidden, 3)).unbind(-1)
        return self._out_proj((x2 * x1 * v).contiguous())

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

