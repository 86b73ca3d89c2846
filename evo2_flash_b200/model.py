"""Engine-free StripedHyena2 (Evo 2) around the B200 Hyena mixers: the harness
for the full-model scoring configuration (random-init 7B, per-token NLL).

The blocks restate the reference's model.py (vLLM building blocks replaced by
plain torch, since the engine is not part of this path):

  Evo2RMSNorm ........ y = w * x / (||x||_2 H^-0.5 + eps), eps outside the sqrt,
                       in the activation dtype (model.py:47-74)
  Evo2MLP ............ l3(act(l1 x) * l2 x), gelu on layer 0 only (model.py:77-101)
  Evo2Attention ...... qkv (no bias) -> neox RoPE -> causal softmax attention ->
                       o_proj (bias) (model.py:104-152)
  Evo2DecoderLayer ... pre_norm -> mixer -> (post_norm(m + x), m + x) -> mlp + res
                       (model.py:155-197)
  StripedHyena2 ...... embedding, layers, final norm, tied lm_head
                       (model.py:200-245, 335-356)

Hyena layers are `HyenaFIRMixer` / `HyenaIIRMixer` from this package (the hot
path); attention, MLP and norms are torch ops (outside the mixer path).
`score` runs teacher-forced prefill over packed varlen steps -- a long sequence
may be split across steps, which exercises the mixers' state continuation -- and
returns each sequence's mean -log p(x_t | x_<t) over t >= 1 with an fp32
log-softmax, like evo2_flash's `score_sequences` (api.py:605-639).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn

from .forward_context import set_forward_metadata


@dataclass
class StripedHyena2Config:
    """Layer map and shapes (config.py:14-205); defaults = evo2-7b-8k."""

    vocab_size: int = 512
    hidden_size: int = 4096
    num_hidden_layers: int = 32
    attn_layer_idxs: tuple = (3, 10, 17, 24, 31)
    hcs_layer_idxs: tuple = (0, 4, 7, 11, 14, 18, 21, 25, 28)
    hcm_layer_idxs: tuple = (1, 5, 8, 12, 15, 19, 22, 26, 29)
    hcl_layer_idxs: tuple = (2, 6, 9, 13, 16, 20, 23, 27, 30)
    short_filter_length: int = 3
    hcs_filter_length: int = 7
    hcm_filter_length: int = 128
    state_size: int = 16
    num_attention_heads: int = 32
    intermediate_size: int = 11008
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    use_fp8_input_projections: bool = True
    extra: dict = field(default_factory=dict)

    @classmethod
    def evo2_7b(cls, **kw):
        return replace(cls(), **kw)

    @classmethod
    def evo2_40b(cls, **kw):
        """evo2-40b-1m layer map: 50 blocks, 8 MHA, 42 Hyena, H = 8192."""
        base = cls(hidden_size=8192, num_hidden_layers=50,
                   attn_layer_idxs=(3, 10, 17, 24, 31, 35, 42, 49),
                   hcs_layer_idxs=(0, 4, 7, 11, 14, 18, 21, 25, 28, 32, 36, 39, 43, 46),
                   hcm_layer_idxs=(1, 5, 8, 12, 15, 19, 22, 26, 29, 33, 37, 40, 44, 47),
                   hcl_layer_idxs=(2, 6, 9, 13, 16, 20, 23, 27, 30, 34, 38, 41, 45, 48),
                   num_attention_heads=64, intermediate_size=22528, rope_theta=1e6)
        return replace(base, **kw)

    @classmethod
    def small(cls, hidden=256, **kw):
        """A 7-block test model with the 7B block pattern [HCS, HCM, HCL, MHA, ...]."""
        base = cls(hidden_size=hidden, num_hidden_layers=7, attn_layer_idxs=(3,),
                   hcs_layer_idxs=(0, 4), hcm_layer_idxs=(1, 5), hcl_layer_idxs=(2, 6),
                   num_attention_heads=max(1, hidden // 128), intermediate_size=2 * hidden)
        return replace(base, **kw)

    def layer_kind(self, i):
        for kind, idx in (("attn", self.attn_layer_idxs), ("hcs", self.hcs_layer_idxs),
                          ("hcm", self.hcm_layer_idxs), ("hcl", self.hcl_layer_idxs)):
            if i in idx:
                return kind
        raise ValueError(f"layer {i} is in no layer-type list")

    def inner_filter_length(self, i):
        return {"hcs": self.hcs_filter_length, "hcm": self.hcm_filter_length}[self.layer_kind(i)]


# ---------------------------------------------------------------- blocks
class Evo2RMSNorm(nn.Module):
    def __init__(self, hidden, eps, device=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden, dtype=torch.bfloat16, device=device),
                                   requires_grad=False)
        self.eps = eps
        self.hidden = hidden

    def forward(self, x, residual=None):
        """norm(x), or (norm(x + residual), x + residual) (model.py:47-76).  On
        CUDA one kernel pass (ops.rms_norm); the torch code is the CPU arm."""
        if x.is_cuda:
            from . import ops

            s = torch.empty_like(x) if residual is not None else None
            y, _ = ops.rms_norm(x, self.weight, self.eps, residual, s_out=s)
            return y if residual is None else (y, s)
        if residual is not None:
            x = x + residual
            return self._norm(x), x
        return self._norm(x)

    def add_norm_(self, x, residual):
        """norm(x + residual), with residual <- x + residual in place (vLLM's
        fused add-RMSNorm)."""
        if x.is_cuda:
            from . import ops

            return ops.rms_norm(x, self.weight, self.eps, residual, s_out=residual)[0]
        residual.add_(x)
        return self._norm(residual)

    def _norm(self, x):
        y = x / (x.norm(2, dim=-1, keepdim=True) * self.hidden ** -0.5 + self.eps)
        return self.weight * y


class Evo2MLP(nn.Module):
    def __init__(self, hidden, inner, use_act, device=None):
        super().__init__()
        kw = dict(bias=False, device=device, dtype=torch.bfloat16)
        self.l1 = nn.Linear(hidden, inner, **kw)
        self.l2 = nn.Linear(hidden, inner, **kw)
        self.l3 = nn.Linear(inner, hidden, **kw)
        self.use_act = use_act
        for p in self.parameters():
            p.requires_grad_(False)

    def forward(self, x):
        z1 = self.l1(x)
        if self.use_act:
            z1 = F.gelu(z1)
        return self.l3(z1 * self.l2(x))


def _rope_neox(x, positions, theta):
    """Rotary embedding, neox style (halves rotated), computed in fp32."""
    hd = x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd)
    ang = positions.to(torch.float32)[:, None] * inv[None]
    cos, sin = ang.cos()[:, None], ang.sin()[:, None]
    xf = x.float()
    a, b = xf[..., : hd // 2], xf[..., hd // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1).to(x.dtype)


class Evo2Attention(nn.Module):
    """MHA with RoPE over packed segments; keys/values of sequences that continue
    in a later step are kept in `self.kv[seq_id]`."""

    def __init__(self, cfg, device=None):
        super().__init__()
        h = cfg.hidden_size
        self.heads = cfg.num_attention_heads
        self.hd = h // self.heads
        self.theta = cfg.rope_theta
        self.qkv_proj = nn.Linear(h, 3 * h, bias=False, device=device, dtype=torch.bfloat16)
        self.o_proj = nn.Linear(h, h, bias=True, device=device, dtype=torch.bfloat16)
        for p in self.parameters():
            p.requires_grad_(False)
        self.kv = {}

    def forward(self, x, positions, segments):
        q, k, v = self.qkv_proj(x).split(x.shape[-1], dim=-1)
        q = _rope_neox(q.view(-1, self.heads, self.hd), positions, self.theta)
        k = _rope_neox(k.view(-1, self.heads, self.hd), positions, self.theta)
        v = v.view(-1, self.heads, self.hd)
        out = torch.empty_like(q)
        for a, b, sid, p0 in segments:
            kk, vv = k[a:b], v[a:b]
            if p0:
                pk, pv = self.kv[sid]
                kk, vv = torch.cat([pk, kk]), torch.cat([pv, vv])
            self.kv[sid] = (kk, vv)
            qs = q[a:b].transpose(0, 1)[None]
            ks, vs = kk.transpose(0, 1)[None], vv.transpose(0, 1)[None]
            if p0:
                qpos = torch.arange(p0, p0 + (b - a), device=x.device)
                mask = torch.arange(p0 + (b - a), device=x.device)[None] <= qpos[:, None]
                o = F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask, scale=self.hd ** -0.5)
            else:
                o = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=self.hd ** -0.5)
            out[a:b] = o[0].transpose(0, 1)
        return self.o_proj(out.reshape(x.shape[0], -1))

    def release(self, sid):
        self.kv.pop(sid, None)


def default_mixer_factory(cfg, layer_idx, kind, k_inner, prefix, device):
    from .mixers import HyenaFIRMixer, HyenaIIRMixer

    if kind == "hcl":
        return HyenaIIRMixer(cfg, layer_idx, prefix=prefix, device=device)
    return HyenaFIRMixer(cfg, layer_idx, prefix=prefix, k_inner=k_inner, device=device)


class Evo2DecoderLayer(nn.Module):
    def __init__(self, cfg, i, device, mixer_factory):
        super().__init__()
        self.kind = cfg.layer_kind(i)
        h = cfg.hidden_size
        self.pre_norm = Evo2RMSNorm(h, cfg.rms_norm_eps, device)
        self.post_norm = Evo2RMSNorm(h, cfg.rms_norm_eps, device)
        if self.kind == "attn":
            self.mixer = Evo2Attention(cfg, device)
        else:
            k = cfg.inner_filter_length(i) if self.kind != "hcl" else 0
            self.mixer = mixer_factory(cfg, i, self.kind, k, f"layers.{i}.mixer", device)
        self.mlp = Evo2MLP(h, cfg.intermediate_size, use_act=(i == 0), device=device)

    def forward(self, x, positions, segments, add=None, input_ids=None):
        """One block (model.py:190-198) on the residual stream x, which it updates
        in place.  `add`: the previous block's MLP output, not yet added to x
        (None for the first block).  Returns (this block's MLP output, x): the
        caller adds them in the next block's pre-norm or in the final norm, the
        sum the reference forms at the end of each block."""
        if self.kind != "attn" and getattr(self.mixer, "fuses_pre_norm", False):
            # pre-norm, residual add and the in_proj quantisation in one pass
            m = (self.mixer(x, input_ids, pre_norm=self.pre_norm) if add is None
                 else self.mixer(add, input_ids, pre_norm=self.pre_norm, residual=x))
        else:
            pre = self.pre_norm(x) if add is None else self.pre_norm.add_norm_(add, x)
            m = (self.mixer(pre, positions, segments) if self.kind == "attn"
                 else self.mixer(pre, input_ids))
        post = self.post_norm.add_norm_(m, x)  # x <- m + x
        return self.mlp(post), x


class StripedHyena2(nn.Module):
    """The full model for prefill scoring.  `mixer_factory(cfg, layer_idx, kind,
    k_inner, prefix, device)` builds each Hyena mixer (default: this package's)."""

    def __init__(self, cfg: StripedHyena2Config, device="cuda", mixer_factory=None):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        factory = mixer_factory or default_mixer_factory
        h = cfg.hidden_size
        self.embed = nn.Parameter(torch.empty(cfg.vocab_size, h, dtype=torch.bfloat16, device=device),
                                  requires_grad=False)
        self.layers = nn.ModuleList(Evo2DecoderLayer(cfg, i, device, factory)
                                    for i in range(cfg.num_hidden_layers))
        self.norm = Evo2RMSNorm(h, cfg.rms_norm_eps, device)

    # ---- weights --------------------------------------------------------------
    def random_tensors(self, seed=0, gen_device="cpu", input_scale=8.0 / 448.0):
        """Seeded random-init weights, name -> tensor.  Embedding (tied lm_head),
        MLP and attention projections N(0, 0.02), o_proj bias 0, norm weights 1;
        Hyena layers by the `synthetic.mixer_tensors` recipes with a fixed static
        input scale (the normed mixer input is RMS 1)."""
        from .synthetic import mixer_tensors

        cfg = self.cfg
        h, inner = cfg.hidden_size, cfg.intermediate_size
        dev = torch.device(gen_device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)

        def n(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)

        t = {"embed": n(cfg.vocab_size, h)}
        for i, layer in enumerate(self.layers):
            pre = f"layers.{i}."
            t[pre + "mlp.l1.weight"] = n(inner, h)
            t[pre + "mlp.l2.weight"] = n(inner, h)
            t[pre + "mlp.l3.weight"] = n(h, inner)
            if layer.kind == "attn":
                t[pre + "mixer.qkv_proj.weight"] = n(3 * h, h)
                t[pre + "mixer.o_proj.weight"] = n(h, h)
                t[pre + "mixer.o_proj.bias"] = torch.zeros(h, dtype=torch.bfloat16, device=dev)
            else:
                k = cfg.inner_filter_length(i) if layer.kind != "hcl" else 0
                mt = mixer_tensors(layer.kind, h, k, seed * 1000 + i,
                                   fp8=cfg.use_fp8_input_projections, device=dev)
                if cfg.use_fp8_input_projections:
                    mt["in_proj.input_scale"] = torch.tensor([input_scale], device=dev)
                for kk, v in mt.items():
                    t[pre + "mixer." + kk] = v
        return t

    def load_tensors(self, tensors):
        """Copies `tensors` (names from `random_tensors`) into the model."""
        mixers = {}
        with torch.no_grad():
            for name, v in tensors.items():
                if name == "embed":
                    self.embed.copy_(v)
                    continue
                parts = name.split(".")
                i, rest = int(parts[1]), ".".join(parts[2:])
                layer = self.layers[i]
                if rest.startswith("mixer.") and layer.kind != "attn":
                    mixers.setdefault(i, {})[rest[len("mixer."):]] = v
                else:
                    dict(layer.named_parameters())[rest].copy_(v)
        for i, mt in mixers.items():
            self.layers[i].mixer.load_full_weights({k: v.to(self.device) for k, v in mt.items()})

    def allocate_state(self, num_blocks):
        for layer in self.layers:
            if layer.kind != "attn":
                layer.mixer.allocate_state(num_blocks, self.device)

    # ---- forward ------------------------------------------------------------------
    def forward(self, input_ids, positions, meta, segments, block_outputs=None):
        """Hidden states after the final norm for one packed step.
        `meta`: mixer metadata (prefill rows, or one-token decode rows);
        `segments`: (row_start, row_end, seq_id, first_position) per sequence
        chunk in the step.  `block_outputs`: a dict whose integer keys name
        blocks; each gets that block's output residual stream (m + x + mlp,
        the reference's block output, model.py:189-198) as a new tensor."""
        x = self.embed[input_ids]
        add = None
        with set_forward_metadata(meta):
            for i, layer in enumerate(self.layers):
                add, x = layer(x, positions, segments, add, input_ids)
                if block_outputs is not None and i in block_outputs:
                    block_outputs[i] = x + add
        return self.norm.add_norm_(add, x)

    def logprobs(self, h, targets):
        logits = F.linear(h, self.embed).float()
        return torch.log_softmax(logits, -1).gather(1, targets[:, None]).squeeze(1)

    @torch.no_grad()
    def prefill_steps(self, seqs, max_tokens_per_step=None, block_outputs=None, keep_cache=False):
        """Teacher-forced prefill of `seqs` (1-D int token tensors) packed in
        order into steps of at most `max_tokens_per_step` tokens (default: all
        in one step); a sequence that does not fit finishes in later steps from
        its cached state (has_initial_state).  Sequence j owns state block j + 1
        (block 0 is the null block) and attention cache entry j; with
        keep_cache the attention entries stay after the last step, so that
        decode_step can continue the sequences (else each is dropped once its
        sequence is done).  Yields (h, segments) per step: h (rows, H) after
        the final norm.
        `block_outputs` (a set of block indices) adds a third item, the dict of
        those blocks' outputs for the step's rows."""
        dev = self.device
        lens = [int(s.numel()) for s in seqs]
        budget = max_tokens_per_step or max(1, sum(lens))
        self.allocate_state(len(seqs) + 1)
        for layer in self.layers:
            if layer.kind == "attn":
                layer.mixer.kv.clear()
        done = [0] * len(seqs)
        nxt = 0
        while nxt < len(seqs) and lens[nxt] == 0:
            nxt += 1
        while nxt < len(seqs):
            rows, segs, used = [], [], 0
            j = nxt
            while j < len(seqs) and used < budget:
                take = min(lens[j] - done[j], budget - used)
                if take > 0:
                    segs.append((used, used + take, j, done[j]))
                    rows.append(seqs[j][done[j]:done[j] + take])
                    used += take
                if done[j] + take < lens[j]:
                    break
                j += 1
            ids = torch.cat(rows).to(dev)
            positions = torch.cat([torch.arange(p0, p0 + (b - a)) for a, b, _, p0 in segs]).to(dev)
            meta = _prefill_meta(segs, dev)
            taps = None if block_outputs is None else dict.fromkeys(block_outputs)
            h = self(ids, positions, meta, segs, taps)
            yield (h, segs) if taps is None else (h, segs, taps)
            for a, b, sid, p0 in segs:
                done[sid] = p0 + (b - a)
                if done[sid] == lens[sid] and not keep_cache:
                    for layer in self.layers:
                        if layer.kind == "attn":
                            layer.mixer.release(sid)
            while nxt < len(seqs) and done[nxt] == lens[nxt]:
                nxt += 1

    @torch.no_grad()
    def token_logprobs(self, seqs, max_tokens_per_step=None):
        """log p(x_t | x_<t) for t = 1 .. L-1 of each sequence (fp32 log-softmax,
        float64 values on the CPU), by teacher-forced prefill_steps."""
        lens = [int(s.numel()) for s in seqs]
        out = [torch.empty(max(0, n - 1), dtype=torch.float64) for n in lens]
        for h, segs in self.prefill_steps(seqs, max_tokens_per_step):
            tgt_rows, tgt, dst = [], [], []
            for a, b, sid, p0 in segs:
                last = min(b - a, lens[sid] - 1 - p0)  # rows with a next token
                if last > 0:
                    tgt_rows.append(torch.arange(a, a + last))
                    tgt.append(seqs[sid][p0 + 1:p0 + 1 + last])
                    dst.append((sid, p0, last))
            if tgt_rows:
                r = torch.cat(tgt_rows).to(self.device)
                lp = self.logprobs(h[r], torch.cat(tgt).to(self.device)).double().cpu()
                off = 0
                for sid, p0, last in dst:
                    out[sid][p0:p0 + last] = lp[off:off + last]
                    off += last
        self.release_all()
        return out

    @torch.no_grad()
    def score(self, seqs, max_tokens_per_step=None):
        """Mean per-token NLL of each sequence (list of 1-D int token tensors).

        Sequences are packed in order into steps of at most `max_tokens_per_step`
        tokens (default: all in one step); a sequence that does not fit finishes in
        later steps from its cached state (has_initial_state)."""
        dev = self.device
        lens = [int(s.numel()) for s in seqs]
        budget = max_tokens_per_step or max(1, sum(lens))
        self.allocate_state(len(seqs) + 1)
        done = [0] * len(seqs)
        sums = [0.0] * len(seqs)
        cnt = [0] * len(seqs)
        nxt = 0
        while nxt < len(seqs):
            rows, segs, used = [], [], 0
            j = nxt
            while j < len(seqs) and used < budget:
                take = min(lens[j] - done[j], budget - used)
                if take > 0:
                    segs.append((used, used + take, j, done[j]))
                    rows.append(seqs[j][done[j]:done[j] + take])
                    used += take
                if done[j] + take < lens[j]:
                    break
                j += 1
            ids = torch.cat(rows).to(dev)
            positions = torch.cat([torch.arange(p0, p0 + (b - a)) for a, b, _, p0 in segs]).to(dev)
            meta = _prefill_meta(segs, dev)
            h = self(ids, positions, meta, segs)
            tgt_rows, tgt = [], []
            for a, b, sid, p0 in segs:
                last = min(b - a, lens[sid] - 1 - p0)  # rows with a next token
                if last > 0:
                    tgt_rows.append(torch.arange(a, a + last))
                    tgt.append(seqs[sid][p0 + 1:p0 + 1 + last])
            if tgt_rows:
                r = torch.cat(tgt_rows).to(dev)
                lp = self.logprobs(h[r], torch.cat(tgt).to(dev)).double().cpu()
                off = 0
                for a, b, sid, p0 in segs:
                    last = min(b - a, lens[sid] - 1 - p0)
                    if last > 0:
                        sums[sid] += float(lp[off:off + last].sum())
                        cnt[sid] += last
                        off += last
            for a, b, sid, p0 in segs:
                done[sid] = p0 + (b - a)
                if done[sid] == lens[sid]:
                    for layer in self.layers:
                        if layer.kind == "attn":
                            layer.mixer.release(sid)
            while nxt < len(seqs) and done[nxt] == lens[nxt]:
                nxt += 1
        return [-s / c if c else math.nan for s, c in zip(sums, cnt)]

    @torch.no_grad()
    def decode_step(self, token_ids, positions, seq_ids):
        """One token for each of the given sequences, continuing their cached
        state (Hyena: one-token decode rows on state block seq_id + 1; attention:
        the sequence's key/value cache): (B, H) hidden states after the final
        norm.  token_ids, positions: (B,) ints; seq_ids: B distinct ints."""
        dev = self.device
        ids = torch.as_tensor(token_ids, dtype=torch.long).to(dev)
        pos = torch.as_tensor(positions, dtype=torch.long)
        segs = [(i, i + 1, int(sid), int(p)) for i, (sid, p) in enumerate(zip(seq_ids, pos.tolist()))]
        meta = _decode_meta([int(sid) + 1 for sid in seq_ids], dev)
        return self(ids, pos.to(dev), meta, segs)

    def release_all(self):
        """Drops every sequence's attention key/value cache."""
        for layer in self.layers:
            if layer.kind == "attn":
                layer.mixer.kv.clear()


def _prefill_meta(segs, device):
    """Prefill-only mixer metadata for one step; sequence j owns state block j+1."""
    qsl = [0]
    for a, b, _, _ in segs:
        qsl.append(qsl[-1] + (b - a))
    n = len(segs)
    return SimpleNamespace(
        num_decodes=0, num_decode_tokens=0, num_prefills=n, num_prefill_tokens=qsl[-1],
        query_start_loc_p=torch.tensor(qsl, dtype=torch.int32, device=device),
        has_initial_states_p=torch.tensor([p0 > 0 for _, _, _, p0 in segs], dtype=torch.bool,
                                          device=device),
        state_indices_tensor_p=torch.tensor([sid + 1 for _, _, sid, _ in segs], dtype=torch.int32,
                                            device=device),
        state_indices_tensor_d=torch.zeros(0, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.tensor([p0 + (b - a) for a, b, _, p0 in segs], dtype=torch.int32,
                              device=device))


def _decode_meta(blocks, device):
    """One-token decode metadata for the mixers: request i on state block blocks[i]."""
    n = len(blocks)
    return SimpleNamespace(
        num_decodes=n, num_decode_tokens=n, num_prefills=0, num_prefill_tokens=0,
        query_start_loc_p=torch.zeros(1, dtype=torch.int32, device=device),
        has_initial_states_p=torch.zeros(0, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.zeros(0, dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.tensor(blocks, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.zeros(n, dtype=torch.int32, device=device))
