"""Shared helpers for the test-suite: fixtures, metadata, tolerances."""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# The parity bar of the hot path: max |a - b| / max |b| <= 2e-2 on bf16 mixer outputs.
REL_TOL = 2e-2


def max_rel_err(a, b):
    """max |a - b| / max |b| (0 when both are zero)."""
    a = a.float()
    b = b.float()
    den = b.abs().max().item()
    num = (a - b).abs().max().item()
    if den == 0.0:
        return num
    return num / den


def max_slice_rel_err(a, b, floor=1e-3):
    """The larger of the row- and the column-normalised errors of 2-D outputs:
    for every row (token) and every column (channel), max |a - b| over the
    slice / max |b| over the slice.  Unlike max_rel_err, a wrong small-magnitude
    token or channel cannot hide behind the largest value of the tensor.  A
    slice whose max |b| is below `floor` x the global max |b| (an all-zero row,
    say) is measured against that floor instead."""
    a = a.float().reshape(a.shape[0], -1)
    b = b.float().reshape(b.shape[0], -1)
    diff = (a - b).abs()
    mag = b.abs()
    top = mag.max().item()
    if top == 0.0:
        return diff.max().item()
    lo = floor * top
    worst = 0.0
    for dim in (1, 0):
        den = mag.amax(dim).clamp_min(lo)
        worst = max(worst, (diff.amax(dim) / den).max().item())
    return worst


def load_fixture(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def meta_from_dict(d, device="cpu"):
    m = SimpleNamespace()
    for k, v in d.items():
        setattr(m, k, v.to(device) if isinstance(v, torch.Tensor) else v)
    return m


def oracle_params(fx):
    from oracle.hyena_oracle import MixerParams

    p = fx["params"]
    kind = "iir" if fx["kind"] == "hcl" else "fir"
    return MixerParams(
        H=fx["H"], kind=kind, k_inner=fx["k_inner"], short_filter=p["short_filter"],
        conv=p.get("conv"), D=p.get("D"), log_poles=p.get("log_poles"), residues=p.get("residues"),
        in_proj_weight=p["in_proj.weight"], in_proj_scales=None,
        out_proj_weight=p["out_proj.weight"], out_proj_bias=p["out_proj.bias"])


def empty_states(fx, device="cpu"):
    H, nb, ns = fx["H"], fx["num_blocks"], fx["num_spec"]
    return [torch.zeros(nb, 2 + ns, 3 * H, dtype=torch.bfloat16, device=device),
            torch.zeros(nb, 127, H, dtype=torch.float32, device=device),
            torch.zeros(nb, H, 16 + (1 if ns else 0), dtype=torch.float32, device=device)]


def spec_accepted(meta, stamps, num_spec):
    """Accepted counts from position stamps (mixers.py:959-999), host side."""
    slots = meta.state_indices_tensor_d
    if slots.dim() == 1:
        slots = slots[:, None]
    nd = int(meta.num_decodes)
    first = slots[:nd, 0].long()
    offset = meta.num_computed_tokens_d[:nd].long() - stamps[first].long()
    return offset.clamp(0, num_spec) + 1


def record_stamps(meta, stamps, num_spec):
    """Stamp every snapshot written this step (mixers.py:1048-1074), host side."""
    nd = int(meta.num_decodes)
    if nd:
        slots = meta.state_indices_tensor_d
        if slots.dim() == 1:
            slots = slots[:, None]
        qsl = meta.query_start_loc_d
        for r in range(nd):
            n = int(qsl[r + 1] - qsl[r]) if qsl is not None else 1
            for p in range(n):
                b = int(slots[r, p])
                if b != 0:
                    stamps[b] = float(int(meta.num_computed_tokens_d[r]) + p + 1)
    npf = int(meta.num_prefills)
    for j in range(npf):
        stamps[int(meta.state_indices_tensor_p[j])] = float(int(meta.seq_lens[nd + j]))


def random_params(kind, H, k_inner, seed, device="cpu"):
    """Seeded layer weights with the BASELINE recipes: projections N(0, 0.02),
    short filter N(0,1)/sqrt(3), FIR w[:, K-1-lag] = N(0,1)/sqrt(K) exp(-0.05 lag),
    log-poles -exp(U(-6, 0)), residues N(0,1)/16, D N(0, 0.02)."""
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    p = {
        "in_proj.weight": (torch.randn(3 * H, H, generator=g) * 0.02).to(bf),
        "out_proj.weight": (torch.randn(H, H, generator=g) * 0.02).to(bf),
        "out_proj.bias": (torch.randn(H, generator=g) * 0.02).to(bf),
        "short_filter": (torch.randn(3 * H, 1, 3, generator=g) / 3 ** 0.5).to(bf),
    }
    if kind == "hcl":
        p["log_poles"] = (-torch.exp(torch.rand(H, 16, 1, generator=g) * 6 - 6)).float()
        p["residues"] = (torch.randn(H, 16, generator=g) / 16).float()
        p["D"] = (torch.randn(H, generator=g) * 0.02).to(bf)
    else:
        lag = torch.arange(k_inner, dtype=torch.float32)
        filt = torch.randn(H, k_inner, generator=g) / k_inner ** 0.5 * torch.exp(-0.05 * lag)
        p["conv"] = filt.flip(-1).reshape(H, 1, k_inner).to(bf)
        if k_inner >= 128:
            p["D"] = (torch.randn(H, generator=g) * 0.02).to(bf)
    return {k: v.to(device) for k, v in p.items()}


def params_to_oracle(p, kind, H, k_inner):
    from oracle.hyena_oracle import MixerParams

    return MixerParams(
        H=H, kind="iir" if kind == "hcl" else "fir", k_inner=k_inner,
        short_filter=p["short_filter"].cpu(), conv=p.get("conv", None),
        D=p.get("D"), log_poles=p.get("log_poles"), residues=p.get("residues"),
        in_proj_weight=p["in_proj.weight"].cpu(), in_proj_scales=None,
        out_proj_weight=p["out_proj.weight"].cpu(), out_proj_bias=p["out_proj.bias"].cpu())


def prefill_meta(lengths, blocks, has_init, device="cpu"):
    qsl = [0]
    for n in lengths:
        qsl.append(qsl[-1] + n)
    m = SimpleNamespace(
        num_decodes=0, num_decode_tokens=0, num_prefills=len(lengths),
        num_prefill_tokens=qsl[-1],
        query_start_loc_p=torch.tensor(qsl, dtype=torch.int32, device=device),
        has_initial_states_p=torch.tensor(has_init, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.tensor(blocks, dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.zeros(0, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.tensor(lengths, dtype=torch.int32, device=device))
    return m


def decode_meta(slots, lengths=None, computed=None, device="cpu"):
    """Decode-only metadata; `slots` is a list of ints (ordinary) or of lists (spec)."""
    nd = len(slots)
    spec = isinstance(slots[0], (list, tuple))
    lengths = lengths or [1] * nd
    qsl = [0]
    for n in lengths:
        qsl.append(qsl[-1] + n)
    m = SimpleNamespace(
        num_decodes=nd, num_decode_tokens=qsl[-1], num_prefills=0, num_prefill_tokens=0,
        query_start_loc_p=torch.zeros(1, dtype=torch.int32, device=device),
        has_initial_states_p=torch.zeros(0, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.zeros(0, dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.tensor(slots, dtype=torch.int32, device=device),
        query_start_loc_d=torch.tensor(qsl, dtype=torch.int32, device=device) if spec else None,
        num_accepted_tokens=None,
        num_computed_tokens_d=(torch.tensor(computed, dtype=torch.int32, device=device)
                               if computed is not None else None),
        seq_lens=torch.tensor(computed or [0] * nd, dtype=torch.int32, device=device))
    return m


def meta_to(m, device):
    return SimpleNamespace(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v)
                              for k, v in vars(m).items()})


class OracleMixer(torch.nn.Module):
    """A Hyena mixer computed by the CPU oracle, with the mixer-module surface the
    model harness uses (load_full_weights, allocate_state, forward): the
    all-reference arm of the full-model NLL comparison."""

    def __init__(self, cfg, layer_idx, kind, k_inner, prefix, device="cpu"):
        super().__init__()
        self.kind, self.k_inner, self.H = kind, k_inner, cfg.hidden_size
        self.p = None
        self.states = None

    def load_full_weights(self, t):
        from oracle.hyena_oracle import MixerParams

        t = {k: v.cpu() for k, v in t.items()}
        fp8 = t["in_proj.weight"].dtype == torch.float8_e4m3fn
        self.p = MixerParams(
            H=self.H, kind="iir" if self.kind == "hcl" else "fir", k_inner=self.k_inner,
            short_filter=t["short_filter"], conv=t.get("conv"), D=t.get("D"),
            log_poles=t.get("log_poles"), residues=t.get("residues"),
            in_proj_weight=t["in_proj.weight"],
            in_proj_scales=(t["in_proj.input_scale"], t["in_proj.weight_scale"]) if fp8 else None,
            out_proj_weight=t["out_proj.weight"], out_proj_bias=t["out_proj.bias"])

    def allocate_state(self, num_blocks, device=None):
        H = self.H
        self.states = [torch.zeros(num_blocks, 2, 3 * H, dtype=torch.bfloat16),
                       torch.zeros(num_blocks, 127, H), torch.zeros(num_blocks, H, 16)]

    def forward(self, x, token_ids=None):
        """Runs on the CPU whatever device the model is on; the result returns
        to x's device (so the rest of the reference arm can stay on the GPU)."""
        from evo2_flash_b200.forward_context import get_forward_metadata
        from oracle.hyena_oracle import mixer_forward

        meta = get_forward_metadata()
        meta = SimpleNamespace(**{k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                  for k, v in vars(meta).items()})
        return mixer_forward(x.cpu(), self.p, meta, self.states).to(x.device)
