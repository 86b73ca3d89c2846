"""Seeded synthetic weights and ACGT token streams for the benchmark
configurations (no checkpoint or dataset is available offline).

Weight recipes (one per Hyena layer kind, names as in the reference's converted
checkpoints, convert.py:466-497):

  in_proj.weight   (3H, H)   N(0, 0.02); fp8: e4m3 with per-tensor scale amax/448
  out_proj.weight  (H, H)    N(0, 0.02) bf16, out_proj.bias zeros
  short_filter     (3H,1,3)  N(0,1)/sqrt(3)
  conv             (H,1,K)   w[:, K-1-lag] = N(0,1)/sqrt(K) exp(-0.05 lag)
                             (cross-correlation order: the last tap meets the
                             current sample)
  log_poles        (H,16,1)  -exp(U(-6, 0));  residues (H,16) N(0,1)/16
  D                (H,)      N(0, 0.02)  (HCM and HCL only)

Token ids are the byte codes of A, C, G, T (65, 67, 71, 84).
"""

from __future__ import annotations

import torch

ACGT = (65, 67, 71, 84)


def _gen(seed, device):
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g, dev


def mixer_tensors(kind, hidden, k_inner, seed, fp8=True, device="cpu"):
    """One Hyena layer's checkpoint tensors (`kind` in {"hcs", "hcm", "hcl"}).

    With fp8 the in_proj is returned as e4m3 `weight` + `weight_scale`; the caller
    adds `input_scale` (a calibration amax / 448).  Draws come from a generator on
    `device`, so a given (seed, device) pair always yields the same tensors."""
    g, dev = _gen(seed, device)
    H = hidden
    w_in = torch.randn(3 * H, H, generator=g, device=dev) * 0.02
    p = {}
    if fp8:
        sw = w_in.abs().amax() / 448.0
        p["in_proj.weight"] = (w_in / sw).clamp(-448, 448).to(torch.float8_e4m3fn)
        p["in_proj.weight_scale"] = sw.reshape(1).float()
    else:
        p["in_proj.weight"] = w_in.to(torch.bfloat16)
    del w_in
    p["out_proj.weight"] = (torch.randn(H, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    p["out_proj.bias"] = torch.zeros(H, dtype=torch.bfloat16, device=dev)
    p["short_filter"] = (torch.randn(3 * H, 1, 3, generator=g, device=dev) / 3 ** 0.5).to(torch.bfloat16)
    if kind == "hcl":
        p["log_poles"] = -torch.exp(torch.rand(H, 16, 1, generator=g, device=dev) * 6 - 6)
        p["residues"] = torch.randn(H, 16, generator=g, device=dev) / 16
        p["D"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    else:
        lag = torch.arange(k_inner, dtype=torch.float32, device=dev)
        filt = torch.randn(H, k_inner, generator=g, device=dev) / k_inner ** 0.5 * torch.exp(-0.05 * lag)
        p["conv"] = filt.flip(-1).reshape(H, 1, k_inner).to(torch.bfloat16)
        if k_inner >= 128:
            p["D"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return p


def uniform_acgt(n, gen):
    """n uniform-random ACGT byte ids (int64, CPU) from torch generator `gen`."""
    lut = torch.tensor(ACGT)
    return lut[torch.randint(0, 4, (n,), generator=gen)]


def markov_acgt(lengths, seed=3, order=3):
    """ACGT sequences from an order-`order` Markov chain: 4**order contexts, each
    with a transition row drawn from Dirichlet(1) (normalised Exp(1) draws), all
    seeded.  The first `order` letters are uniform.  Returns a list of int64 CPU
    tensors of byte ids, one per length."""
    g = torch.Generator().manual_seed(seed)
    n_ctx = 4 ** order
    e = -torch.log(torch.rand(n_ctx, 4, generator=g).clamp_min(1e-12))
    rows = e / e.sum(-1, keepdim=True)
    cdf = rows.cumsum(-1)
    n, L = len(lengths), max(lengths) if lengths else 0
    sym = torch.zeros(n, L, dtype=torch.long)
    if L:
        sym[:, :min(order, L)] = torch.randint(0, 4, (n, min(order, L)), generator=g)
        ctx = torch.zeros(n, dtype=torch.long)
        for t in range(min(order, L)):
            ctx = ctx * 4 + sym[:, t]
        u = torch.rand(L, n, generator=g)
        for t in range(order, L):
            nxt = torch.searchsorted(cdf[ctx], u[t][:, None]).squeeze(1).clamp_max(3)
            sym[:, t] = nxt
            ctx = (ctx * 4 + nxt) % n_ctx
    lut = torch.tensor(ACGT)
    return [lut[sym[i, :ln]] for i, ln in enumerate(lengths)]
