"""Generates the golden fixtures in this directory by running the REFERENCE
evo2_flash mixers (its own CPU torch paths) on seeded inputs.

Run in a container that has the reference checkout and vLLM importable:

    python tests/golden/make_golden.py /path/to/evo2_flash_checkout

Shims (the reference's mixers are vLLM modules; nothing here changes their math):
  * `ReplicatedLinear`        -> a bf16 nn.Linear returning (y, None)
  * `get_current_vllm_config` -> a stub carrying `speculative_config` and an empty
                                 `static_forward_context`
  * `layer._meta`             -> the seeded metadata object of the step
  * `causal_conv1d_update`    -> oracle.hyena_oracle.conv_update: vLLM's K=3
                                 decode update is a Triton kernel with no CPU path,
                                 so decode/verify fixtures pin the K=3 decode step
                                 to the oracle's restatement of it; everything
                                 after it (inner FIR / LI snapshots, gates, stamps)
                                 is the reference's own code.
  * EVO2_TORCH_SHORT_FIR=1    -> the reference's own torch twin for the K=3 prefill.
The fp8 fixture calls the reference's fp8_emul functions directly; the norm
fixture runs the reference's Evo2RMSNorm (model.py) on CPU.

Each fixture is a torch.save'd dict: config, parameters, and per step the
metadata, the mixer input x, and the reference's in_proj output z, out_proj input
g, output, plus the final paged state.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import hyena_oracle as O  # noqa: E402

H = 128
BF = torch.bfloat16


class _Linear(nn.Module):
    def __init__(self, in_f, out_f, bias=False, prefix="", quant_config=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_f, in_f, dtype=BF), requires_grad=False)
        self.bias = nn.Parameter(torch.empty(out_f, dtype=BF), requires_grad=False) if bias else None

    def forward(self, x):
        return F.linear(x, self.weight, self.bias), None


def _conv_update_shim(x, conv_state, weight, bias, activation=None, conv_state_indices=None,
                      block_idx_last_scheduled_token=None, initial_state_idx=None,
                      num_accepted_tokens=None, query_start_loc=None, max_query_len=-1,
                      **kw):
    assert bias is None and activation is None and block_idx_last_scheduled_token is None
    idx = conv_state_indices
    nreq = idx.shape[0]
    meta = SimpleNamespace(state_indices_tensor_d=idx, num_decodes=nreq,
                           query_start_loc_d=query_start_loc)
    sd = conv_state.transpose(-1, -2)  # dim-first view -> SD view of the same storage
    return O.conv_update(x, weight, sd, meta, num_accepted_tokens, bf16_products=True)


def _import_reference(ref_root):
    sys.path.insert(0, str(ref_root))
    os.environ["EVO2_TORCH_SHORT_FIR"] = "1"
    import evo2_flash.mixers as M

    M.ReplicatedLinear = _Linear
    M.causal_conv1d_update = _conv_update_shim
    return M


def _vllm_cfg(num_spec):
    spec = SimpleNamespace(num_speculative_tokens=num_spec) if num_spec else None
    comp = SimpleNamespace(static_forward_context={}, splitting_ops=None)
    return SimpleNamespace(speculative_config=spec, compilation_config=comp)


def make_params(kind, k_inner, seed):
    """Seeded weights with the BASELINE recipes (see tests/helpers for the same)."""
    g = torch.Generator().manual_seed(seed)
    p = {
        "in_proj.weight": (torch.randn(3 * H, H, generator=g) * 0.02).to(BF),
        "out_proj.weight": (torch.randn(H, H, generator=g) * 0.02).to(BF),
        "out_proj.bias": (torch.randn(H, generator=g) * 0.02).to(BF),
        "short_filter": (torch.randn(3 * H, 1, 3, generator=g) / 3 ** 0.5).to(BF),
    }
    if kind == "hcl":
        p["log_poles"] = (-torch.exp(torch.rand(H, 16, 1, generator=g) * 6 - 6)).float()
        p["residues"] = (torch.randn(H, 16, generator=g) / 16).float()
        p["D"] = (torch.randn(H, generator=g) * 0.02).to(BF)
    else:
        lag = torch.arange(k_inner, dtype=torch.float32)
        filt = torch.randn(H, k_inner, generator=g) / k_inner ** 0.5 * torch.exp(-0.05 * lag)
        p["conv"] = filt.flip(-1).reshape(H, 1, k_inner).to(BF)  # w[:, K-1-lag]
        if k_inner >= 128:
            p["D"] = (torch.randn(H, generator=g) * 0.02).to(BF)
    return p


def build_layer(M, kind, k_inner, num_spec, params):
    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False, vocab_size=512)
    M.get_current_vllm_config = lambda: _vllm_cfg(num_spec)
    mc = SimpleNamespace(dtype=BF)
    if kind == "hcl":
        layer = M.HyenaIIRMixer(cfg, 0, mc, None, f"golden.{kind}")
    else:
        layer = M.HyenaFIRMixer(cfg, 0, mc, None, f"golden.{kind}", k_inner=k_inner)
    with torch.no_grad():
        for name, t in layer.named_parameters():
            t.copy_(params[name])
    return layer


def make_states(num_blocks, num_spec):
    return (torch.zeros(num_blocks, 2 + num_spec, 3 * H, dtype=BF),
            torch.zeros(num_blocks, 127, H, dtype=torch.float32),
            torch.zeros(num_blocks, H, 16 + (1 if num_spec else 0), dtype=torch.float32))


def make_meta(decode_blocks, decode_lens, prefill, computed=None, num_spec=0):
    """prefill: list of (length, block, has_init, seq_len_total)."""
    nd = len(decode_blocks)
    m = SimpleNamespace()
    m.num_decodes = nd
    m.num_decode_tokens = sum(decode_lens)
    m.num_prefills = len(prefill)
    m.num_prefill_tokens = sum(p[0] for p in prefill)
    qsl = [0]
    for p in prefill:
        qsl.append(qsl[-1] + p[0])
    m.query_start_loc_p = torch.tensor(qsl, dtype=torch.int32)
    m.has_initial_states_p = torch.tensor([p[2] for p in prefill], dtype=torch.bool)
    m.state_indices_tensor_p = torch.tensor([p[1] for p in prefill], dtype=torch.int32)
    if num_spec:
        m.state_indices_tensor_d = torch.tensor(decode_blocks, dtype=torch.int32).reshape(nd, -1) \
            if nd else torch.zeros(0, 1 + num_spec, dtype=torch.int32)
    else:
        m.state_indices_tensor_d = torch.tensor([b if isinstance(b, int) else b[0] for b in decode_blocks],
                                                dtype=torch.int32)
    dq = [0]
    for n in decode_lens:
        dq.append(dq[-1] + n)
    m.query_start_loc_d = torch.tensor(dq, dtype=torch.int32) if num_spec else None
    m.num_accepted_tokens = None
    seq = list(computed or [0] * nd) + [p[3] for p in prefill]
    m.seq_lens = torch.tensor(seq, dtype=torch.int32)
    m.num_computed_tokens_d = torch.tensor(computed, dtype=torch.int32) if computed else None
    m.computed_before_p = None
    m.state_src_block_p = None
    m.block_idx_last_scheduled_token = None
    m.block_idx_last_scheduled_token_prev_step = None
    m.block_idx_last_computed_token = None
    return m


def meta_dict(m):
    return {k: v for k, v in vars(m).items()}


def run_case(M, name, kind, k_inner, num_spec, num_blocks, steps, seed):
    params = make_params(kind, k_inner, seed)
    layer = build_layer(M, kind, k_inner, num_spec, params)
    states = make_states(num_blocks, num_spec)
    layer.kv_cache = states
    g = torch.Generator().manual_seed(seed + 1000)
    emb = torch.randn(512, H, generator=g)
    captured = {}
    layer.in_proj.register_forward_hook(lambda mod, a, out: captured.__setitem__("z", out[0].clone()))
    layer.out_proj.register_forward_hook(lambda mod, a, out: captured.__setitem__("g", a[0].clone()))
    out_steps = []
    for meta in steps:
        T = int(meta.num_decode_tokens) + int(meta.num_prefill_tokens)
        toks = torch.tensor([b"ACGT"[i] for i in torch.randint(0, 4, (T,), generator=g).tolist()])
        x = emb[toks].to(BF)
        layer._meta = (lambda m=meta: m)
        with torch.no_grad():
            out = layer._forward_impl(x)
        out_steps.append({"meta": meta_dict(meta), "x": x, "z": captured["z"], "g": captured["g"],
                          "out": out})
    fixture = {
        "name": name, "kind": kind, "k_inner": k_inner, "num_spec": num_spec, "H": H,
        "num_blocks": num_blocks, "params": params, "steps": out_steps,
        "final_states": [s.clone() for s in states],
    }
    # Only the slice a kind uses is interesting; keep fixtures small.
    if kind == "hcl":
        fixture["final_states"][1] = None
    else:
        fixture["final_states"][2] = None if not num_spec else fixture["final_states"][2][:, 0, 16].clone()
    torch.save(fixture, HERE / f"{name}.pt")
    print(f"wrote {name}.pt ({len(out_steps)} steps)")


def fp8_fixture(ref_root):
    from evo2_flash import fp8_emul as FE

    g = torch.Generator().manual_seed(77)
    x = (torch.randn(64, 256, generator=g)).to(BF)
    w = torch.randn(96, 256, generator=g) * 0.05
    sw = (w.abs().amax() / 448.0).float()
    w8 = (w / sw).clamp(-448, 448).to(torch.float8_e4m3fn)
    sx = (x.float().abs().amax() / 448.0 * 1.5).float()  # some saturation
    xq = FE.quantize_input(x, sx)
    out_hopper = FE.static_fp8_linear_emulated(x, w8, sx, sw)
    torch.save({"x": x, "w8": w8.view(torch.uint8), "sx": sx, "sw": sw, "xq": xq,
                "out_hopper": out_hopper}, HERE / "fp8_in_proj.pt")
    print("wrote fp8_in_proj.pt")


def norm_fixture(ref_root):
    """Evo2RMSNorm with and without the residual add, then the in_proj input
    quantisation of its output.  Rows 0-15 hold multiples of 1/4 in [-4, 4]:
    their sum of squares is exact in fp32 in any order, so a kernel that sums in
    another order must still match them bit for bit; the other rows mix
    magnitudes up to the 1e12 a late residual stream reaches."""
    from evo2_flash import fp8_emul as FE
    from evo2_flash.model import Evo2RMSNorm

    g = torch.Generator().manual_seed(91)
    rows, h = 48, 256
    x = torch.randn(rows, h, generator=g)
    x[:16] = torch.randint(-16, 17, (16, h), generator=g).float() / 4
    x[32:] *= torch.logspace(0, 12, 16)[:, None]
    x = x.to(BF)
    r = torch.randn(rows, h, generator=g)
    r[:16] = torch.randint(-4, 5, (16, h), generator=g).float() / 4  # sums stay on the grid
    r = r.to(BF)
    norm = Evo2RMSNorm(h, 1e-6)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(h, generator=g))
        norm.weight.data = norm.weight.data.to(BF)
        y = norm(x)
        y_add, s_add = norm(x, r)
    sx = torch.tensor(4.0 / 448.0)
    torch.save({"x": x, "r": r, "weight": norm.weight.data.clone(), "eps": 1e-6, "y": y,
                "y_add": y_add, "s_add": s_add, "sx": sx,
                "q_add": FE.quantize_input(y_add, sx)}, HERE / "rms_norm.pt")
    print("wrote rms_norm.pt")


def main(ref_root):
    M = _import_reference(ref_root)
    torch.manual_seed(0)
    mm = make_meta
    # HCM prefill: fresh ragged segments, then continuations (one shorter than K-1).
    run_case(M, "hcm_prefill", "hcm", 128, 0, 6, [
        mm([], [], [(150, 1, False, 150), (37, 2, False, 37), (200, 3, False, 200)]),
        mm([], [], [(5, 2, True, 42), (140, 1, True, 290), (20, 4, False, 20)]),
    ], seed=1)
    # HCS: prefill, then decode rows mixed with a fresh prefill, then pure decode.
    run_case(M, "hcs_mixed", "hcs", 7, 0, 6, [
        mm([], [], [(30, 1, False, 30), (9, 2, False, 9), (64, 3, False, 64)]),
        mm([1, 2, 3], [1, 1, 1], [(40, 4, False, 40)]),
        mm([1, 2, 3, 4], [1, 1, 1, 1], []),
    ], seed=2)
    # HCL: prefill (multi-chunk and tiny segments), continuation + decode, decode.
    run_case(M, "hcl_mixed", "hcl", 16, 0, 6, [
        mm([], [], [(300, 1, False, 300), (3, 2, False, 3), (97, 3, False, 97)]),
        mm([2, 3], [1, 1], [(50, 1, True, 350), (600, 4, False, 600)]),
        mm([1, 2, 3, 4], [1, 1, 1, 1], []),
        mm([1, 2, 3, 4], [1, 1, 1, 1], []),
    ], seed=3)
    # HCM decode after prefill.
    run_case(M, "hcm_decode", "hcm", 128, 0, 4, [
        mm([], [], [(64, 1, False, 64), (130, 2, False, 130)]),
        mm([1, 2], [1, 1], []),
        mm([1, 2], [1, 1], []),
        mm([1, 2], [1, 1], []),
    ], seed=4)
    # Speculative verify (K=3 drafts, q=4): ragged lengths and accepted counts
    # resolved from position stamps.
    for kind, k in (("hcm", 128), ("hcl", 16), ("hcs", 7)):
        slots = [[1, 3, 4, 5], [2, 6, 7, 8]]
        run_case(M, f"{kind}_spec", kind, k, 3, 9, [
            mm([], [], [(40, 1, False, 40), (50, 2, False, 50)], num_spec=3),
            mm(slots, [4, 2], [], computed=[40, 50], num_spec=3),
            mm(slots, [4, 1], [], computed=[43, 52], num_spec=3),
            mm(slots, [1, 3], [], computed=[47, 53], num_spec=3),
        ], seed=5 + k)
    fp8_fixture(ref_root)
    norm_fixture(ref_root)


if __name__ == "__main__":
    # The reference checkout to run: first argument, else $EVO2_REFERENCE_ROOT.
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EVO2_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <evo2_flash checkout> (or set EVO2_REFERENCE_ROOT)")
    main(root)
