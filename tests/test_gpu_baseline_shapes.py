"""Parity at the BASELINE shapes, against the CPU oracle on the same seeded inputs.

  config 2  7B triple prefill: H = 4096, fp8 in_proj, 8192-token segments and a
            continuation chunk that resumes from the paged state, for each of
            HCS (K=7), HCM (K=128) and HCL (order 16), through the mixer modules
            (quantiser, e4m3 GEMM, prefill core, out_proj) and through the core
            alone at two full 8192-token segments;
  config 3  7B decode: 128 requests, ordinary single-token steps and one q = 4
            speculative verify step whose accepted counts are resolved from the
            position stamps on the device;
  config 5  one channel shard of the 40B shape (H = 8192 split over 2 ranks):
            the rank-0 shard's fp8 in_proj (12288 x 8192), core and row-parallel
            out_proj partial (8192 x 4096, bias on rank 0), before the all-reduce.

Every bf16 output is held to the path's bar, max|a-b| / max|b| <= 2e-2, and to
the same bar per token row and per channel (max_slice_rel_err), so that a wrong
small-magnitude row or channel cannot hide behind the tensor's maximum.  Copied
windows must match bit for bit; the LI modal state within 1e-4 relative."""

from types import SimpleNamespace

import pytest
import torch

from oracle import hyena_oracle as O
from tests.helpers import (REL_TOL, decode_meta, max_rel_err, max_slice_rel_err, meta_to,
                           prefill_meta, spec_accepted)

pytestmark = pytest.mark.gpu
DEV = "cuda"
H7 = 4096
KINDS = [("hcs", 7), ("hcm", 128), ("hcl", 16)]


def _tensors(kind, k, H, seed, fp8=True):
    from evo2_flash_b200.synthetic import mixer_tensors

    t = mixer_tensors(kind, H, k, seed, fp8=fp8)
    t["out_proj.bias"] = torch.randn(H, generator=torch.Generator().manual_seed(seed)).mul(
        0.02).to(torch.bfloat16)
    if fp8:
        t["in_proj.input_scale"] = torch.tensor([8.0 / 448.0])
    return t


def _oracle_params(t, kind, k, H):
    fp8 = t["in_proj.weight"].dtype == torch.float8_e4m3fn
    return O.MixerParams(
        H=H, kind="iir" if kind == "hcl" else "fir", k_inner=k, short_filter=t["short_filter"],
        conv=t.get("conv"), D=t.get("D"), log_poles=t.get("log_poles"), residues=t.get("residues"),
        in_proj_weight=t["in_proj.weight"],
        in_proj_scales=(t["in_proj.input_scale"], t["in_proj.weight_scale"]) if fp8 else None,
        out_proj_weight=t["out_proj.weight"], out_proj_bias=t["out_proj.bias"])


def _mixer(kind, k, H, t, num_blocks, tp_rank=0, tp_size=1, num_spec=0):
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=True)
    kw = dict(tp_rank=tp_rank, tp_size=tp_size, device=DEV, num_spec=num_spec)
    m = (HyenaIIRMixer(cfg, 0, prefix="baseline", **kw) if kind == "hcl"
         else HyenaFIRMixer(cfg, 0, prefix="baseline", k_inner=k, **kw))
    m.load_full_weights({kk: v.to(DEV) for kk, v in t.items()})
    m.allocate_state(num_blocks, DEV)
    return m


def _hidden(T, H, seed):
    """Mixer inputs as the bench feeds them: RMS-normed N(0,1) embeddings of
    uniform ACGT tokens."""
    g = torch.Generator().manual_seed(seed)
    table = torch.randn(512, H, generator=g)
    ids = torch.tensor([65, 67, 71, 84])[torch.randint(0, 4, (T,), generator=g)]
    x = table[ids]
    return (x / (x.norm(dim=-1, keepdim=True) * H ** -0.5 + 1e-6)).to(torch.bfloat16)


def _check_states(kind, k, got, want):
    """Same z in, same state out: windows bit for bit, modal state to 1e-4."""
    assert torch.equal(got[0].cpu(), want[0])
    if kind == "hcl":
        assert max_rel_err(got[2].cpu(), want[2]) < 1e-4
    else:
        assert torch.equal(got[1].cpu()[:, : k - 1], want[1][:, : k - 1])


def _check_states_after_gemm(kind, k, got, want):
    """Through the modules the windows hold in_proj outputs, which the e4m3
    GEMM (fp32 accumulation in tcgen05 order) and the oracle (float64) round
    to bf16 differently in the last bit now and then: windows within bf16
    rounding, the modal state within 1e-3."""
    assert max_rel_err(got[0].cpu(), want[0]) < 1e-2
    if kind == "hcl":
        assert max_rel_err(got[2].cpu(), want[2]) < 1e-3
    else:
        assert max_rel_err(got[1].cpu()[:, : k - 1], want[1][:, : k - 1]) < REL_TOL


def _ref_states(m):
    return [s.cpu().clone() for s in m.kv_cache]


@pytest.mark.parametrize("kind,k", KINDS)
def test_config2_mixer_fp8_prefill_and_continuation(kind, k):
    from evo2_flash_b200 import set_forward_metadata

    t = _tensors(kind, k, H7, seed=201 + k)
    m = _mixer(kind, k, H7, t, 4)
    po = _oracle_params(t, kind, k, H7)
    ref_states = _ref_states(m)
    steps = [([8192, 700], [1, 2], [False, False]),   # fresh 8192-token segment
             ([1024, 300], [1, 3], [True, False])]    # continue block 1, fresh block 3
    for i, (lengths, blocks, init) in enumerate(steps):
        x = _hidden(sum(lengths), H7, seed=210 + i)
        meta = prefill_meta(lengths, blocks, init)
        ref = O.mixer_forward(x, po, meta, ref_states)
        with set_forward_metadata(meta_to(meta, DEV)):
            out = m(x.to(DEV)).cpu()
        assert max_rel_err(out, ref) < REL_TOL, i
        assert max_slice_rel_err(out, ref) < REL_TOL, i
    _check_states_after_gemm(kind, k, m.kv_cache, ref_states)


@pytest.mark.parametrize("kind,k", KINDS)
def test_config2_core_two_full_segments(kind, k):
    """The prefill core alone on z with the in_proj's statistics: two fresh
    8192-token segments, then a continuation of each."""
    from evo2_flash_b200 import ops
    from tests.test_gpu_kernels import _weights

    t = _tensors(kind, k, H7, seed=221 + k, fp8=False)
    po = _oracle_params(t, kind, k, H7)
    w = _weights({kk: v.to(DEV) for kk, v in t.items()}, kind)
    states = [torch.zeros(3, 2, 3 * H7, dtype=torch.bfloat16), torch.zeros(3, 127, H7),
              torch.zeros(3, H7, 16)]
    ds = [s.to(DEV) for s in states]
    g = torch.Generator().manual_seed(222)
    for lengths, init in (([8192, 8192], [False, False]), ([513, 2048], [True, True])):
        T = sum(lengths)
        z = (torch.randn(T, 3 * H7, generator=g) * 0.7).to(torch.bfloat16)
        meta = prefill_meta(lengths, [1, 2], init)
        ref = O.mixer_core(z, po, meta, states, None, bf16_products=True)
        out = torch.empty(T, H7, dtype=torch.bfloat16, device=DEV)
        dm = meta_to(meta, DEV)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        ops.prefill(w, z.to(DEV), out, dm.query_start_loc_p, dm.has_initial_states_p,
                    dm.state_indices_tensor_p, ds[0], ds[2] if kind == "hcl" else ds[1],
                    error_flags=flags)
        torch.cuda.synchronize()
        assert int(flags.item()) == 0
        assert max_rel_err(out.cpu(), ref) < REL_TOL
        assert max_slice_rel_err(out.cpu(), ref) < REL_TOL
    _check_states(kind, k, ds, states)


def _random_states(H, nb, W0, seed, spec_col):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(nb, W0, 3 * H, generator=g) * 0.3).to(torch.bfloat16),
            (torch.randn(nb, 127, H, generator=g) * 0.1).to(torch.bfloat16).float(),
            torch.randn(nb, H, 17 if spec_col else 16, generator=g) * 0.5]


@pytest.mark.parametrize("kind,k", KINDS)
def test_config3_decode_128_requests(kind, k):
    """128 requests in scattered blocks, three single-token steps (the q = 1
    kernels of the SD layout)."""
    from evo2_flash_b200 import ops
    from tests.test_gpu_kernels import _weights

    B = 128
    t = _tensors(kind, k, H7, seed=231 + k, fp8=False)
    po = _oracle_params(t, kind, k, H7)
    w = _weights({kk: v.to(DEV) for kk, v in t.items()}, kind)
    nb = 2 * B + 1
    states = _random_states(H7, nb, 2, seed=232, spec_col=False)
    ds = [s.to(DEV) for s in states]
    slots = torch.randperm(nb - 1, generator=torch.Generator().manual_seed(233))[:B].add(1)
    idx = slots.int().to(DEV)
    g = torch.Generator().manual_seed(234)
    for _ in range(3):
        z = (torch.randn(B, 3 * H7, generator=g) * 0.7).to(torch.bfloat16)
        ref = O.mixer_core(z, po, decode_meta(slots.tolist()), states, None, bf16_products=True)
        out = torch.empty(B, H7, dtype=torch.bfloat16, device=DEV)
        ops.decode(w, z.to(DEV), out, idx, idx, idx[:, None], idx[:, None], ds[0],
                   ds[2] if kind == "hcl" else ds[1], zero_null_rows=True)
        torch.cuda.synchronize()
        assert max_rel_err(out.cpu(), ref) < REL_TOL
        assert max_slice_rel_err(out.cpu(), ref) < REL_TOL
    _check_states(kind, k, ds, states)


@pytest.mark.parametrize("kind,k", KINDS)
def test_config3_verify_q4_stamp_resolved(kind, k):
    """One speculative verify step (anchor + 3 drafts) for 128 requests with
    ragged draft counts; the accepted count of the previous step (1..4) is
    resolved from the position stamps by hyena_spec_accepted on the device and
    must equal the host rule before it drives the verify kernel."""
    from evo2_flash_b200 import ops
    from tests.test_gpu_kernels import _weights

    B, q, ns = 128, 4, 3
    t = _tensors(kind, k, H7, seed=241 + k, fp8=False)
    po = _oracle_params(t, kind, k, H7)
    w = _weights({kk: v.to(DEV) for kk, v in t.items()}, kind)
    nb = q * B + 1
    states = _random_states(H7, nb, 2 + ns, seed=242, spec_col=True)
    gen = torch.Generator().manual_seed(243)
    slots = (torch.randperm(nb - 1, generator=gen)[: q * B].add(1)).view(B, q)
    lengths = torch.randint(1, q + 1, (B,), generator=gen)
    prev_acc = torch.randint(1, q + 1, (B,), generator=gen)
    computed = torch.randint(100, 5000, (B,), generator=gen)
    states[2][slots[:, 0], 0, 16] = (computed - (prev_acc - 1)).float()
    meta = decode_meta(slots.tolist(), lengths.tolist(), computed=computed.tolist())
    acc_ref = spec_accepted(meta, states[2][:, 0, 16], ns)
    assert torch.equal(acc_ref, prev_acc)
    ds = [s.to(DEV) for s in states]
    dslots = slots.int().to(DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    acc = ops.spec_accepted(dslots, computed.int().to(DEV), ds[2][:, 0, 16], ns,
                            error_flags=flags)
    T = int(lengths.sum())
    z = (torch.randn(T, 3 * H7, generator=gen) * 0.7).to(torch.bfloat16)
    ref = O.mixer_core(z, po, meta, states, acc_ref, bf16_products=True)
    starts = torch.cat([torch.zeros(1, dtype=torch.long), lengths.cumsum(0)]).int().to(DEV)
    out = torch.empty(T, H7, dtype=torch.bfloat16, device=DEV)
    ops.decode(w, z.to(DEV), out, dslots[:, 0], dslots[:, 0], dslots, dslots, ds[0],
               ds[2] if kind == "hcl" else ds[1], token_start=starts, accepted=acc,
               error_flags=flags)
    torch.cuda.synchronize()
    assert torch.equal(acc.cpu().long(), prev_acc)
    assert int(flags.item()) == 0
    assert max_rel_err(out.cpu(), ref) < REL_TOL
    assert max_slice_rel_err(out.cpu(), ref) < REL_TOL
    assert torch.equal(ds[0].cpu()[1:], states[0][1:])
    if kind == "hcl":
        assert max_rel_err(ds[2].cpu()[1:, :, :16], states[2][1:, :, :16]) < 1e-4
    else:
        assert torch.equal(ds[1].cpu()[1:, : k - 1], states[1][1:, : k - 1])


@pytest.mark.parametrize("kind,k", KINDS)
def test_config5_rank0_shard_of_the_40b_shape(kind, k):
    """The rank-0 channel shard of a 40B-shape layer (H = 8192 over 2 ranks):
    fp8 in_proj rows of its 4096 channels, the core, and the row-parallel
    out_proj partial with the bias added once (on rank 0), before the
    all-reduce; a fresh 4096-token segment, then a continuation."""
    from evo2_flash_b200 import set_forward_metadata
    from evo2_flash_b200.parallel import shard_mixer_tensors

    H = 8192
    full = _tensors(kind, k, H, seed=251 + k)
    shard = shard_mixer_tensors(full, 0, 2, H)
    m = _mixer(kind, k, H, full, 3, tp_rank=0, tp_size=2)
    hl = H // 2
    po = _oracle_params(shard, kind, k, hl)
    ref_states = _ref_states(m)
    for i, (lengths, init) in enumerate((([4096], [False]), ([640], [True]))):
        x = _hidden(sum(lengths), H, seed=252 + i)
        meta = prefill_meta(lengths, [1], init)
        z = O.in_proj(x, po)
        g = O.mixer_core(z, po, meta, ref_states, None, bf16_products=True)
        ref = (g.float() @ po.out_proj_weight.float().t() + po.out_proj_bias.float()).to(
            torch.bfloat16)
        with set_forward_metadata(meta_to(meta, DEV)):
            dz = m._project(x.to(DEV))
            dg = m._run_core(dz, meta_to(meta, DEV), None)
            part, _ = m.out_proj(dg)
        out = part.cpu()
        assert max_rel_err(out, ref) < REL_TOL, i
        assert max_slice_rel_err(out, ref) < REL_TOL, i
    _check_states_after_gemm(kind, k, m.kv_cache, ref_states)
