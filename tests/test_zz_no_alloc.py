"""hyena_prefill_noalloc: prefill for callers that cannot allocate device memory.

Some hosts reach this library only through its C ABI and have no CUDA allocator
to hand it a workspace (a Go, Java or Rust program over cgo/JNI/FFI), and a
serving loop may not call cudaMalloc once it runs, since cudaMalloc can
synchronise the device.  This entry point keeps the LI prefill's scratch in a fixed
device array inside the library instead.  The test calls it through the C ABI
twice in a row (a fresh prefill, then a continuation that reads the state the
first call wrote) and compares output and paged state with hyena_prefill run
with a torch-allocated workspace on identical inputs.  It lives in its own file,
collected last, and needs nothing from earlier tests.
"""

import ctypes as C

import pytest
import torch

from tests.helpers import REL_TOL, max_rel_err, prefill_meta, random_params

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _noalloc_prefill(w, z, out, meta, conv_state, inner_state):
    """Calls hyena_prefill_noalloc with the argument structs hyena_prefill takes."""
    from evo2_flash_b200 import _lib, ops
    from evo2_flash_b200._lib import PrefillArgs

    n = meta.num_prefills
    qsl = meta.query_start_loc_p.to(torch.int32).contiguous()
    idx = meta.state_indices_tensor_p.to(torch.int32).contiguous()
    flags = meta.has_initial_states_p.contiguous().view(torch.uint8)
    a = PrefillArgs()
    a.z, a.ldz = z.data_ptr(), z.stride(0)
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.T, a.num_segments = z.shape[0], n
    a.query_start_loc = qsl.data_ptr()
    a.has_initial_state = flags.data_ptr()
    a.state_indices, a.state_indices_stride = idx.data_ptr(), 1
    a.conv_state = ops.state_view(conv_state, 1, 2)
    a.inner_state = ops.state_view(inner_state, 2, 1, cols=16)
    p = w.params()
    lib = _lib.load()
    rc = lib.hyena_prefill_noalloc(C.byref(p), C.byref(a),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return rc, lib.hyena_last_error().decode()


def test_noalloc_prefill_matches_workspace_prefill_on_two_calls():
    from evo2_flash_b200 import ops

    H = 256
    p = {k: v.to(DEV) for k, v in random_params("hcl", H, 16, seed=91).items()}
    w = ops.layer_weights("iir", p["short_filter"], D=p["D"], log_poles=p["log_poles"],
                          residues=p["residues"])
    g = torch.Generator().manual_seed(92)
    ref_states = [torch.zeros(6, 2, 3 * H, dtype=torch.bfloat16, device=DEV),
                  torch.zeros(6, 127, H, device=DEV), torch.zeros(6, H, 16, device=DEV)]
    new_states = [s.clone() for s in ref_states]
    steps = [([700, 300], [1, 2], [False, False]),   # fresh sequences
             ([50, 900], [1, 3], [True, False])]     # continue block 1, start block 3
    for lengths, blocks, init in steps:
        T = sum(lengths)
        z = (torch.randn(T, 3 * H, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        meta = prefill_meta(lengths, blocks, init, device=DEV)
        ref = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
        ops.prefill(w, z, ref, meta.query_start_loc_p, meta.has_initial_states_p,
                    meta.state_indices_tensor_p, ref_states[0], ref_states[2])
        out = torch.full((T, H), 7.0, dtype=torch.bfloat16, device=DEV)
        rc, msg = _noalloc_prefill(w, z, out, meta, new_states[0], new_states[2])
        assert rc == 0, msg
        assert max_rel_err(out, ref) < REL_TOL
        assert torch.equal(new_states[0], ref_states[0])
        assert torch.equal(new_states[2], ref_states[2])  # the same kernels run


def test_noalloc_prefill_rejects_a_step_beyond_the_scratch():
    from evo2_flash_b200 import _lib
    from evo2_flash_b200._lib import LayerParams, PrefillArgs

    p = LayerParams()
    p.kind, p.H, p.K = _lib.HYENA_KIND_IIR, 4096, 16
    p.short_w, p.log_poles, p.residues = 1, 1, 1  # rejected before any is read
    a = PrefillArgs()
    # one 256 KiB modal state per segment (H = 4096): 200 segments need ~50 MiB
    a.T, a.num_segments = 1 << 20, 200
    lib = _lib.load()
    assert lib.hyena_prefill_workspace_size(C.byref(p), a.T, a.num_segments) > 32 << 20
    assert lib.hyena_prefill_noalloc(C.byref(p), C.byref(a), None) == 1
    assert b"32 MiB" in lib.hyena_last_error()
