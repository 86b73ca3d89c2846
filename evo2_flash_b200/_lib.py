"""ctypes binding of `libhyena_b200.so` (the C ABI in include/hyena_b200.h).

The library is built in-tree by `evo2_flash_b200._build.build()`.  Loading fails
loudly when it is missing: there is no fallback implementation of any kernel.
"""

from __future__ import annotations

import ctypes as C
import threading

from ._build import LIB_PATH

HYENA_KIND_FIR = 0
HYENA_KIND_IIR = 1
ABI_VERSION = 8


class StateView(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("block_stride", C.c_int64),
        ("col_stride", C.c_int64),
        ("dim_stride", C.c_int64),
        ("cols", C.c_int32),
        ("num_blocks", C.c_int32),
    ]


class LayerParams(C.Structure):
    _fields_ = [
        ("kind", C.c_int32),
        ("H", C.c_int32),
        ("K", C.c_int32),
        ("short_w", C.c_void_p),
        ("inner_w", C.c_void_p),
        ("inner_w_stride_h", C.c_int64),
        ("inner_w_stride_k", C.c_int64),
        ("log_poles", C.c_void_p),
        ("lp_stride_h", C.c_int64),
        ("lp_stride_s", C.c_int64),
        ("residues", C.c_void_p),
        ("res_stride_h", C.c_int64),
        ("res_stride_s", C.c_int64),
        ("D", C.c_void_p),
    ]


class PrefillArgs(C.Structure):
    _fields_ = [
        ("z", C.c_void_p),
        ("ldz", C.c_int64),
        ("out", C.c_void_p),
        ("ldo", C.c_int64),
        ("T", C.c_int32),
        ("num_segments", C.c_int32),
        ("query_start_loc", C.c_void_p),
        ("has_initial_state", C.c_void_p),
        ("state_indices", C.c_void_p),
        ("state_indices_stride", C.c_int64),
        ("conv_state", StateView),
        ("inner_state", StateView),
        ("error_flags", C.c_void_p),
    ]


class StateBlock(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("block_stride_bytes", C.c_int64),
        ("block_bytes", C.c_int64),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("z", C.c_void_p),
        ("ldz", C.c_int64),
        ("out", C.c_void_p),
        ("ldo", C.c_int64),
        ("num_reqs", C.c_int32),
        ("q", C.c_int32),
        ("token_start", C.c_void_p),
        ("accepted", C.c_void_p),
        ("conv_in_block", C.c_void_p),
        ("conv_out_block", C.c_void_p),
        ("in_slots", C.c_void_p),
        ("in_stride0", C.c_int64),
        ("in_stride1", C.c_int64),
        ("out_slots", C.c_void_p),
        ("out_stride0", C.c_int64),
        ("out_stride1", C.c_int64),
        ("zero_null_rows", C.c_int32),
        ("skip_null_writes", C.c_int32),
        ("null_block", C.c_int32),
        ("conv_state", StateView),
        ("inner_state", StateView),
        ("error_flags", C.c_void_p),
        ("conv_in_stride", C.c_int64),
        ("conv_out_stride", C.c_int64),
    ]


# Every symbol include/hyena_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "hyena_abi_version": (C.c_int, []),
    "hyena_last_error": (C.c_char_p, []),
    "hyena_prefill_workspace_size": (C.c_size_t, [C.POINTER(LayerParams), C.c_int32, C.c_int32]),
    "hyena_prefill": (C.c_int, [C.POINTER(LayerParams), C.POINTER(PrefillArgs), C.c_void_p,
                                C.c_size_t, C.c_void_p]),
    "hyena_prefill_noalloc": (C.c_int, [C.POINTER(LayerParams), C.POINTER(PrefillArgs),
                                        C.c_void_p]),
    "hyena_decode": (C.c_int, [C.POINTER(LayerParams), C.POINTER(DecodeArgs), C.c_void_p]),
    "hyena_quant_e4m3": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int32,
                                   C.c_int32, C.c_void_p, C.c_void_p]),
    "hyena_gemm_e4m3": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                  C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "hyena_gemm_bf16": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                  C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                  C.c_void_p, C.c_size_t, C.c_void_p]),
    "hyena_rms_norm": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                 C.c_float, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                 C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_int32,
                                 C.c_void_p]),
    "hyena_gemm_fp8_emulated": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                          C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                          C.c_void_p, C.c_void_p, C.c_void_p]),
    "hyena_gemm_workspace_size": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "hyena_set_gemm_max_ctas": (None, [C.c_int32]),
    "hyena_gemm_wait_timeouts": (C.c_int, [C.POINTER(C.c_int32), C.c_int32]),
    "hyena_set_launch_chaining": (None, [C.c_int32]),
    "hyena_nvls_allreduce_bf16": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int32,
                                            C.c_int32, C.c_uint32, C.c_int32, C.c_void_p,
                                            C.c_void_p]),
    "hyena_spec_accepted": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p,
                                      C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                      C.c_void_p]),
    "hyena_spec_record_prefill": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p,
                                            C.c_void_p, C.c_int64, C.c_int32, C.c_void_p,
                                            C.c_void_p]),
    "hyena_state_repair": (C.c_int, [C.c_int32, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                     C.POINTER(StateBlock), C.c_int32, C.c_void_p, C.c_void_p,
                                     C.c_void_p]),
    "hyena_spec_record": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                    C.c_void_p, C.c_void_p]),
}

_lock = threading.Lock()
_lib = None


def load():
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build the sm_100a kernels first "
                "(python -m evo2_flash_b200._build, or __graft_entry__.build())")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.hyena_abi_version() != ABI_VERSION:
            raise ImportError("libhyena_b200.so ABI version mismatch; rebuild it")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().hyena_last_error().decode(errors="replace")
        if rc == 1:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")
