"""The C-ABI library (CPU-side checks; nothing here launches a kernel):
it loads, exports exactly the entry points include/hyena_b200.h declares, and
rejects invalid arguments on the host before touching the device."""

import ctypes as C
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "hyena_b200.h").read_text()
    return set(re.findall(r"HYENA_API\s+[\w\s\*]+?\b(hyena_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from evo2_flash_b200 import _build, _lib

    _build.build()
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {"hyena_prefill", "hyena_decode", "hyena_gemm_e4m3", "hyena_gemm_bf16",
            "hyena_quant_e4m3", "hyena_prefill_workspace_size"} <= syms


def test_library_exports_every_declared_symbol(lib):
    from evo2_flash_b200 import _lib

    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.hyena_abi_version() == _lib.ABI_VERSION


def test_invalid_arguments_are_rejected_on_host(lib):
    from evo2_flash_b200._lib import LayerParams, PrefillArgs

    p = LayerParams()
    p.kind, p.H, p.K = 0, 100, 128  # H not a multiple of 64
    a = PrefillArgs()
    rc = lib.hyena_prefill(C.byref(p), C.byref(a), None, 0, None)
    assert rc == 1
    assert b"multiple of 64" in lib.hyena_last_error()
    p.H, p.K = 128, 9  # unsupported taps
    assert lib.hyena_prefill(C.byref(p), C.byref(a), None, 0, None) == 1
    # null GEMM operands
    assert lib.hyena_gemm_bf16(None, 64, None, 64, None, 64, 1, 8, 64, None, None, 0, None) == 1


def test_empty_work_is_a_no_op(lib):
    from evo2_flash_b200._lib import LayerParams, PrefillArgs

    p = LayerParams()
    p.kind, p.H, p.K = 0, 128, 7
    p.short_w = 1  # never dereferenced: no segments
    p.inner_w = 1
    a = PrefillArgs()
    a.T, a.num_segments = 0, 0
    assert lib.hyena_prefill(C.byref(p), C.byref(a), None, 0, None) == 0


def test_workspace_size_only_for_li(lib):
    from evo2_flash_b200._lib import LayerParams

    p = LayerParams()
    p.kind, p.H, p.K = 0, 4096, 128
    assert lib.hyena_prefill_workspace_size(C.byref(p), 65536, 8) == 0
    p.kind, p.K = 1, 16
    state = 4096 * 16 * 4  # one (H, 16) fp32 modal state
    n = lib.hyena_prefill_workspace_size(C.byref(p), 65536, 8)
    # a 256-byte range table, then one state per range: at least one range per
    # segment plus one for a segment that is split
    assert (n - 256) % state == 0 and (n - 256) // state >= 9
    # ranges grow with the tokens only until the grid is full: 16x the tokens
    # needs far less than 16x the scratch
    n16 = lib.hyena_prefill_workspace_size(C.byref(p), 16 * 65536, 8)
    assert n16 < 2 * n


def test_gemms_need_no_workspace(lib):
    # decode-sized GEMMs reduce their K slices inside a thread-block cluster
    for m in (0, 1, 128, 65536):
        assert lib.hyena_gemm_workspace_size(m, 12288, 4096, 1) == 0
        assert lib.hyena_gemm_workspace_size(m, 4096, 4096, 0) == 0


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "hyena_b200.h"
int main(void) {
  if (hyena_abi_version() != HYENA_ABI_VERSION) return 2;
  hyena_layer_params p;
  memset(&p, 0, sizeof p);
  p.kind = HYENA_KIND_IIR; p.H = 4096; p.K = 16;
  size_t ws = hyena_prefill_workspace_size(&p, 65536, 8);
  hyena_prefill_args a;
  memset(&a, 0, sizeof a);
  p.kind = HYENA_KIND_FIR; p.H = 100; p.K = 128;
  int rc = hyena_prefill(&p, &a, NULL, 0, NULL);
  printf("%zu %d %s\n", ws, rc, hyena_last_error());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_host_program_builds_and_calls_the_abi(lib, tmp_path):
    """A plain C host (no torch, no Python) compiles against the header with
    warnings as errors, links the library and gets host-side answers from it:
    the workspace query and an argument rejected before any device work."""
    from evo2_flash_b200._build import LIB_DIR

    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                    str(src), f"-L{LIB_DIR}", "-lhyena_b200", f"-Wl,-rpath,{LIB_DIR}",
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split(" ", 2)
    from evo2_flash_b200._lib import LayerParams

    lp = LayerParams()
    lp.kind, lp.H, lp.K = 1, 4096, 16
    assert int(out[0]) == lib.hyena_prefill_workspace_size(C.byref(lp), 65536, 8)
    assert int(out[1]) == 1 and "multiple of 64" in out[2]
