"""The C-ABI library loads and exports exactly what include/vt_b200.h declares (no compute calls)."""
import ctypes
import os
import re

import pytest

from strix_halo_maxx_b200 import build
from strix_halo_maxx_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vt_b200.h")


def header_decls():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = {}
    for m in re.finditer(r"^\s*(?:const\s+)?(?:(?:unsigned|long)\s+)*\w+\**\s+\**(vt_\w+)\s*\(([^;]*?)\)\s*;", src, flags=re.M | re.S):
        args = m.group(2).strip()
        n = 0 if args in ("", "void") else len(args.split(","))
        decls[m.group(1)] = n
    return decls


@pytest.fixture(scope="module")
def lib():
    build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_matches_binding_table():
    decls = header_decls()
    assert set(decls) == set(_lib.SIGNATURES), (set(decls) ^ set(_lib.SIGNATURES))
    for name, n in decls.items():
        assert len(_lib.SIGNATURES[name][1]) == n, (name, n, len(_lib.SIGNATURES[name][1]))


def test_library_exports_every_declared_symbol(lib):
    for name in header_decls():
        assert hasattr(lib, name), name


def test_binding_loads_and_reports_version():
    assert _lib.lib().vt_abi_version() == 1


def test_errors_are_reported_without_a_gpu():
    # shape validation happens on the host before any CUDA call
    L = _lib.lib()
    rc = L.vt_gemm_bf16(None, 16, 588, 16, 588, None, 16, 8, 4, 8, 588, 0)
    assert rc == -2 and b"16-byte" in L.vt_last_error_string()
    rc = L.vt_attn_tiles_fwd(None, 16, 16, 1, 10, 2, 72 + 4, 8, 8, 8, 1.0)
    assert rc == -1 and b"head_dim" in L.vt_last_error_string()
    rc = L.vt_attn_pack(None, 16, 16, 16, 16, 1, 10, 2, 72, *([4] * 9))
    assert rc == -2 and b"multiples of 8" in L.vt_last_error_string()


def test_int8_entry_points_validate_on_the_host():
    """The W8A8 entry points reject bad shapes / scales before any CUDA call."""
    L = _lib.lib()
    # K not a multiple of 8
    assert L.vt_quant_rows(None, 16, 16, 4, 12, 16, 16, 16) == -2
    assert b"multiple of 8" in L.vt_last_error_string()
    # missing scales
    assert L.vt_gemm_i8(None, 16, 64, 16, 64, None, None, 4, 8, 64, None, 16, 8, 0, 0, None, 0, 0, None, 0) == -2
    assert b"scales" in L.vt_last_error_string()
    # LayerNorm width not a multiple of 4
    assert L.vt_layernorm_quant(None, 16, 16, 0, 16, 16, 4, 6, 1e-5, 16, 16, 16, None, 0) == -2
    # empty problems are no-ops
    assert L.vt_quant_rows(None, 16, 16, 0, 16, 16, 16, 16) == 0
    assert L.vt_gemm_i8(None, 16, 64, 16, 64, None, None, 0, 8, 64, None, 16, 8, 0, 0, None, 0, 0, None, 0) == 0


def test_fused_gemm_and_head_entry_points_validate_on_the_host():
    """vt_gemm_fused_lnstats, the gated GELU mode of vt_gemm_fused_ws and vt_head_linear reject bad arguments
    before any CUDA call (fake 16-byte aligned addresses, never dereferenced)."""
    L = _lib.lib()
    A = W = O = S = 4096
    common = (None, A, 64, W, 64, 4, 64, 64, None, O, 64, 0)   # stream .. out_f32 (M 4, N 64, K 64)
    tail = (None, 0, 0, 0, None, 0, None)                      # res, ldr, res_period, res_bf16, out2, ldo2, stats_out
    # no chunk statistics
    assert L.vt_gemm_fused_lnstats(*common, 0, *tail, None, 2, 1e-6, 0, S, None, 0, 0, 0, None, 0) == -2
    assert b"ln_stats is required" in L.vt_last_error_string()
    # statistics without the rowsum vector ln_c
    assert L.vt_gemm_fused_lnstats(*common, 0, *tail, S, 2, 1e-6, 0, None, None, 0, 0, 0, None, 0) == -1
    assert b"chunk statistics" in L.vt_last_error_string()
    # the gated GELU needs N % 32 == 0 (N = 48 here) and a bf16 output
    gated = (None, A, 64, W, 64, 4, 48, 64, None, O, 64, 0, 2)
    assert L.vt_gemm_fused_ws(*gated, *tail, None, None, 0, 0, 0, None, 0) == -1
    assert b"gated GELU" in L.vt_last_error_string()
    # head GEMM: K = 0
    assert L.vt_head_linear(None, A, 64, 1, W, 64, None, O, 64, 4, 64, 0) == -2
