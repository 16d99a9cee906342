"""ctypes binding of libvt_b200.so, loaded the way the reference loads its HIP libraries
(moondream/gpu/hgemm.py:21-33, moondream/gpu/hattn.py:5-16): one CDLL, argtypes set once, every call
on torch's current stream, negative return codes turned into exceptions (the reference asserts rc == 0,
hgemm.py:176).  There is no fallback: if the library is missing the import of an op raises.
"""
import ctypes
import os

_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_DIR, "libvt_b200.so")

P, I, LL, F, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_uint

# name -> (restype, argtypes); must match include/vt_b200.h (tests check both directions)
SIGNATURES = {
    "vt_abi_version": (I, []),
    "vt_last_error_string": (ctypes.c_char_p, []),
    "vt_device_status": (I, [I, ctypes.POINTER(U)]),
    "vt_wait_selftest": (I, [P, LL, P]),
    "vt_gemm_bf16": (I, [P, P, LL, P, LL, P, P, LL, I, I, I, I]),
    "vt_gemm_ex": (I, [P, P, LL, P, LL, I, I, I, P, P, LL, I, I, P, LL, I, I, P, LL]),
    "vt_gemm_qkv_tiles": (I, [P, P, LL, P, LL, P, P, I, I, I, I, I]),
    "vt_gemm_fused": (I, [P, P, LL, P, LL, I, I, I, P, P, LL, I, I, P, LL, I, I, P, LL, P, P, P, I, I, I]),
    "vt_gemm_ws_bytes": (LL, [I, I]),
    "vt_gemm_fused_ws": (I, [P, P, LL, P, LL, I, I, I, P, P, LL, I, I, P, LL, I, I, P, LL, P, P, P, I, I, I, P, LL]),
    "vt_gemm_fused_lnstats": (I, [P, P, LL, P, LL, I, I, I, P, P, LL, I, I, P, LL, I, I, P, LL, P, P, I, F, I, P, P, I, I,
                                  I, P, LL]),
    "vt_quant_rows": (I, [P, P, LL, I, I, P, LL, P]),
    "vt_layernorm_quant": (I, [P, P, LL, I, P, P, I, I, F, P, LL, P, P, LL]),
    "vt_gemm_i8": (I, [P, P, LL, P, LL, P, P, I, I, I, P, P, LL, I, I, P, LL, I, P, LL]),
    "vt_rowstats": (I, [P, P, LL, P, LL, P, I, I]),
    "vt_row_moments": (I, [P, P, I, I, F, P]),
    "vt_attn_tiles_bytes": (LL, [I, I, I, I]),
    "vt_attn_pack": (I, [P, P, P, P, P, I, I, I, I, LL, LL, LL, LL, LL, LL, LL, LL, LL]),
    "vt_attn_tiles_fwd": (I, [P, P, P, I, I, I, I, LL, LL, LL, F]),
    "vt_head_linear": (I, [P, P, LL, I, P, LL, P, P, LL, I, I, I]),
    "vt_head_ln_gelu": (I, [P, P, LL, I, I, P, P, I, F]),
    "vt_soft_argmax": (I, [P, P, LL, I, I, I, F, P, LL]),
    "vt_attn_fwd_noalloc": (I, [P, P, P, P, P, I, I, I, I, LL, LL, LL, LL, LL, LL, LL, LL, LL, LL, LL, LL, F]),
    "vt_layernorm": (I, [P, P, LL, I, P, P, P, LL, I, I, I, F]),
    "vt_rmsnorm": (I, [P, P, LL, I, P, P, LL, I, I, I, F]),
    "vt_im2col": (I, [P, P, I, I, I, I, I, P, LL]),
    "vt_crop_combine": (I, [P, P, LL, LL, I, I, I, P, LL]),
    "vt_row_rms": (I, [P, P, I, I, F, P]),
    "vt_rglru_fold": (I, [P, P, LL, P, P, P, P, LL, P, LL, P, LL, P, I, I, F, I]),
    "vt_rglru": (I, [P, P, LL, P, P, LL, P, LL, P, LL, I, I, F, I]),
    "vt_ssm_step": (I, [P, P, P, LL, P, P, P, LL, P, LL, P, P, P, P, P, P, P, P, LL, I, I, I, I]),
    "vt_gated_gelu_mul": (I, [P, P, LL, P, LL, I, I]),
    "vt_gelu_erf": (I, [P, P, LL, I, I]),
    "vt_rope_qkv": (I, [P, P, LL, I, I, I, P, P, P, P, P, I]),
    "vt_attn_causal": (I, [P, P, P, P, I, I, I, I, F, P, LL]),
    "vt_resize_pass_u8": (I, [P, P, LL, LL, LL, P, LL, LL, LL, I, I, P, P, I]),
}


class VtError(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise VtError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                          "or `python -m strix_halo_maxx_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, what):
    if rc != 0:
        msg = lib().vt_last_error_string()
        raise VtError(f"{what} failed with code {rc}: {msg.decode() if msg else ''}")


def device_status(clear=True):
    """Status word the kernels set when a bounded wait gives up (0 = healthy).  Synchronises."""
    s = ctypes.c_uint(0)
    check(lib().vt_device_status(1 if clear else 0, ctypes.byref(s)), "vt_device_status")
    return s.value
