"""vt_attn_fwd_noalloc, the attention entry point for callers that cannot allocate device memory: hosts that
fix their device-memory budget at start-up and allow no allocation while serving, and plain C / FFI callers
that have no device allocator to hand out a scratch buffer.  It keeps the attention tiles in the library's
fixed 16 MiB device array instead of a caller-owned buffer.

Here it is called through the C ABI, several calls in a row, and compared with the caller-owned-buffer path
(vt_attn_pack + vt_attn_tiles_fwd, via VtAttn): both run the same kernels on the same tile layout, so the
outputs must be bit-identical; each output is also checked against fp32 SDPA at the attention tolerance of
the other tests.  The first call fills every slot of the scratch it uses with data (1280 tokens, head_dim 64:
no pad rows or lanes); the later calls have pad rows and lanes where that call left data, so a pad not cleared
would show.  Around each call after the warm-up, neither torch's allocator nor the device's free memory may
change.

This file is named to be collected last: if it fails, a run that stops at the first failure has already
run every other test."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import ops
from strix_halo_maxx_b200._lib import lib, device_status

DEV = "cuda"
BF = torch.bfloat16
ATTN_TOL = 1e-2   # the tolerance of the other attention tests (tests/test_kernels_gpu.py)
SHAPES = [(1, 12, 1280, 64), (2, 16, 729, 72), (1, 16, 200, 72)]   # (crops B, heads H, tokens T, head_dim D)


def _noalloc(q, k, v, out):
    B, H, T, D = q.shape
    return lib().vt_attn_fwd_noalloc(torch.cuda.current_stream().cuda_stream, q.data_ptr(), k.data_ptr(),
                                     v.data_ptr(), out.data_ptr(), B, T, H, D, q.stride(0), q.stride(2), q.stride(1),
                                     k.stride(0), k.stride(2), k.stride(1), v.stride(0), v.stride(2), v.stride(1),
                                     out.stride(0), out.stride(1), D, D ** -0.5)


def _qkv(B, H, T, D, seed):
    qkv = torch.randn(B, T, 3 * H * D, device=DEV, generator=torch.Generator(DEV).manual_seed(seed)).to(BF)
    return [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]


def test_noalloc_matches_caller_buffer_path_on_calls_in_a_row():
    device_status(clear=True)
    # warm-up: the first call per device does the set-up (address lookup, kernel attributes); one call per
    # shape also loads every kernel the calls below use before memory is compared
    for i, (B, H, T, D) in enumerate(SHAPES):
        q, k, v = _qkv(B, H, T, D, 100 + i)
        assert _noalloc(q, k, v, torch.empty(B, T, H * D, device=DEV, dtype=BF)) == 0, lib().vt_last_error_string()
    for call, (B, H, T, D) in enumerate(SHAPES):
        q, k, v = _qkv(B, H, T, D, call)
        ref = ops.VtAttn(H, T, D)(q, k, v)
        out = torch.full((B, T, H * D), float("nan"), device=DEV, dtype=BF)
        torch.cuda.synchronize()
        alloc0, free0 = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
        assert _noalloc(q, k, v, out) == 0, lib().vt_last_error_string()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == alloc0, f"call {call}: torch allocated device memory"
        assert torch.cuda.mem_get_info()[0] == free0, f"call {call}: the device's free memory changed"
        assert torch.equal(out, ref), f"call {call}: differs from vt_attn_pack + vt_attn_tiles_fwd"
        sdpa = F.scaled_dot_product_attention(q.float(), k.float(), v.float()).transpose(1, 2).reshape(B, T, -1)
        err = float((out.float() - sdpa).norm() / sdpa.norm())
        assert err < ATTN_TOL, (call, err)
    assert device_status(clear=True) == 0


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    B, H, T, D = 3, 16, 729, 72          # 17.7 MB of tiles > 16 MiB
    qkv = torch.zeros(B, T, 3 * H * D, device=DEV, dtype=BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = torch.empty(B, T, H * D, device=DEV, dtype=BF)
    assert _noalloc(q, k, v, out) == -2
    assert b"16777216-byte scratch" in lib().vt_last_error_string()
