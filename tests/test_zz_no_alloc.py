"""vt_attn_fwd_noalloc, the attention entry point for callers that cannot allocate device memory (code
running during CUDA-graph stream capture, hosts with a device-memory budget fixed at start-up, plain C /
FFI callers without a device allocator).  It keeps the attention tiles in the library's fixed 16 MiB
device array instead of a caller-owned buffer; here it is called through the C ABI and compared with the
caller-owned-buffer path (vt_attn_pack + vt_attn_tiles_fwd, via VtAttn) on two calls in a row.  The
second call uses a smaller problem than the first, so stale tiles from the first call would show.

This file is named to be collected last: if it fails, a run that stops at the first failure has already
run every other test."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import ops
from strix_halo_maxx_b200._lib import lib, device_status

DEV = "cuda"
BF = torch.bfloat16
ATTN_TOL = 1e-2   # the tolerance of the other attention tests (tests/test_kernels_gpu.py)


def _noalloc(q, k, v, out):
    B, H, T, D = q.shape
    return lib().vt_attn_fwd_noalloc(torch.cuda.current_stream().cuda_stream, q.data_ptr(), k.data_ptr(),
                                     v.data_ptr(), out.data_ptr(), B, T, H, D, q.stride(0), q.stride(2), q.stride(1),
                                     k.stride(0), k.stride(2), k.stride(1), v.stride(0), v.stride(2), v.stride(1),
                                     out.stride(0), out.stride(1), D, D ** -0.5)


def test_noalloc_matches_caller_buffer_path_on_two_calls_in_a_row():
    device_status(clear=True)
    for call, (B, H, T, D) in enumerate([(2, 16, 729, 72), (1, 12, 1280, 64)]):
        qkv = torch.randn(B, T, 3 * H * D, device=DEV, generator=torch.Generator(DEV).manual_seed(call)).to(BF)
        q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
        ref = ops.VtAttn(H, T, D)(q, k, v)
        out = torch.full((B, T, H * D), float("nan"), device=DEV, dtype=BF)
        assert _noalloc(q, k, v, out) == 0, lib().vt_last_error_string()
        torch.cuda.synchronize()
        err = float((out.float() - ref.float()).norm() / ref.float().norm())
        assert err < ATTN_TOL, (call, err)
    assert device_status(clear=True) == 0


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    B, H, T, D = 3, 16, 729, 72          # 17.7 MB of tiles > 16 MiB
    qkv = torch.zeros(B, T, 3 * H * D, device=DEV, dtype=BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = torch.empty(B, T, H * D, device=DEV, dtype=BF)
    assert _noalloc(q, k, v, out) == -2
    assert b"16777216-byte scratch" in lib().vt_last_error_string()
