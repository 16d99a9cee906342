"""Kernel parity on the GPU, through the C ABI (ctypes), against plain PyTorch fp32 on the same
bf16-rounded operands.  GEMM shapes: the reference's vision shapes (moondream/gpu/test_hgemm.py:16) plus
tails and edge cases; tolerance rel < 5e-3 as test_hgemm.py:45.  Attention: the reference's
(16, 729, 72) strided QKV layout (hattn.py:48-51) and the TAPNext (12, 1280, 64) case."""
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import ops
from strix_halo_maxx_b200._lib import lib, device_status, VtError

DEV = "cuda"
BF = torch.bfloat16


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm())


@pytest.fixture(autouse=True)
def _status():
    device_status(clear=True)
    yield
    assert device_status(clear=True) == 0, "a kernel recorded a timed-out wait"


def _operands(M, K, N, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(M, K, device=DEV, generator=g).to(BF)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.02).to(BF)
    b = torch.randn(N, device=DEV, generator=g)
    return x, w, b


VIS = [(729, 1152, 3456), (729, 1152, 1152), (729, 1152, 4304), (729, 4304, 1152), (729, 2304, 8192),
       (729, 8192, 2048), (729, 588, 1152)]
EDGE = [(1, 64, 8), (7, 72, 24), (128, 64, 256), (129, 1152, 264), (300, 8, 40), (9477, 1152, 3456), (2048, 4304, 1152)]


@pytest.mark.parametrize("M,K,N", VIS + EDGE)
@pytest.mark.parametrize("gelu", [False, True])
def test_gemm_bf16(M, K, N, gelu):
    x, w, b = _operands(M, K, N)
    lin = ops.VtLin(w, b)
    out = lin(x, gelu=gelu)
    ref = F.linear(x.float(), w.float(), b)
    if gelu:
        ref = F.gelu(ref.to(BF).float(), approximate="tanh")
    assert out.shape == (M, N) and out.dtype == BF
    assert rel(out, ref) < 5e-3


@pytest.mark.parametrize("M,K,N", [(729, 1152, 1152), (1458, 4304, 1152), (77, 200, 96), (730, 2048, 2048),
                                   (730, 1024, 2040)])
@pytest.mark.parametrize("res_dtype", [torch.float32, BF])
def test_gemm_residual(M, K, N, res_dtype):
    x, w, b = _operands(M, K, N, 1)
    res = torch.randn(M, N, device=DEV).to(res_dtype)
    out = ops.VtLin(w, b)(x, res=res)
    ref = F.linear(x.float(), w.float(), b) + res.float()
    assert out.dtype == res_dtype
    assert rel(out, ref) < 5e-3


def test_gemm_inplace_residual_periodic_addend_and_bf16_copy():
    M, K, N, P = 3 * 729, 592, 1152, 729
    x, w, b = _operands(M, K, N, 2)
    pos = torch.randn(P, N, device=DEV)
    out = torch.empty(M, N, device=DEV)
    ops.gemm(x, w, K, K, N, b, res=pos, res_period=P, out=out)
    ref = F.linear(x.float(), w.float(), b) + pos.repeat(3, 1)
    assert rel(out, ref) < 5e-3
    x2 = out.clone()
    copy = torch.empty(M, N, device=DEV, dtype=BF)
    ops.gemm(x, w, K, K, N, b, res=x2, out=x2, out2=copy)       # in place: x2 += x . w^T + b
    ref2 = ref + F.linear(x.float(), w.float(), b)
    assert rel(x2, ref2) < 5e-3
    assert torch.equal(copy, x2.to(BF))


@pytest.mark.parametrize("M,N", [(729, 1152), (1000, 1152), (3 * 729, 1152), (300, 96), (1000, 1184)])
def test_gemm_residual_row_statistics(M, N):
    K = 1152
    x, w, b = _operands(M, K, N, 7)
    res = torch.randn(M, N, device=DEV) * 3 + 1
    out = torch.empty(M, N, device=DEV)
    xb = torch.empty(M, N, device=DEV, dtype=BF)
    stats = torch.empty(M, N // 32, 2, device=DEV)
    ops.gemm(x, w, K, K, N, b, res=res, out=out, out2=xb, stats_out=stats)
    ch = out.view(M, N // 32, 32)
    assert torch.allclose(stats[..., 0], ch.mean(-1), rtol=1e-5, atol=1e-5)
    assert torch.allclose(stats[..., 1], ((ch - ch.mean(-1, keepdim=True)) ** 2).sum(-1), rtol=1e-4, atol=1e-4)
    assert torch.equal(xb, out.to(BF))
    st2 = torch.empty_like(stats)
    xb2 = torch.empty_like(xb)
    ops.row_stats(out, st2, xb2)
    assert torch.allclose(st2, stats, rtol=1e-5, atol=1e-5) and torch.equal(xb2, xb)


@pytest.mark.parametrize("gelu", [False, True])
def test_gemm_folded_layernorm(gelu):
    """LN(x) . W^T + b computed as rstd * (x . (W gamma)^T - mean * rowsum) + b + W beta from row statistics."""
    M, K, N = 1458, 1152, 4304
    g = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(M, K, device=DEV, generator=g) * 2 + 0.3
    w = torch.randn(N, K, device=DEV, generator=g) * 0.02
    b = torch.randn(N, device=DEV, generator=g) * 0.1
    gamma = 1 + 0.1 * torch.randn(K, device=DEV, generator=g)
    beta = 0.05 * torch.randn(K, device=DEV, generator=g)
    stats = torch.empty(M, K // 32, 2, device=DEV)
    xb = torch.empty(M, K, device=DEV, dtype=BF)
    ops.row_stats(x, stats, xb)
    wf, c, bf = ops.fold_layernorm(w, b, gamma, beta)
    mom = ops.row_moments(stats, 1e-6, torch.empty(M, 2, device=DEV))
    assert torch.allclose(mom[:, 0], x.mean(-1), rtol=1e-4, atol=1e-5)
    assert torch.allclose(mom[:, 1], torch.rsqrt(x.var(-1, unbiased=False) + 1e-6), rtol=1e-4)
    out = ops.gemm(xb, wf.contiguous(), K, K, N, bf.to(DEV), gelu=gelu, ln=(mom, c.to(DEV)))
    ref = F.linear(F.layer_norm(x, (K,), gamma, beta, 1e-6), w, b)
    if gelu:
        ref = F.gelu(ref, approximate="tanh")
    assert rel(out, ref) < 8e-3


@pytest.mark.parametrize("M,N,rms,split", [(1280, 2304, False, False), (1280, 1536, True, False),
                                           (96, 64, False, False), (37, 768, True, False), (37, 768, False, True)])
def test_gemm_norm_factors_merged_in_the_epilogue(M, N, rms, split):
    """vt_gemm_fused_lnstats (the folded norm's row factors merged from the chunk statistics in the epilogue)
    against the same GEMM fed by a vt_row_moments / vt_row_rms pass: the factors it stores (ln_mom_out) and its
    outputs match to fp32 rounding (the chunks are summed in another order); CTA-pair tiles (1280 rows) and
    single-CTA tiles (few tiles), LayerNorm and RMSNorm, a partial row block, and K split across CTAs (a
    workspace: every slice merges the factors, the last one runs the epilogue)."""
    K = 768
    g = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(M, K, device=DEV, generator=g) * 2 + 0.3
    w = torch.randn(N, K, device=DEV, generator=g) * 0.02
    b = torch.randn(N, device=DEV, generator=g) * 0.1
    gamma = 1 + 0.1 * torch.randn(K, device=DEV, generator=g)
    beta = torch.zeros(K, device=DEV) if rms else 0.05 * torch.randn(K, device=DEV, generator=g)
    stats = torch.empty(M, K // 32, 2, device=DEV)
    xb = torch.empty(M, K, device=DEV, dtype=BF)
    ops.row_stats(x, stats, xb)
    wf, c, bf = ops.fold_layernorm(w, b, gamma, beta)
    wf, c, bf = wf.contiguous(), c.to(DEV), bf.to(DEV)
    mom_ref = (ops.row_rms if rms else ops.row_moments)(stats, 1e-6, torch.empty(M, 2, device=DEV))
    out_ref = ops.gemm(xb, wf, K, K, N, bf, out_f32=True, ln=(mom_ref, c))
    mom = torch.full((M, 2), float("nan"), device=DEV)
    ws = ops.gemm_workspace(M, N, DEV) if split else None
    out = ops.gemm(xb, wf, K, K, N, bf, out_f32=True, ln_rows=(stats, 1e-6, rms, c, mom), ws=ws)
    torch.cuda.synchronize()
    assert torch.allclose(mom, mom_ref, rtol=1e-5, atol=1e-6)
    assert torch.allclose(out, out_ref, rtol=1e-4, atol=1e-4)
    if not rms:
        ref = F.linear(F.layer_norm(x, (K,), gamma, beta, 1e-6), w, b)
        assert rel(out, ref) < 8e-3


@pytest.mark.parametrize("bn", ["192", "256"])
def test_gemm_both_tile_widths_in_a_subprocess(bn):
    """VT_GEMM_BN forces the 192- or 256-wide N tile: both give correct results on the tower shapes."""
    import subprocess
    import sys
    code = ("import torch, torch.nn.functional as F; from strix_halo_maxx_b200 import ops\n"
            "for M, K, N in [(1000, 1152, 1152), (729, 1152, 3456), (729, 4304, 1152), (300, 1152, 4304)]:\n"
            "    x = torch.randn(M, K, device='cuda').to(torch.bfloat16)\n"
            "    w = (torch.randn(N, K, device='cuda') * 0.02).to(torch.bfloat16)\n"
            "    o = ops.VtLin(w, None)(x); r = F.linear(x.float(), w.float())\n"
            "    e = float((o.float() - r).norm() / r.norm()); assert e < 5e-3, (M, K, N, e)\n")
    env = dict(os.environ, VT_GEMM_BN=bn)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-2000:]


def test_gemm_k588_in_padded_pitch_matches_contiguous():
    M, K, N = 729, 588, 1152
    x, w, b = _operands(M, K, N, 3)
    buf = torch.zeros(M, 592, device=DEV, dtype=BF)
    buf[:, :K] = x
    a = ops.VtLin(w, b)(buf[:, :K])
    c = ops.VtLin(w, b)(x)      # copied into a padded operand by the wrapper
    assert torch.equal(a, c)


def test_gemm_empty_and_errors():
    x, w, b = _operands(8, 64, 16)
    out = torch.empty(0, 16, device=DEV, dtype=BF)
    assert lib().vt_gemm_bf16(0, x.data_ptr(), 64, w.data_ptr(), 64, None, out.data_ptr(), 16, 0, 16, 64, 0) == 0
    with pytest.raises(VtError):
        ops.gemm(x, w, 64, 64, 16, b, gelu=True, out_f32=True)
    bad = torch.empty(8, 70, device=DEV, dtype=BF)
    assert lib().vt_gemm_bf16(0, bad.data_ptr(), 70, w.data_ptr(), 64, None, out.data_ptr(), 16, 8, 16, 64, 0) == -2


SPLITK = [(32, 2048, 2048), (32, 8192, 2048), (32, 2048, 6144), (1, 2048, 4), (5, 4304, 1000), (100, 1152, 264)]


def _counters_zero(ws, M, N):
    """The split-K arrival counters (the first M * ceil(N/32) ints of the workspace) are back at zero."""
    n = M * ((N + 31) // 32) * 4
    return int(ws[:n].count_nonzero()) == 0


@pytest.mark.parametrize("M,K,N", SPLITK)
@pytest.mark.parametrize("epi", ["bf16", "gelu", "res_inplace"])
def test_gemm_split_k_workspace(M, K, N, epi):
    """vt_gemm_fused_ws: the small-tile path splits K across CTAs (fp32 partial sums in the workspace, the
    last slice adds them in slice order and runs the epilogue); same result as the unsplit GEMM up to
    summation order, bit-identical from run to run, and the arrival counters are zero again after a call."""
    x, w, b = _operands(M, K, N, 11)
    ws = ops.gemm_workspace(M, N, DEV)
    if epi == "res_inplace":
        x0 = torch.randn(M, N, device=DEV)
        NP = (N + 7) // 8 * 8  # fp32 output pitches are multiples of 8 elements
        y_ws, y = torch.zeros(M, NP, device=DEV)[:, :N], torch.zeros(M, NP, device=DEV)[:, :N]
        y_ws.copy_(x0)
        y.copy_(x0)
        ops.gemm(x, w, K, K, N, b, res=y_ws, out=y_ws, ws=ws)
        ops.gemm(x, w, K, K, N, b, res=y, out=y)
        ref = F.linear(x.float(), w.float(), b) + x0
        assert rel(y_ws, ref) < 1e-4 and rel(y, ref) < 1e-4
        assert torch.allclose(y_ws, y, rtol=1e-4, atol=1e-4)
    else:
        gelu = epi == "gelu"
        o_ws = ops.gemm(x, w, K, K, N, b, gelu=gelu, ws=ws)
        assert torch.equal(ops.gemm(x, w, K, K, N, b, gelu=gelu, ws=ws), o_ws)
        o = ops.gemm(x, w, K, K, N, b, gelu=gelu)
        ref = F.linear(x.float(), w.float(), b)
        if gelu:
            ref = F.gelu(ref.to(BF).float(), approximate="tanh")
        assert rel(o_ws, ref) < 5e-3
        assert rel(o_ws, o) < 5e-3 and (o_ws.float() - o.float()).abs().max() <= 0.05 * o.float().abs().max()
    torch.cuda.synchronize()
    assert _counters_zero(ws, M, N)


def test_gemm_split_k_workspace_reused_across_shapes_and_too_small():
    """One workspace sized for the widest output serves GEMMs of other shapes back to back (the text
    question's qkv / proj / fc1 / fc2), and a workspace below vt_gemm_ws_bytes is an error, not a fault."""
    ws = ops.gemm_workspace(32, 8192, DEV)
    for M, K, N in [(32, 2048, 6144), (32, 2048, 2048), (1, 2048, 4), (32, 2048, 8192), (32, 8192, 2048),
                    (1, 2048, 4), (32, 2048, 2048)]:
        x, w, b = _operands(M, K, N, K + N)
        out = ops.gemm(x, w, K, K, N, b, ws=ws)
        assert rel(out, F.linear(x.float(), w.float(), b)) < 5e-3, (M, K, N)
    torch.cuda.synchronize()
    assert _counters_zero(ws, 32, 8192)
    x, w, b = _operands(32, 2048, 2048, 3)
    with pytest.raises(VtError):
        ops.gemm(x, w, 2048, 2048, 2048, b, ws=ops.gemm_workspace(8, 2048, DEV))


def test_gemm_graph_replay_bit_exact():
    """test_hgemm.py:51-67: a captured launch replays bit-exactly like eager."""
    M, K, N = 729, 1152, 4304
    x, w, b = _operands(M, K, N, 4)
    lin = ops.VtLin(w, b)
    xin = x.clone()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        lin(xin, gelu=True)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = lin(xin, gelu=True)
    x2 = torch.randn_like(x.float()).to(BF)
    xin.copy_(x2)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, lin(x2, gelu=True))


def test_gemm_rows_are_batch_invariant():
    """A row's result does not depend on which M tile it lands in (fixed K order): crops batched into
    one GEMM give bit-identical features to crops run alone."""
    K, N = 1152, 3456
    x, w, b = _operands(3 * 729, K, N, 5)
    lin = ops.VtLin(w, b)
    full = lin(x)
    one = lin(x[729:1458].contiguous())
    assert torch.equal(full[729:1458], one)


def _attn_ref(q, k, v):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float())


ATTN_CASES = [(1, 16, 729, 72), (3, 16, 729, 72), (1, 12, 1280, 64), (2, 2, 1, 72), (1, 3, 7, 16), (2, 4, 65, 64),
              (1, 1, 200, 80), (1, 2, 129, 72), (1, 1, 256, 64)]


@pytest.mark.parametrize("B,H,T,D", ATTN_CASES)
def test_attention_strided_qkv(B, H, T, D):
    qkv = torch.randn(B, T, 3 * H * D, device=DEV).to(BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = ops.VtAttn(H, T, D)(q, k, v)
    ref = _attn_ref(q, k, v).transpose(1, 2).reshape(B, T, H * D)
    assert rel(out, ref) < 1e-2
    sdpa_bf16 = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, T, H * D)
    assert rel(out, ref) < 3 * max(rel(sdpa_bf16, ref), 2e-3)


@pytest.mark.parametrize("B,H,T,D", [(8, 16, 729, 72), (40, 16, 64, 64), (30, 12, 200, 64)])
def test_attention_many_items_each_within_tolerance(B, H, T, D):
    """More (query tile, head, crop) items than resident CTAs (2 per SM), so CTAs start while others run;
    T = 64 gives one key tile per item.  The error is checked per item, so one wrong item cannot hide in
    the global norm."""
    qkv = torch.randn(B, T, 3 * H * D, device=DEV).to(BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = ops.VtAttn(H, T, D)(q, k, v).float().view(B, T, H, D)
    ref = _attn_ref(q, k, v).transpose(1, 2).float()
    Tt = (T + 127) // 128
    pad = Tt * 128 - T
    e = F.pad((out - ref).transpose(1, 2), (0, 0, 0, pad)).reshape(B, H, Tt, 128 * D).norm(dim=-1)
    r = F.pad(ref.transpose(1, 2), (0, 0, 0, pad)).reshape(B, H, Tt, 128 * D).norm(dim=-1)
    assert B * H * Tt > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    assert float((e / r).max()) < 1e-2


@pytest.mark.parametrize("B,H,T,D,scale", [(1, 12, 1280, 64, 1.0), (1, 4, 1100, 72, 6.0), (2, 2, 1025, 64, 1.0),
                                           (1, 3, 1500, 80, 3.0)])
def test_attention_key_split_each_item_within_tolerance(B, H, T, D, scale):
    """Grids of fewer than two query-tile CTAs per SM with 16 or more key tiles: the keys of each query tile are
    split over a cluster of two CTAs and rank 0 merges the halves (each half's unnormalised O rescaled by
    2^(m_half - m)).  Even and odd key-tile counts, a partial last key tile (T = 1025: one key), head_dim 64 / 72 /
    80, and scaled logits whose row maxima differ between the halves; the error is checked per (crop, head,
    query tile)."""
    qkv = (torch.randn(B, T, 3 * H * D, device=DEV) * scale).to(BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = ops.VtAttn(H, T, D)(q, k, v).float().view(B, T, H, D)
    ref = _attn_ref(q, k, v).transpose(1, 2).float()
    Tt = (T + 127) // 128
    pad = Tt * 128 - T
    e = F.pad((out - ref).transpose(1, 2), (0, 0, 0, pad)).reshape(B, H, Tt, 128 * D).norm(dim=-1)
    r = F.pad(ref.transpose(1, 2), (0, 0, 0, pad)).reshape(B, H, Tt, 128 * D).norm(dim=-1)
    assert B * H * Tt < 2 * torch.cuda.get_device_properties(0).multi_processor_count and (T + 63) // 64 >= 16
    assert torch.isfinite(out).all()
    assert float((e / r).max()) < 1e-2


def test_attention_fused_qkv_tiles_match_pack_path():
    """QKV GEMM writing attention tiles == separate GEMM + pack (bit-exact: same GEMM rows)."""
    B, H, T, D, K = 2, 16, 729, 72, 1152
    x, w, b = _operands(B * T, K, 3 * H * D, 6)
    tiles = ops.attn_tiles(B, T, H, D, DEV)
    ops.gemm_qkv_tiles(x, w, K, K, b, tiles, T, H, D)
    out = torch.empty(B * T, H * D, device=DEV, dtype=BF)
    ops.attention_tiles(tiles, B, T, H, D, out)
    qkv = ops.VtLin(w, b)(x).view(B, T, -1)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    att = ops.VtAttn(H, T, D)
    ref = att(q, k, v)
    assert torch.equal(att._tiles[B], tiles)
    assert torch.equal(out.view(B, T, -1), ref)


def test_attention_large_logits_stay_finite():
    B, H, T, D = 1, 2, 300, 72
    qkv = (torch.randn(B, T, 3 * H * D, device=DEV) * 8).to(BF)
    q, k, v = [t.view(B, T, H, D).transpose(1, 2) for t in qkv.chunk(3, dim=-1)]
    out = ops.VtAttn(H, T, D)(q, k, v)
    assert torch.isfinite(out.float()).all()
    assert rel(out, _attn_ref(q, k, v).transpose(1, 2).reshape(B, T, -1)) < 1e-2


@pytest.mark.parametrize("M,N,in_bf16,out_f32", [(729, 1152, False, False), (1280, 768, False, True),
                                                 (5, 1152, True, False), (33, 2048, False, False), (3, 4096, True, True)])
def test_layernorm(M, N, in_bf16, out_f32):
    x = (torch.randn(M, N, device=DEV) * 3 + 0.5)
    if in_bf16:
        x = x.to(BF)
    w = torch.randn(N, device=DEV)
    b = torch.randn(N, device=DEV)
    out = ops.layer_norm(x, w, b, 1e-6, out_f32=out_f32)
    ref = F.layer_norm(x.float(), (N,), w, b, 1e-6)
    assert rel(out, ref) < (1e-5 if out_f32 else 4e-3)


@pytest.mark.parametrize("N,in_bf16", [(1152, False), (2048, True), (768, False), (4096, False)])
def test_layernorm_rows_do_not_depend_on_the_row_count(N, in_bf16):
    """Few rows run one CTA per row, many rows one warp per row: the same row gives the same bits either way
    (LayerNorm, RMSNorm and the fused int8 quantisation)."""
    gen = torch.Generator().manual_seed(N)
    big = (torch.randn(3000, N, generator=gen) * 2 + 0.3).to(DEV)
    if in_bf16:
        big = big.to(BF)
    w = (torch.randn(N, generator=gen) + 1).to(DEV)
    b = torch.randn(N, generator=gen).to(DEV)
    few = big[:17].clone()
    assert torch.equal(ops.layer_norm(few, w, b, 1e-5), ops.layer_norm(big, w, b, 1e-5)[:17])
    assert torch.equal(ops.rms_norm(few, w, 1e-6, out_f32=True), ops.rms_norm(big, w, 1e-6, out_f32=True)[:17])
    qf, sf = torch.empty(17, N, dtype=torch.int8, device=DEV), torch.empty(17, device=DEV)
    qb, sb = torch.empty(3000, N, dtype=torch.int8, device=DEV), torch.empty(3000, device=DEV)
    ops.layer_norm_quant(few, w, b, 1e-5, qf, sf)
    ops.layer_norm_quant(big, w, b, 1e-5, qb, sb)
    assert torch.equal(qf, qb[:17]) and torch.equal(sf, sb[:17])


@pytest.mark.parametrize("kind", [torch.float32, BF, torch.uint8])
def test_im2col(kind):
    from oracle.tower_ref import im2col, normalize_u8
    B = 2
    if kind == torch.uint8:
        pix = torch.randint(0, 256, (B, 378, 378, 3), dtype=torch.uint8, device=DEV)
        ref = im2col(normalize_u8(pix.cpu()))
    else:
        pix = (torch.rand(B, 3, 378, 378, device=DEV) * 2 - 1).to(kind)
        ref = im2col(pix.float().cpu())
    out = torch.zeros(B * 729, 592, device=DEV, dtype=BF)
    ops.im2col(pix, 14, out)
    assert torch.equal(out[:, :588].cpu(), ref.reshape(-1, 588).to(BF))
    assert not out[:, 588:].any()


@pytest.mark.parametrize("M,N", [(1280, 768), (7, 1152)])
def test_rmsnorm(M, N):
    from oracle.tapnext_ref import rms_norm
    x = torch.randn(M, N, device=DEV) * 4
    w = torch.randn(N, device=DEV)
    out = ops.rms_norm(x, w, 1e-6, out_f32=True)
    assert rel(out, rms_norm(x.cpu(), w.cpu(), 1e-6)) < 1e-5


def test_crop_combine():
    f = torch.randn(13, 729, 1152, device=DEV).to(BF)
    out = torch.empty(729, 2304, device=DEV, dtype=BF)
    ops.crop_combine(f, out)
    assert torch.equal(out[:, :1152], f[0])
    assert rel(out[:, 1152:], f[1:].float().mean(0)) < 4e-3


@pytest.mark.parametrize("first", [True, False])
def test_rglru(first):
    from oracle.tapnext_ref import rglru as rglru_ref
    M, W = 1280, 768
    x = torch.randn(M, W, device=DEV)
    u = torch.randn(M, W, device=DEV).to(BF)
    h0 = torch.randn(M, W, device=DEV)
    Wd = {"blocks.0.gx_w": torch.randn(W, W) * 0.02, "blocks.0.gx_b": torch.randn(W) * 0.1,
          "blocks.0.ga_w": torch.randn(W, W) * 0.02, "blocks.0.ga_b": torch.randn(W) * 0.1,
          "blocks.0.a_param": torch.randn(W)}
    uf = u.float().cpu()
    G = torch.cat([F.linear(uf, Wd["blocks.0.gx_w"], Wd["blocks.0.gx_b"]),
                   F.linear(uf, Wd["blocks.0.ga_w"], Wd["blocks.0.ga_b"])], 1).to(DEV)
    ref = rglru_ref(uf, Wd, "blocks.0.", None if first else h0.cpu(), 8.0)
    state, xx = h0.clone(), x.clone()
    sp = F.softplus(Wd["blocks.0.a_param"].double()).float().to(DEV)
    ops.rglru(G, sp, u, state, xx, 8.0, first)
    assert rel(state, ref) < 1e-5
    assert rel(xx, x + ref.to(DEV)) < 1e-5
