"""Full TAPNext++ block step on the GPU: its new kernels against the oracle's restatements, and the whole
step against the CPU fp32 oracle over several frames (recurrent state and conv history carried)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200.config import TapNextConfig
from strix_halo_maxx_b200 import ops, weights as wg
from strix_halo_maxx_b200.tapnextpp import TapNextPPStep
from strix_halo_maxx_b200._lib import device_status
from oracle import tapnextpp_ref as R
from helpers import assert_tokens_close

CFG = TapNextConfig()
BF = torch.bfloat16
DEV = "cuda"


def _bf(a):
    return torch.as_tensor(a, dtype=torch.float32).to(BF)


@pytest.mark.parametrize("first", [True, False])
def test_ssm_step_matches_bf16_restatement(first):
    """vt_ssm_step against ssm_bf16 (the reference's ssm_ref rounding points) on every head, with a
    partial row block (R = 100): equal to the last bf16 bit except where an fp32 sum falls within a few ulps
    of a bf16 rounding boundary (the reference sums in float64), and then by one bf16 step."""
    g = torch.Generator().manual_seed(5)
    Rn, W, H = 100, 768, 12
    rnd = lambda *s, sc=1.0: torch.randn(*s, generator=g) * sc
    y, xx, xm1, xm2, xm3 = [_bf(rnd(Rn, W)) for _ in range(5)]
    h0 = rnd(Rn, W)
    conv_w, conv_b = rnd(4, W, sc=0.5), rnd(W, sc=0.1)
    a_param = rnd(W)
    wx, wa = _bf(rnd(H, 64, 64, sc=0.15)).float(), _bf(rnd(H, 64, 64, sc=0.15)).float()  # bf16 weights
    bx, ba = rnd(W, sc=0.1), rnd(W, sc=0.1)
    hist = [t.to(DEV).contiguous() for t in (xm3, xm2, xm1)]
    h = h0.clone().to(DEV)
    z = torch.empty(Rn, W, dtype=BF, device=DEV)
    sp = torch.nn.functional.softplus(a_param.double()).float()
    dv = lambda t: t.to(DEV).contiguous()
    ops.ssm_step(dv(y), dv(xx), hist, h, dv(conv_w), dv(conv_b), dv(sp), dv(wx), dv(bx), dv(wa), dv(ba), z, first)
    zr, hr = [], []
    for q in range(H):
        s = slice(64 * q, 64 * q + 64)
        zq, hq = R.ssm_bf16(y[:, s].float(), xx[:, s].float(), xm1[:, s].float(), xm2[:, s].float(), xm3[:, s].float(),
                            h0[:, s], conv_w[:, s], conv_b[s], a_param[s], wx[q], bx[s], wa[q], ba[s], first)
        zr.append(zq)
        hr.append(hq)
    zr, hr = torch.cat(zr, 1), torch.cat(hr, 1)
    zg = z.float().cpu()
    mism = (zg != zr)
    assert mism.float().mean() < 1e-3, float(mism.float().mean())
    # any mismatch is one bf16 step at most
    assert torch.all((zg - zr).abs() <= zr.abs() * 2 ** -7 + 1e-30)
    assert torch.allclose(h.cpu(), hr, rtol=2e-6, atol=1e-6)
    assert torch.equal(hist[0].cpu(), xx)  # x_t replaced the oldest tap


def test_gated_gelu_mul_and_gelu_erf():
    g = torch.Generator().manual_seed(6)
    G = _bf(torch.randn(77, 2 * 3072, generator=g) * 2).to(DEV)
    out = torch.empty(77, 3072, dtype=BF, device=DEV)
    ops.gated_gelu_mul(G, out)
    gf = G.float()
    ref = (R.gelu_tanh(gf[:, :3072]).to(BF).float() * gf[:, 3072:]).to(BF).float()
    assert torch.allclose(out.float(), ref, rtol=2e-2, atol=1e-3)
    x = _bf(torch.randn(50, 3072, generator=g) * 3).to(DEV)
    ref2 = R.gelu_erf(x.float()).to(BF).float()
    ops.gelu_erf(x)
    assert torch.allclose(x.float(), ref2, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("M", [1280, 77])
def test_gemm_gated_gelu_epilogue_against_gemm_then_gated_gelu_mul(M):
    """gemm(gelu="gated") over gate / up weight rows interleaved by 16 against the same GEMM with a bf16 output
    followed by vt_gated_gelu_mul: the linear outputs are the same, so the results differ only where the two
    GELU-tanh formulas round to neighbouring bf16 values (a bf16 step or two of the product).  CTA-pair tiles
    (1280 rows) and single-CTA tiles (77 rows)."""
    K, Fh = 768, 3072
    g = torch.Generator(device=DEV).manual_seed(12)
    x = torch.randn(M, K, device=DEV, generator=g).to(BF)
    w = (torch.randn(2 * Fh, K, device=DEV, generator=g) * 0.05).to(BF)
    b = torch.randn(2 * Fh, device=DEV, generator=g) * 0.1
    G = ops.gemm(x, w, K, K, 2 * Fh, b)
    ref = torch.empty(M, Fh, dtype=BF, device=DEV)
    ops.gated_gelu_mul(G, ref)
    wi, bi = ops.gate_up_interleave(w, Fh).contiguous(), ops.gate_up_interleave(b, Fh).contiguous()
    out = ops.gemm(x, wi, K, K, 2 * Fh, bi, gelu="gated")
    torch.cuda.synchronize()
    assert out.shape == (M, Fh)
    d = (out.float() - ref.float()).abs()
    assert float((d > 0).float().mean()) < 5e-2
    assert torch.all(d <= ref.float().abs() * 2 ** -6 + 1e-6)


NORMS = {"in_gemm": dict(), "row_pass": dict(rows_in_gemm=False), "unfolded": dict(fold_ln=False)}


@pytest.mark.parametrize("n_blocks,n_frames,affine,norms", [(12, 2, "zero", "in_gemm"), (2, 6, "random", "in_gemm"),
                                                           (2, 6, "random", "row_pass"), (2, 6, "random", "unfolded")])
def test_tapnextpp_stream(n_blocks, n_frames, affine, norms):
    """The full TAPNext++ step against the fp32 restatement, state and conv history carried, with the four norms
    of a block folded into the GEMMs after them and their row factors merged in those GEMMs' epilogues
    (default), folded with a row-moment pass before each, and as separate passes."""
    device_status(clear=True)
    W = wg.tapnextpp_weights(CFG, seed=9, n_blocks=n_blocks, affine=affine)
    frames, queries = wg.tapnext_inputs(CFG, n_frames, seed=2)
    eng = TapNextPPStep(W, CFG, device=DEV, **NORMS[norms])
    state = None
    for f in range(n_frames):
        ref, state = R.step(frames[f], queries[f], W, CFG, state, n_blocks)
        out = eng.step(torch.from_numpy(frames[f]).to(DEV), torch.from_numpy(queries[f]).to(DEV))
        assert_tokens_close(out.float().cpu(), ref, what=f"frame {f}")
    assert device_status(clear=True) == 0


def test_tapnextpp_graph_replay_matches_eager():
    """Frames after the first replay the graph of their history-ring position (three graphs): bit-identical
    to launching eagerly, across a reset to a new video."""
    W = wg.tapnextpp_weights(CFG, seed=9, n_blocks=2, affine="random")
    frames, queries = wg.tapnext_inputs(CFG, 6, seed=4)
    eg, ee = TapNextPPStep(W, CFG, device=DEV), TapNextPPStep(W, CFG, device=DEV, graphs=False)
    for f in list(range(5)) + ["reset"] + list(range(3)):
        if f == "reset":
            eg.reset()
            ee.reset()
            continue
        fr, q = torch.from_numpy(frames[f]).to(DEV), torch.from_numpy(queries[f]).to(DEV)
        assert torch.equal(eg.step(fr, q), ee.step(fr, q)), f"frame {f}"
    assert sorted(eg._graphs) == [0, 1, 2]


def _heads_fixture():
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "heads_ref_cases.npz"))
    HW = wg.heads_weights(CFG, seed=int(g["wseed"]))
    x = torch.from_numpy(wg.heads_input(CFG, seed=int(g["xseed"]))).to(BF)
    return HW, x, g


def test_track_heads_against_reference_heads_np():
    """TrackHeads (fp32 kernels) on the fixture's query tokens against the reference's own Step8.heads_np
    outputs (tests/golden/heads_ref_cases.npz): tracks within 1e-3 px, logits and visibility within 1e-4."""
    from strix_halo_maxx_b200.tapnextpp import TrackHeads
    device_status(clear=True)
    HW, x, g = _heads_fixture()
    heads = TrackHeads(HW, CFG, DEV)
    tracks, logits, vis = heads(x.to(DEV))
    torch.cuda.synchronize()
    assert np.abs(tracks.cpu().numpy() - g["tracks"]).max() < 1e-3
    assert np.allclose(logits.cpu().numpy(), g["logits"], rtol=1e-4, atol=1e-4)
    assert np.allclose(vis.cpu().numpy(), g["vis"], rtol=1e-4, atol=1e-4)
    # a partial query block (37 rows) takes the same per-row path
    t37, _, v37 = heads(x[:37].to(DEV))
    assert np.abs(t37.cpu().numpy() - g["tracks"][:37]).max() < 1e-3
    assert np.allclose(v37.cpu().numpy(), g["vis"][:37], rtol=1e-4, atol=1e-4)
    assert device_status(clear=True) == 0


@pytest.mark.parametrize("x_bf16", [True, False])
def test_head_linear_ring_kernel_equals_plain_kernel(x_bf16):
    """vt_head_linear's two kernels give the same fp32 results bit for bit: the cp.async-ring kernel (16-byte
    aligned rows, N % 4 == 0) and the plain one (taken here by N = 515 on the same rows and pitches) both sum
    every output over k in order with fp32 FMAs.  A partial row block (M = 77) and a float64 check."""
    g = torch.Generator(device=DEV).manual_seed(5)
    M, K, N = 77, 768, 516
    x = torch.randn(M, K, device=DEV, generator=g)
    x = x.to(BF) if x_bf16 else x
    w = torch.randn(K, N, device=DEV, generator=g)
    b = torch.randn(N, device=DEV, generator=g)
    y_ring = torch.full((M, N), float("nan"), device=DEV)
    ops.head_linear(x, w, b, y_ring)
    y_plain = torch.full((M, N), float("nan"), device=DEV)
    ops.head_linear(x, w[:, :515], b, y_plain[:, :515])
    torch.cuda.synchronize()
    assert torch.equal(y_ring[:, :515], y_plain[:, :515])
    ref = x.double() @ w.double() + b.double()
    assert torch.allclose(y_ring.double(), ref, rtol=1e-4, atol=1e-3)


def test_tapnextpp_track_runs_the_heads_inside_the_step():
    """TapNextPPStep(heads=...).track: the tracks of frames replayed from the CUDA graph equal TrackHeads run on
    the step's own query tokens, and the oracle heads of those tokens (CPU fp32) within 1e-3 px."""
    from strix_halo_maxx_b200.tapnextpp import TrackHeads
    W = wg.tapnextpp_weights(CFG, seed=8, n_blocks=2, affine="random")
    HW = wg.heads_weights(CFG, seed=21)
    frames, queries = wg.tapnext_inputs(CFG, 3, seed=4)
    eng = TapNextPPStep(W, CFG, device=DEV, heads=HW)
    ref_heads = TrackHeads(HW, CFG, DEV)
    for f in range(3):
        tracks, logits, vis, xq = eng.track(torch.from_numpy(frames[f]).cuda(), torch.from_numpy(queries[f]).cuda())
        t2, l2, v2 = ref_heads(xq)
        assert torch.equal(tracks, t2) and torch.equal(logits, l2) and torch.equal(vis, v2), f"frame {f}"
        rt, rl, rv = R.heads(xq.float().cpu(), HW, CFG)
        assert float((tracks.cpu() - rt).abs().max()) < 1e-3, f"frame {f}"
        assert torch.allclose(vis.cpu(), rv, rtol=1e-4, atol=1e-4)
    assert len(eng._graphs) == 2


@pytest.mark.parametrize("first", [True, False])
def test_ssm_step_gelu_y_equals_gelu_in_the_gemm(first):
    """linear_yx as one GEMM with the GELU of y taken in vt_ssm_step (gelu_y) gives the same z, h and history
    bit for bit as the GELU-tanh GEMM epilogue on the y half."""
    g = torch.Generator(device=DEV).manual_seed(9)
    Rn, W = 1280, 768
    t = torch.randn(Rn, W, device=DEV, generator=g).to(BF)
    wyx = (torch.randn(2 * W, W, device=DEV, generator=g) * 0.04).to(BF)
    byx = torch.randn(2 * W, device=DEV, generator=g) * 0.1
    H = W // 64
    conv_w, conv_b = torch.randn(4, W, device=DEV, generator=g) * 0.5, torch.randn(W, device=DEV, generator=g) * 0.1
    sp = torch.nn.functional.softplus(torch.randn(W, device=DEV, generator=g))
    wx = (torch.randn(H, 64, 64, device=DEV, generator=g) * 0.15).to(BF).float()
    wa = (torch.randn(H, 64, 64, device=DEV, generator=g) * 0.15).to(BF).float()
    bx, ba = torch.randn(W, device=DEV, generator=g) * 0.1, torch.randn(W, device=DEV, generator=g) * 0.1
    hist0 = [torch.randn(Rn, W, device=DEV, generator=g).to(BF) for _ in range(3)]
    h0 = torch.randn(Rn, W, device=DEV, generator=g)
    yx_raw = ops.gemm(t, wyx, W, W, 2 * W, byx)
    yx_gelu = yx_raw.clone()       # y and x share one row pitch in vt_ssm_step: [gelu(y) | x]
    yx_gelu[:, :W] = ops.gemm(t, wyx[:W], W, W, W, byx[:W], gelu=True)
    outs = []
    for gelu_y, yx in ((True, yx_raw), (False, yx_gelu)):
        hist = [x.clone() for x in hist0]
        h, z = h0.clone(), torch.empty(Rn, W, dtype=BF, device=DEV)
        ops.ssm_step(yx[:, :W], yx[:, W:], hist, h, conv_w, conv_b, sp, wx, bx, wa, ba, z, first, gelu_y=gelu_y)
        outs.append((z, h, hist[0]))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
