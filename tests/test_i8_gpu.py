"""The W8A8 int8 path on the GPU -- vt_quant_rows, vt_gemm_i8 (tcgen05 kind::i8) and the int8 text decoder --
against the CPU oracle oracle/i8_ref.py, which tests/test_oracle_golden.py pins to the reference's own HI8Lin
numerics (tests/golden/i8_quant_gemm.npz).  Integer work (quantisation, the int32 products, split-K sums)
and the fp32 epilogue without GELU are compared bit for bit; GELU outputs within one bf16 step."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import ops, weights as wg
from strix_halo_maxx_b200.config import TEXT
from strix_halo_maxx_b200.text import TextDecoder
from strix_halo_maxx_b200._lib import device_status
from oracle import i8_ref, text_ref as R
from helpers import assert_tokens_close, rel

DEV = "cuda"
BF = torch.bfloat16


def _golden():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "i8_quant_gemm.npz"))


def _bf16_close(out, ref):
    """GELU outputs: within one bf16 step of the reference, or 4e-6 absolute.  The GPU evaluates GELU-tanh as
    x * sigmoid(2u) (relative error ~1e-6 everywhere); the reference's 0.5 x (1 + (1 - 2 / (1 + e^(2u)))) loses
    its relative accuracy in the negative tail, where 1 + tanh u cancels (absolute error up to ~1.2e-7 |x|)."""
    out, ref = np.asarray(out, np.float32), np.asarray(ref, np.float32)
    tol = np.maximum(np.abs(out), np.abs(ref)) * 2.0 ** -7 + 4e-6
    bad = np.abs(out - ref) > tol
    assert not bad.any(), f"{bad.sum()} elements off, worst {np.abs(out - ref).max()}"


def test_quant_rows_matches_reference_golden():
    """The fixture's bf16-representable activations (zero row, sub-floor row, exact half-way points)."""
    device_status(clear=True)
    g = _golden()
    q, s = ops.quant_rows(torch.from_numpy(g["x"]).to(DEV, BF))
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(s.cpu().numpy(), g["sx"])
    assert device_status(clear=True) == 0


@pytest.mark.parametrize("M,K,scale", [(730, 2048, 1.0), (32, 8192, 30.0), (5, 136, 1e-3), (3, 16384, 1.0),
                                       (1, 8, 1e-7)])
def test_quant_rows_bit_exact(M, K, scale):
    gen = torch.Generator().manual_seed(M * 7 + K)
    x = torch.randn(M, K, generator=gen) * scale * torch.exp(torch.rand(M, 1, generator=gen) * 4 - 2)
    if M > 2:
        x[1] = 0.0
    x = x.to(BF)
    q, s = ops.quant_rows(x.to(DEV))
    qr, sr = i8_ref.quant_rows(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), sr)
    assert np.array_equal(q.cpu().numpy(), qr)


@pytest.mark.parametrize("M,N,in_bf16", [(730, 2048, False), (32, 2048, True), (9, 1152, False)])
def test_layernorm_quant_equals_layernorm_then_quant_rows(M, N, in_bf16):
    """The fused LayerNorm + quantisation gives the bits of vt_layernorm (bf16 out) followed by vt_quant_rows."""
    gen = torch.Generator().manual_seed(M + N)
    x = (torch.randn(M, N, generator=gen) * 3 + 1).to(DEV)
    if in_bf16:
        x = x.to(BF)
    w = (torch.randn(N, generator=gen) * 0.5 + 1).to(DEV)
    b = (torch.randn(N, generator=gen) * 0.1).to(DEV)
    h = ops.layer_norm(x, w, b, 1e-5)
    q0, s0 = ops.quant_rows(h)
    q1 = torch.empty(M, N, dtype=torch.int8, device=DEV)
    s1 = torch.empty(M, dtype=torch.float32, device=DEV)
    y = torch.empty(M, N, dtype=BF, device=DEV)
    ops.layer_norm_quant(x, w, b, 1e-5, q1, s1, out=y)
    assert torch.equal(q0, q1) and torch.equal(s0, s1) and torch.equal(h, y)


def test_weight_quantisation_matches_reference_golden():
    """I8Lin's on-device weight quantisation (hgemm.py:100-103) reproduces the fixture's weights and scales."""
    g = _golden()
    lin = ops.I8Lin(g["w"], g["bias"], DEV)
    assert np.array_equal(lin.wq[:, :lin.K].cpu().numpy(), g["wq"])
    assert np.array_equal(lin.sw.cpu().numpy(), g["sw"])


def test_gemm_i8_matches_reference_golden():
    """The fixture's quantised operands through vt_gemm_i8: fp32 output bit for bit, GELU within a bf16 step."""
    g = _golden()
    q, wq = torch.from_numpy(g["q"]).to(DEV), torch.from_numpy(g["wq"]).to(DEV)
    sx, sw, b = (torch.from_numpy(g[k]).to(DEV) for k in ("sx", "sw", "bias"))
    M, K = q.shape
    N = wq.shape[0]
    y0 = ops.gemm_i8(q, sx, wq, K, K, N, sw, b, out_f32=True)
    assert np.array_equal(y0.cpu().numpy(), g["y0"])
    y1 = ops.gemm_i8(q, sx, wq, K, K, N, sw, b, gelu=True)
    _bf16_close(y1.float().cpu().numpy(), i8_ref.bf16_round(g["y1"]))


def _operands(M, N, K, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (M, K), generator=gen, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=gen, dtype=torch.int8)
    sx = torch.rand(M, generator=gen) * 1e-2 + 1e-4
    sw = torch.rand(N, generator=gen) * 1e-3 + 1e-5
    b = torch.randn(N, generator=gen)
    return q, w, sx, sw, b


def _dev_i8(t):
    """int8 [R, K] on the device with a 16-byte row pitch (the GEMM's operand rule)."""
    R_, K = t.shape
    buf = torch.zeros(R_, (K + 15) // 16 * 16, dtype=torch.int8, device=DEV)
    buf[:, :K] = t.to(DEV)
    return buf[:, :K]


# (M, N, K, ws): the CTA-pair kernel (full and half-width last column tile, N and K tails; 256 x 128 tiles for
# the 24-tile 730 x 2048 shapes, with the staged and the register residual epilogue), the 128 x 256
# tile (M <= 128, many columns), the 128 x 64 tile with and without split-K (the text question's shapes)
SHAPES = [(730, 6144, 2048, False), (730, 5960, 2048, False), (730, 2048, 8192, False), (730, 2048, 2048, False),
          (730, 2040, 1024, False), (100, 19000, 200, False),
          (32, 2048, 8192, True), (32, 6144, 2048, True), (32, 2048, 2048, False), (7, 40, 72, True)]


@pytest.mark.parametrize("M,N,K,ws", SHAPES)
def test_gemm_i8_bit_exact(M, N, K, ws):
    device_status(clear=True)
    q, w, sx, sw, b = _operands(M, N, K, seed=M + N + K)
    acc = i8_ref.i8_matmul(q.numpy(), w.numpy())
    ref = i8_ref.epilogue(acc, sx.numpy(), sw.numpy(), b.numpy())
    wsb = ops.gemm_workspace(M, N, DEV) if ws else None
    qd, wd = _dev_i8(q), _dev_i8(w)
    out = ops.gemm_i8(qd, sx.to(DEV), wd, wd.stride(0), K, N, sw.to(DEV), b.to(DEV), ws=wsb)
    assert np.array_equal(out.float().cpu().numpy(), i8_ref.bf16_round(ref))
    # fp32 output with an fp32 residual updated in place (the text decoder's proj / fc2)
    res = torch.randn(M, N, generator=torch.Generator().manual_seed(9))
    x = torch.zeros(M, (N + 7) // 8 * 8, dtype=torch.float32, device=DEV)[:, :N]
    x.copy_(res)
    ops.gemm_i8(qd, sx.to(DEV), wd, wd.stride(0), K, N, sw.to(DEV), b.to(DEV), res=x, out=x, ws=wsb)
    assert np.array_equal(x.cpu().numpy(), (ref + res.numpy()).astype(np.float32))
    # GELU on the fp32 value, bf16 output
    out = ops.gemm_i8(qd, sx.to(DEV), wd, wd.stride(0), K, N, sw.to(DEV), b.to(DEV), gelu=True, ws=wsb)
    _bf16_close(out.float().cpu().numpy(), i8_ref.bf16_round(i8_ref.gelu_tanh(ref)))
    assert device_status(clear=True) == 0


def test_gemm_i8_rejects_bad_operands():
    q = _dev_i8(torch.zeros(4, 64, dtype=torch.int8))
    s = torch.ones(4, device=DEV)
    with pytest.raises(Exception):
        ops.gemm_i8(q, s, q, 24, 64, 4, s, None)  # weight pitch not a multiple of 16
    with pytest.raises(Exception):
        ops.quant_rows(torch.zeros(4, 12, dtype=BF, device=DEV))  # K % 8 != 0


def test_text_decoder_int8_prefill_and_question():
    """The int8 text decoder (FastMD2 with tlin_cls=HI8Lin) against the oracle's int8 layers, 2 layers."""
    device_status(clear=True)
    nl = 2
    W = wg.text_weights(TEXT, seed=3, n_layers=nl, affine="random")
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    i8 = R.quantize_weights(W, nl)
    x_ref, cache = R.encode(emb, bos, W, TEXT, n_layers=nl, i8=i8)
    logits_ref = R.query(ids, last, W, TEXT, cache, n_layers=nl, i8=i8)
    dec = TextDecoder(W, TEXT, device=DEV, int8=True)
    x = dec.encode(torch.from_numpy(emb).to(DEV), bos).float().cpu()  # a copy: query() reuses the buffer
    assert_tokens_close(x, x_ref, what="int8 prefix hidden states")
    logits = dec.query(torch.from_numpy(ids).to(DEV), last).float().cpu()
    assert rel(logits, logits_ref) < 3e-2, (logits, logits_ref)
    # the int8 model stays close to the fp32 one (the reference's accepted quantisation error)
    x32, _ = R.encode(emb, bos, W, TEXT, n_layers=nl)
    assert rel(x, x32) < 0.05
    assert device_status(clear=True) == 0


def test_text_decoder_int8_graph_replay_matches_eager():
    W = wg.text_weights(TEXT, seed=3, n_layers=2, affine="random")
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    dg, de = TextDecoder(W, TEXT, device=DEV, int8=True), TextDecoder(W, TEXT, device=DEV, graphs=False, int8=True)
    g = torch.Generator().manual_seed(2)
    for r in range(3):
        e = torch.from_numpy(emb).to(DEV) if r == 0 else torch.randn(TEXT.prefix - 1, TEXT.dim, generator=g).to(DEV)
        assert torch.equal(dg.encode(e, bos), de.encode(e, bos)), f"prefill {r}"
        q = torch.from_numpy(ids).to(DEV)
        assert torch.equal(dg.query(q, last), de.query(q, last)), f"question {r}"
