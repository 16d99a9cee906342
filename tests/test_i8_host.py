"""Host side of the W8A8 int8 path, without a GPU: I8Lin's weight quantisation (a torch mirror of
hgemm.HI8Lin.__init__, moondream/gpu/hgemm.py:100-103) against the reference's numerics fixture, and the
oracle's int8 text layers against its fp32 ones."""
import os

import numpy as np
import torch

from strix_halo_maxx_b200 import ops, weights as wg
from strix_halo_maxx_b200.config import TEXT
from oracle import i8_ref, text_ref as R
from helpers import rel


def _golden():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "i8_quant_gemm.npz"))


def test_i8lin_weight_quantisation_matches_reference_numerics():
    g = _golden()
    lin = ops.I8Lin(g["w"], g["bias"], "cpu")
    assert lin.ldw % 16 == 0 and lin.ldw >= lin.K
    assert np.array_equal(lin.wq[:, :lin.K].numpy(), g["wq"])
    assert not lin.wq[:, lin.K:].any()
    assert np.array_equal(lin.sw.numpy(), g["sw"])
    assert np.array_equal(lin.b.numpy(), g["bias"])


def test_i8_linear_is_close_to_fp32_linear():
    """Per-token / per-channel int8 keeps a Gaussian layer within ~1 % of its fp32 result."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 512)).astype(np.float32)
    w = (rng.standard_normal((256, 512)) * 0.05).astype(np.float32)
    b = rng.standard_normal(256).astype(np.float32)
    wq, sw = i8_ref.quant_w(w)
    y8 = i8_ref.i8_linear(x, wq, sw, b)
    y32 = x @ w.T + b
    assert rel(torch.from_numpy(y8), torch.from_numpy(y32)) < 2e-2


def test_oracle_int8_text_layer_tracks_fp32():
    """One text layer with the HI8Lin linears stays within a few per cent of the fp32 layer (the parity of the
    GPU int8 decoder is checked against the int8 oracle itself)."""
    W = wg.text_weights(TEXT, seed=3, n_layers=1, affine="random")
    emb, bos, _, _ = wg.text_inputs(TEXT, seed=5)
    i8 = R.quantize_weights(W, 1)
    x8, _ = R.encode(emb, bos, W, TEXT, n_layers=1, i8=i8)
    x32, _ = R.encode(emb, bos, W, TEXT, n_layers=1)
    assert rel(x8, x32) < 3e-2


def _rn32(v):
    """Exact rational v -> nearest float32 (ties to even)."""
    from fractions import Fraction
    c = np.float32(float(v))
    best = None
    for k in (c, np.nextafter(c, np.float32(np.inf)), np.nextafter(c, np.float32(-np.inf))):
        if not np.isfinite(k):
            continue
        dist = abs(Fraction(float(k)) - v)
        even = (int(np.array(k, np.float32).view(np.uint32)) & 1) == 0
        if best is None or dist < best[0] or (dist == best[0] and even):
            best = (dist, k)
    return best[1]


def test_reciprocal_division_equals_ieee_division():
    """The quantisation kernels form x / s as q = x * RN(1/s) followed by two FMA corrections q + (x - q s) RN(1/s)
    (div_rn_by in csrc/vt_common.cuh, Markstein's theorem).  Emulated here in exact arithmetic (each FMA and
    product rounded once) it equals the IEEE quotient on random activations and on the half-way points of the
    int8 grid, for scales over 24 binades."""
    from fractions import Fraction as Fr
    f32 = np.float32

    def fma(a, b, c):
        return _rn32(Fr(float(a)) * Fr(float(b)) + Fr(float(c)))

    rng = np.random.default_rng(3)
    n = 0
    for _ in range(60):
        amax = f32(np.exp(rng.uniform(-12, 12)))
        s = f32(max(amax, f32(1e-5)) / f32(127))
        rs = _rn32(1 / Fr(float(s)))
        xs = i8_ref.bf16_round(np.concatenate([rng.uniform(-1, 1, 40).astype(f32) * amax,
                                                ((rng.integers(-127, 127, 10) + 0.5) * s).astype(f32), [amax, -amax]]))
        for x in xs:
            q = _rn32(Fr(float(x)) * Fr(float(rs)))
            q = fma(fma(-q, s, x), rs, q)
            q = fma(fma(-q, s, x), rs, q)
            assert q == f32(x) / s, (x, s)
            n += 1
    assert n == 60 * 52
