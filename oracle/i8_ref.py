"""CPU restatement of the reference's W8A8 int8 linear layer (HI8Lin) -- TEST INFRASTRUCTURE (only tests/ and
bench.py import it).

numpy, fp32 element-wise arithmetic in the reference's order:
  * quant_w(), moondream/gpu/hgemm.py:100-103: per-output-channel scale s = max(max_k |w|, 1e-8) / 127,
    wq = round-half-to-even(w / s) clamped to [-127, 127];
  * quant_rows(), moondream/gpu/tgemm.py:81-91 (`_quant_rows`, reached through hgemm.py:10-16): per-row scale
    s = max(max_k |x|, 1e-5) / 127, q = trunc(x / s + (x / s >= 0 ? 0.5 : -0.5));
  * i8_matmul(): the exact int32 dot products of the int8 rows (the WMMA int32 accumulation of
    moondream/gpu/hip/i8gemm.hip:91-180), computed as a float64 matrix product, exact while
    K * 127^2 < 2^53;
  * epilogue(), i8gemm.hip:183-197: v = ((float)acc * sa[m]) * sw[n] + bias[n], GELU-tanh on that fp32 value
    (i8gemm.hip:11, tanh(u) written as 1 - 2 / (1 + e^(2u))), then bf16 for the layer output.
Pinned by tests/golden/make_golden_i8.py, which runs the reference's own numpy restatement of the same numerics
(moondream/npu/p4/pack_i8.py: quant_rows, quant_w, epilogue) on the fixture's inputs.
"""
import numpy as np

F32 = np.float32


def quant_w(w):
    """hgemm.py:100-103 -> (wq int8 [N, K], s fp32 [N])."""
    w = np.asarray(w, F32)
    s = (np.maximum(np.abs(w).max(axis=1), F32(1e-8)) / F32(127.0)).astype(F32)
    wq = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return wq, s


def quant_rows(x):
    """tgemm.py:81-91 -> (q int8 [M, K], s fp32 [M]); x fp32 (the bf16 activations widened)."""
    x = np.asarray(x, F32)
    s = (np.maximum(np.abs(x).max(axis=1), F32(1e-5)) / F32(127.0)).astype(F32)
    v = (x / s[:, None]).astype(F32)
    t = (v + np.where(v >= 0, F32(0.5), F32(-0.5))).astype(F32)
    return np.clip(np.trunc(t), -127, 127).astype(np.int8), s


def i8_matmul(q, wq):
    """Exact int32 dot products acc[m, n] = q[m, :] . wq[n, :] (int64 result)."""
    q = np.asarray(q)
    wq = np.asarray(wq)
    assert q.shape[1] * 127 * 127 < 2 ** 53
    return (q.astype(np.float64) @ wq.astype(np.float64).T).astype(np.int64)


def gelu_tanh(v):
    v = np.asarray(v, F32)
    u = F32(0.7978845608028654) * (v + F32(0.044715) * v * v * v)
    with np.errstate(over="ignore"):  # e^(2u) = inf gives t = 1, as on the GPU
        t = F32(1.0) - F32(2.0) / (F32(1.0) + np.exp(F32(2.0) * u, dtype=F32))
    return (F32(0.5) * v * (F32(1.0) + t)).astype(F32)


def epilogue(acc, sa, sw, bias=None, gelu=False):
    """i8gemm.hip:183-197 on acc [M, N] -> fp32 [M, N]."""
    v = (np.asarray(acc).astype(F32) * np.asarray(sa, F32)[:, None]).astype(F32)
    v = (v * np.asarray(sw, F32)[None, :]).astype(F32)
    if bias is not None:
        v = (v + np.asarray(bias, F32)[None, :]).astype(F32)
    return gelu_tanh(v) if gelu else v


def bf16_round(x):
    """fp32 -> nearest bf16 (ties to even), returned as fp32."""
    u = np.ascontiguousarray(np.asarray(x, F32)).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(F32)


def i8_linear(x, wq, sw, bias=None, gelu=False):
    """HI8Lin.__call__ (hgemm.py:126-137) on fp32 activations x [M, K]: quantise, int matmul, epilogue, bf16."""
    q, sa = quant_rows(x)
    return bf16_round(epilogue(i8_matmul(q, wq), sa, sw, bias, gelu))
