"""Generate tests/golden/i8_quant_gemm.npz: pins oracle/i8_ref.py to the reference's int8 W8A8 numerics.

Runs the reference's own numpy restatement of HI8Lin (moondream/npu/p4/pack_i8.py: quant_rows, quant_w,
epilogue -- the "moondream-opt HI8Lin numerics" its NPU int8 path is checked against), imported read-only
from a checkout of the reference, on seeded inputs with the edge cases of the path: an all-zero activation
row and weight row (the 1e-5 / 1e-8 scale floors), a row below the activation floor, rows whose values sit
exactly on the half-way points of the int8 grid (activations round half away from zero, weights half to
even), and bf16-representable activations (what the GPU kernels read).  The exact int32 products come from a
float64 matrix product (exact at this K).

    python tests/golden/make_golden_i8.py /path/to/reference
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
M, N, K = 40, 48, 320


def bf16_representable(x):
    u = np.ascontiguousarray(x.astype(np.float32)).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def inputs():
    rng = np.random.default_rng(2024)
    x = rng.standard_normal((M, K)).astype(np.float32) * np.exp(rng.uniform(-4, 3, (M, 1))).astype(np.float32)
    x[0] = 0.0                                              # amax 0 -> scale floor 1e-5 / 127
    x[1] = rng.uniform(-4e-6, 4e-6, K)                      # below the floor
    halves = (np.arange(K) % 254 - 126.5).astype(np.float32)
    x[2] = halves                                           # amax 126.5: generic scale
    x[3] = np.where(np.arange(K) % 2 == 0, 127.0, halves)   # amax 127 -> scale 1: exact half-way points
    x[3, 1::4] *= -1
    x = bf16_representable(x)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[0] = 0.0                                              # scale floor 1e-8 / 127
    w[1] = np.where(np.arange(K) % 2 == 0, 127.0, halves)   # scale 1: ties to even
    w[2, :] = rng.standard_normal(K).astype(np.float32) * 30.0
    bias = (rng.standard_normal(N) * 0.5).astype(np.float32)
    return x, w, bias


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python " + os.path.basename(__file__) + " /path/to/reference")
    ref = sys.argv[1]
    sys.path.insert(0, os.path.join(ref, "moondream", "npu", "p4"))
    import pack_i8  # noqa: E402  (numpy only)
    x, w, bias = inputs()
    q, sx = pack_i8.quant_rows(x)
    wq, sw = pack_i8.quant_w(w)
    acc = (q.astype(np.float64) @ wq.astype(np.float64).T).astype(np.int64)
    # pack_i8.epilogue works on the weight-rows x tokens orientation: acc^T [N, M]
    y0 = pack_i8.epilogue(acc.T, sx, sw, bias, False).T
    y1 = pack_i8.epilogue(acc.T, sx, sw, bias, True).T
    np.savez_compressed(os.path.join(HERE, "i8_quant_gemm.npz"), x=x, w=w, bias=bias, q=q, sx=sx, wq=wq, sw=sw,
                        acc=acc, y0=np.ascontiguousarray(y0, np.float32), y1=np.ascontiguousarray(y1, np.float32))
    print("wrote i8_quant_gemm.npz", q.shape, wq.shape)


if __name__ == "__main__":
    main()
