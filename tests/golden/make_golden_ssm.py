"""Generate tests/golden/ssm_ref_cases.npz from the reference's own recurrent-block restatement,
tapnext/npu/pack8.py:252-279 (ssm_ref), imported read-only from a checkout of the reference.

ssm_ref needs only numpy and ml_dtypes, but pack8 imports the NPU toolchain's packers at module level
(pack.py -> aie.utils.bfp); empty stand-in modules for `aie` / `aie.utils` let the import finish -- none of
their code is used by ssm_ref.  Run once where the reference is available:

    python tests/golden/make_golden_ssm.py /path/to/reference

Inputs are seeded (numpy PCG64): bf16-valued activations, conv taps, gate weights and biases of the
reference's shapes for one head (64 channels), 96 rows, for a first frame (no state) and a later frame.

A second file, rglru_ref_cases.npz, pins the dense-gate RG-LRU restatement of the TAPNext-style step
(oracle/tapnext_ref.py rglru): ssm_ref is run for all 12 heads (48 rows, distinct seeded weights per head)
with the conv taps set to the identity (w = [0, 0, 0, 1], bias 0, so the conv output is x itself).  Then
ssm_ref's h is exactly the RG-LRU of x with a 768 x 768 gate matrix that is block-diagonal in 12 blocks
of 64 x 64 (the reference's gate structure, pack8.py:124-129), for a first frame and the next one (whose
state is the first frame's h).
"""
import os
import sys
import types

import numpy as np
from ml_dtypes import bfloat16


def load_ssm_ref(ref_root):
    for name in ("aie", "aie.utils"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["aie"].utils = sys.modules["aie.utils"]
    sys.modules["aie.utils"].bfp = types.ModuleType("bfp")
    sys.path.insert(0, os.path.join(ref_root, "tapnext", "npu"))
    import pack8  # noqa: E402
    return pack8.ssm_ref


def bfv(a):
    return np.asarray(a, np.float32).astype(bfloat16).astype(np.float32)


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python " + os.path.basename(__file__) + " /path/to/reference")
    ref_root = sys.argv[1]
    ssm_ref = load_ssm_ref(ref_root)
    rng = np.random.Generator(np.random.PCG64(20261202))
    R, C = 96, 64
    out = {}
    for case, first in (("first", True), ("next", False)):
        y = bfv(rng.standard_normal((R, C)))
        x, xm1, xm2, xm3 = [bfv(rng.standard_normal((R, C))) for _ in range(4)]
        h0 = rng.standard_normal((R, C)).astype(np.float32)
        conv_w = bfv(rng.standard_normal((4, C)) * 0.5)
        conv_b = bfv(rng.standard_normal(C) * 0.1)
        a_param = bfv(rng.standard_normal(C))
        wx = bfv(rng.standard_normal((C, C)) * 0.15)
        wa = bfv(rng.standard_normal((C, C)) * 0.15)
        bx = bfv(rng.standard_normal(C) * 0.1)
        ba = bfv(rng.standard_normal(C) * 0.1)
        z, h = ssm_ref(y, x, xm1, xm2, xm3, h0, conv_w, conv_b, a_param, wx, bx, wa, ba, first)
        for k, v in dict(y=y, x=x, xm1=xm1, xm2=xm2, xm3=xm3, h0=h0, conv_w=conv_w, conv_b=conv_b, a_param=a_param,
                         wx=wx, bx=bx, wa=wa, ba=ba, z=np.asarray(z, np.float32), h=np.asarray(h, np.float32)).items():
            out[f"{case}.{k}"] = v
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ssm_ref_cases.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, sum(v.nbytes for v in out.values()), "bytes")

    # 12 heads, identity conv: ssm_ref's h = RG-LRU(x) with block-diagonal gates; one block's weights, two
    # frames of a stream (the second frame's state is the first frame's h)
    rng = np.random.Generator(np.random.PCG64(20261203))
    R, H = 48, 12
    ident_w = np.zeros((4, C), np.float32)
    ident_w[3] = 1.0
    zero_b = np.zeros(C, np.float32)
    zeros = np.zeros((R, C), np.float32)
    wx = bfv(rng.standard_normal((H, C, C)) * 0.15)
    wa = bfv(rng.standard_normal((H, C, C)) * 0.15)
    bx = bfv(rng.standard_normal((H, C)) * 0.1)
    ba = bfv(rng.standard_normal((H, C)) * 0.1)
    a_param = bfv(rng.standard_normal((H, C)))
    out = dict(wx=wx, bx=bx, wa=wa, ba=ba, a_param=a_param)
    h_prev = np.zeros((R, H * C), np.float32)
    for case, first in (("first", True), ("next", False)):
        x = bfv(rng.standard_normal((R, H * C)))
        h = np.zeros((R, H * C), np.float32)
        for q in range(H):
            cs = slice(q * C, (q + 1) * C)
            _, hq = ssm_ref(zeros, x[:, cs], zeros, zeros, zeros, h_prev[:, cs], ident_w, zero_b, a_param[q],
                            wx[q], bx[q], wa[q], ba[q], first)
            h[:, cs] = np.asarray(hq, np.float32)
        out[f"{case}.x"] = x
        out[f"{case}.h"] = h
        h_prev = h
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rglru_ref_cases.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
