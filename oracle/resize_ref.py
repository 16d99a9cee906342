"""CPU restatement of the image squash of FastMD2.set_image -- TEST INFRASTRUCTURE (only tests/ import it).

The reference resizes every frame to 378 x 378 with Pillow's LANCZOS filter on the host
(moondream/gpu/md2fast.py:223-228: img.resize((IMG, IMG), Image.Resampling.LANCZOS)).  That algorithm lives in
a third-party dependency, Pillow (12.2.0 in this image; its C resampler, Resample.c, is not part of the
reference).  This module restates Pillow's published two-pass resampling for 8-bit images:
  * per output coordinate, a window of input samples around center = (x + 0.5) * scale with support
    3 * max(scale, 1), weights lanczos((x_in - center + 0.5) / max(scale, 1)), lanczos(t) = sinc(t) sinc(t/3)
    for -3 <= t < 3, normalised to sum 1, then quantised to fixed point with 22 fraction bits
    (round half away from zero);
  * a horizontal pass over the rows the vertical pass needs, then a vertical pass: each an integer sum
    2^21 + sum(pixel * weight), shifted right 22 bits and clipped to 0 .. 255 (uint8 between the passes).
It is pinned bit-exactly against Pillow's own output (tests/test_oracle_golden.py, which calls Pillow here).
"""
import math

import numpy as np

PRECISION_BITS = 32 - 8 - 2
SUPPORT = 3.0


def _sinc(x):
    if x == 0.0:
        return 1.0
    x = x * math.pi
    return math.sin(x) / x


def lanczos(x):
    return _sinc(x) * _sinc(x / 3.0) if -3.0 <= x < 3.0 else 0.0


def coeffs(in_size, out_size):
    """(bounds [out, 2] int32 = (first input index, count), weights [out, ksize] int32 fixed point)."""
    scale = in_size / out_size
    filterscale = max(scale, 1.0)
    support = SUPPORT * filterscale
    ksize = int(math.ceil(support)) * 2 + 1
    bounds = np.zeros((out_size, 2), np.int32)
    kk = np.zeros((out_size, ksize), np.float64)
    for xx in range(out_size):
        center = (xx + 0.5) * scale
        ss = 1.0 / filterscale
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), in_size) - xmin
        w = [lanczos((x + xmin - center + 0.5) * ss) for x in range(xmax)]
        ww = sum(w)
        for x in range(xmax):
            kk[xx, x] = w[x] / ww if ww != 0.0 else w[x]
        bounds[xx] = (xmin, xmax)
    one = float(1 << PRECISION_BITS)
    q = np.where(kk < 0, np.trunc(-0.5 + kk * one), np.trunc(0.5 + kk * one)).astype(np.int64).astype(np.int32)
    return bounds, q


def _pass(src, bounds, k, axis):
    """One integer pass along `axis` (1: columns of each row, 0: rows) of a uint8 [H, W, C] image."""
    out_n = bounds.shape[0]
    shape = list(src.shape)
    shape[axis] = out_n
    out = np.empty(shape, np.uint8)
    s = src.astype(np.int64)
    for o in range(out_n):
        x0, n = int(bounds[o, 0]), int(bounds[o, 1])
        w = k[o, :n].astype(np.int64)
        win = s[:, x0:x0 + n] if axis == 1 else s[x0:x0 + n]
        acc = (1 << (PRECISION_BITS - 1)) + np.tensordot(win, w, axes=([axis], [0]))
        val = np.clip(acc >> PRECISION_BITS, 0, 255).astype(np.uint8)
        if axis == 1:
            out[:, o] = val
        else:
            out[o] = val
    return out


def resize_lanczos(img, out_w, out_h):
    """uint8 [H, W, 3] -> uint8 [out_h, out_w, 3], Pillow's two-pass LANCZOS (horizontal first, only over
    the rows the vertical pass reads)."""
    H, W = img.shape[:2]
    bh, kh = coeffs(W, out_w)
    bv, kv = coeffs(H, out_h)
    y_first = int(bv[0, 0])
    y_last = int(bv[-1, 0] + bv[-1, 1])
    tmp = img[y_first:y_last] if out_w == W else _pass(img[y_first:y_last], bh, kh, axis=1)
    if out_h == H:
        return tmp
    bv = bv.copy()
    bv[:, 0] -= y_first
    return _pass(tmp, bv, kv, axis=0)
