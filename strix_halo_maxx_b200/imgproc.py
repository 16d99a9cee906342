"""Frame input on the GPU: JPEG decode and the 378 x 378 LANCZOS squash of FastMD2.set_image
(moondream/gpu/md2fast.py:223-228), which the reference runs on the host with Pillow.

* decode_jpeg: nvJPEG through torchvision.io.decode_jpeg(device="cuda") (a library decoder; its output can
  differ from Pillow's libjpeg by a few levels where the IDCT / chroma upsampling round differently);
* resize_lanczos: Pillow's two-pass fixed-point LANCZOS resampling (Resample.c of Pillow 12.2, published
  source) restated: per output coordinate a window around center = (x + 0.5) * scale, support 3 * max(scale, 1),
  weights sinc(t) sinc(t / 3) normalised and quantised to 22 fraction bits; the horizontal pass over the rows
  the vertical pass reads, then the vertical pass, each clipping to uint8 -- so the result equals Pillow's
  img.resize(..., LANCZOS) bit for bit (tests/test_imgproc_gpu.py).  The weight tables are computed here once
  per size pair with the same double-precision steps (math.sin is the C library's sin, as in Pillow).
"""
import math

import numpy as np
import torch

from ._lib import lib, check
from .ops import _stream

PREC = 22
_TABLES = {}


def _lanczos(x):
    def sinc(v):
        if v == 0.0:
            return 1.0
        v *= math.pi
        return math.sin(v) / v
    return sinc(x) * sinc(x / 3.0) if -3.0 <= x < 3.0 else 0.0


def resize_tables(in_size, out_size, device):
    """(bounds int32 [out, 2] = (first input index, count), weights int32 [out, ksize], ksize, (first, end) of
    the input range the whole output reads) with the tables on `device`."""
    key = (in_size, out_size, str(device))
    if key in _TABLES:
        return _TABLES[key]
    scale = in_size / out_size
    fs = scale if scale > 1.0 else 1.0
    support = 3.0 * fs
    ksize = int(math.ceil(support)) * 2 + 1
    bounds = np.zeros((out_size, 2), np.int32)
    w = np.zeros((out_size, ksize), np.int32)
    one = float(1 << PREC)
    for o in range(out_size):
        center = (o + 0.5) * scale
        x0 = max(int(center - support + 0.5), 0)
        n = min(int(center + support + 0.5), in_size) - x0
        ks = [_lanczos((k + x0 - center + 0.5) / fs) for k in range(n)]
        tot = sum(ks)
        for k in range(n):
            v = ks[k] / tot if tot != 0.0 else ks[k]
            w[o, k] = int(-0.5 + v * one) if v < 0 else int(0.5 + v * one)
        bounds[o] = (x0, n)
    t = (torch.from_numpy(bounds).to(device), torch.from_numpy(w).to(device), ksize,
         (int(bounds[0, 0]), int(bounds[-1, 0] + bounds[-1, 1])))
    _TABLES[key] = t
    return t


def _pass(inp, sa, sb, sc, out, oa, ob, oc, n_out, n_other, bounds, weights, ksize):
    rc = lib().vt_resize_pass_u8(_stream(), inp, sa, sb, sc, out.data_ptr(), oa, ob, oc, n_out, n_other,
                                 bounds.data_ptr(), weights.data_ptr(), ksize)
    check(rc, "vt_resize_pass_u8")


def resize_lanczos(img, out_h=378, out_w=378, chw=False, out=None):
    """uint8 image on the device, [H, W, 3] (or [3, H, W] with chw=True) -> [out_h, out_w, 3] uint8."""
    assert img.dtype == torch.uint8 and img.is_cuda
    H, W = (img.shape[1], img.shape[2]) if chw else (img.shape[0], img.shape[1])
    sc, sy, sx = (img.stride(0), img.stride(1), img.stride(2)) if chw else (img.stride(2), img.stride(0), img.stride(1))
    dev = img.device
    bh, kh, ksh, _ = resize_tables(W, out_w, dev)
    bv, kv, ksv, (y0, y1) = resize_tables(H, out_h, dev)
    rows = y1 - y0
    if out is None:
        out = torch.empty(out_h, out_w, 3, dtype=torch.uint8, device=dev)
    tmp = torch.empty(rows, out_w, 3, dtype=torch.uint8, device=dev)
    # horizontal: resampled axis x, other axis the rows y0 .. y1
    _pass(img.data_ptr() + y0 * sy, sx, sy, sc, tmp, 3, out_w * 3, 1, out_w, rows, bh, kh, ksh)
    # vertical: resampled axis the rows of tmp (bounds shifted by y0), other axis x
    key = (H, out_h, str(dev), "shifted")
    bvs = _TABLES.get(key)
    if bvs is None:
        bvs = _TABLES[key] = bv - torch.tensor([y0, 0], dtype=torch.int32, device=dev)
    _pass(tmp.data_ptr(), out_w * 3, 3, 1, out, out_w * 3, 3, 1, out_h, out_w, bvs, kv, ksv)
    return out


def decode_jpeg(data, device="cuda"):
    """JPEG bytes -> [3, H, W] uint8 RGB on the device (nvJPEG via torchvision)."""
    import torchvision
    t = torch.frombuffer(bytearray(data), dtype=torch.uint8)
    return torchvision.io.decode_jpeg(t, mode=torchvision.io.ImageReadMode.RGB, device=device)


def load_frame(data, device="cuda", out=None):
    """JPEG bytes -> the tower's [378, 378, 3] uint8 input on the device: decode, then the LANCZOS squash."""
    return resize_lanczos(decode_jpeg(data, device), 378, 378, chw=True, out=out)
