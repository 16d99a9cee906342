"""Frame input on the GPU: the LANCZOS squash against Pillow (bit for bit) and the nvJPEG decode against
Pillow's decoder (within a few levels)."""
import io

import numpy as np
import pytest
import torch
from PIL import Image

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import imgproc
from strix_halo_maxx_b200._lib import device_status


def _image(h, w, seed):
    rng = np.random.default_rng(seed)
    img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    yy, xx = np.mgrid[0:h, 0:w]
    img[..., 0] = ((np.sin(xx / 17.0) * np.cos(yy / 11.0)) * 100 + 128).astype(np.uint8)
    return img


@pytest.mark.parametrize("h,w", [(480, 640), (375, 500), (1080, 1920), (300, 200), (378, 378), (97, 1201)])
@pytest.mark.parametrize("chw", [False, True])
def test_resize_lanczos_equals_pillow(h, w, chw):
    device_status(clear=True)
    img = _image(h, w, h + w)
    ref = np.asarray(Image.fromarray(img).resize((378, 378), Image.Resampling.LANCZOS))
    t = torch.from_numpy(img).cuda()
    if chw:
        t = t.permute(2, 0, 1).contiguous()
    out = imgproc.resize_lanczos(t, 378, 378, chw=chw)
    assert np.array_equal(out.cpu().numpy(), ref)
    assert device_status(clear=True) == 0


def _smooth(h, w):
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float64)
    img = np.stack([np.sin(xx / 23.0) * np.cos(yy / 17.0), np.cos(xx / 31.0 + yy / 29.0), np.sin((xx + yy) / 41.0)], -1)
    return (img * 100 + 128).clip(0, 255).astype(np.uint8)


@pytest.mark.parametrize("subsampling,max_d,mean_d", [(0, 4, 1.0), (2, 16, 2.0)])
def test_load_frame_decodes_and_squashes(subsampling, max_d, mean_d):
    """nvJPEG against Pillow's libjpeg on a smooth frame: 4:4:4 differs only by IDCT rounding; 4:2:0 also by
    the chroma upsampling.  The squash of the decoded frame is then Pillow's, bit for bit."""
    buf = io.BytesIO()
    Image.fromarray(_smooth(480, 640)).save(buf, format="JPEG", quality=92, subsampling=subsampling)
    data = buf.getvalue()
    pil = np.asarray(Image.open(io.BytesIO(data)).convert("RGB"))
    dec = imgproc.decode_jpeg(data).permute(1, 2, 0).cpu().numpy()
    d = np.abs(dec.astype(int) - pil.astype(int))
    assert d.max() <= max_d and d.mean() < mean_d, (d.max(), d.mean())
    frame = imgproc.load_frame(data)
    assert frame.shape == (378, 378, 3) and frame.dtype == torch.uint8
    ref = np.asarray(Image.fromarray(np.ascontiguousarray(dec)).resize((378, 378), Image.Resampling.LANCZOS))
    assert np.array_equal(frame.cpu().numpy(), ref)
