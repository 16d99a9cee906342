"""Failure detection on the GPU without a fault: every kernel's waits on mbarriers are bounded, and a wait that
runs out sets its CTA's abort flag (the CTA's other roles leave their own waits) and a bit of the device status
word that vt_device_status reads.  vt_wait_selftest runs that protocol on two barriers nothing completes: one
wait with a short limit, one with the kernels' own ~2 s limit that has to leave on the abort flag.  Afterwards
the context is still usable."""
import time

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200 import ops
from strix_halo_maxx_b200._lib import lib, device_status

DEV = "cuda"
ST_SELFTEST = 1 << 8


def test_bounded_wait_gives_up_sets_the_status_and_releases_the_other_waiter():
    device_status(clear=True)
    result = torch.full((2,), -1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib().vt_wait_selftest(torch.cuda.current_stream().cuda_stream, 2_000_000, result.data_ptr())
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert rc == 0, lib().vt_last_error_string()
    assert result.tolist() == [0, 0]                 # both waits gave up instead of returning "complete"
    assert device_status(clear=True) == ST_SELFTEST  # the site bit, and nothing else
    assert dt < 1.0, dt                              # the long wait left on the abort flag, not its own ~2 s limit
    # the context is still usable: a GEMM right after gives the right answer and records nothing
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(300, 1152, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(1152, 1152, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    out = ops.VtLin(w, None)(x)
    ref = F.linear(x.float(), w.float())
    assert float((out.float() - ref).norm() / ref.norm()) < 5e-3
    assert device_status(clear=True) == 0


def test_selftest_rejects_bad_limits():
    result = torch.zeros(2, dtype=torch.int32, device=DEV)
    assert lib().vt_wait_selftest(None, 10, result.data_ptr()) == -2
    assert lib().vt_wait_selftest(None, 2_000_000, None) == -2
