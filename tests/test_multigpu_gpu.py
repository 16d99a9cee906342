"""Crop sharding on 2 or more GPUs of one box (torchrun, NCCL): the sharded 13-crop frame and the sharded crop
batch equal their single-GPU results bit for bit (per-crop features do not depend on which crops share a
launch).  Skipped on a box with one GPU; the host logic of both paths runs on CPU with gloo ranks in
tests/test_host.py."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_frame_and_crop_batch_on_two_gpus_equal_one_gpu():
    port = 29600 + os.getpid() % 1000
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "sharded_frame_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=480, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "SHARDED_OK 1" in r.stdout, r.stdout[-2000:]
