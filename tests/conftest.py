import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libvt_b200.so; run with -m gpu")


@pytest.fixture(scope="session", autouse=True)
def _threads():
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
