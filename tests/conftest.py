"""Shared test setup. GPU tests carry @pytest.mark.gpu; everything else runs
on a CPU-only machine (the CUDA library still loads there, it just finds no
device)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle and the CUDA library once per session if missing."""
    from oracle import oracle as O
    O.build()
    from eakv_b200 import build as B
    if not os.path.exists(B.LIB):
        B.build()
    yield


@pytest.fixture
def gpu():
    if not HAS_GPU:
        pytest.skip("no CUDA device")
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def golden(name):
    import numpy as np
    return np.load(os.path.join(GOLDEN, name))
