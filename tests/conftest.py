import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "kquant_golden.npz"))


@pytest.fixture(scope="session")
def kernels():
    """The library loaded on cuda:0 (GPU tests only)."""
    import torch

    import kernite_b200 as kb

    assert torch.cuda.is_available(), "GPU test run without a GPU"
    torch.cuda.init()
    k = kb.Kernels.load(0)
    yield k
    k.device_error()
    k.close()
