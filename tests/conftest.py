import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "w4a16-gemm_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def cuda_device():
    """A GPU test on a machine without CUDA is a configuration error, not a skip:
    fail loudly so a silent fallback can never pass for a kernel run."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch.cuda.is_available() is False")
    return torch.device("cuda", 0)
