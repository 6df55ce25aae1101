import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built native extension")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from reelcache_b200.ops import _ext

    _ext.ext()  # GPU tests must run the native path: fail loudly when it is missing
    return torch.device("cuda", 0)
