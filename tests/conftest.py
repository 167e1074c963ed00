import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA extension")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without a CUDA device")
    return torch.device("cuda", 0)
