import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


@pytest.fixture(scope="session")
def require_gpu():
    if not gpu_available():
        pytest.fail("this test needs an sm_100 GPU (run with -m 'not gpu' on CPU)")
