import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA library through its C ABI")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail loudly without one (no CPU fallback)."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert major == 10, f"libchpl targets sm_100a, found sm_{major}{minor}"
    torch.cuda.init()
    return torch.device("cuda:0")
