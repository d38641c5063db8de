import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; parity tests through the C ABI")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


@pytest.fixture
def no_device_error(cuda_dev):
    """Fails the test if any kernel recorded a device-side error (timeout / bounds) while it ran."""
    from periodicdent42_b200 import _capi

    assert _capi.device_error() == 0, "device error word was already set before the test"
    yield
    word = _capi.device_error()
    assert word == 0, f"device error word 0x{word:08x}"
