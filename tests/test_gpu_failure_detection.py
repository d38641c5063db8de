"""Failure detection on the GPU without a fault: a bounded device wait on a barrier nothing completes
runs out, the kernel records the timeout in the device error word and returns, and the context stays
usable for the next launch."""
import pytest
import torch

from periodicdent42_b200 import _capi

pytestmark = pytest.mark.gpu


def test_wait_timeout_reported_and_context_survives(cuda_dev):
    rc = _capi.selftest_wait_timeout(1_000_000)  # 1 ms limit
    assert rc == _capi.BSK_ERR_DEVICE_TIMEOUT, _capi.last_error()
    assert _capi.device_error() == 0  # the self-test clears what it read
    x = torch.arange(1024, device=cuda_dev, dtype=torch.float32)
    assert x.sum().item() == 1024 * 1023 / 2
    A = torch.ones(128, 64, dtype=torch.float16, device=cuda_dev)
    C = torch.empty(128, 256, device=cuda_dev)
    _capi.gemm_f16f32(A, torch.ones(256, 64, dtype=torch.float16, device=cuda_dev), C)
    torch.cuda.synchronize()
    assert torch.all(C == 64.0)
    assert _capi.device_error() == 0
