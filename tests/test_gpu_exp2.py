"""Accuracy of the attention softmax's exponentials on the device (bsk_selftest_exp2).

A quarter of the softmax's 2^x values (forward and both backward passes) come from a polynomial on the FMA pipe
instead of the MUFU: x = n + f with n = round(x), f in [-1/2, 1/2], 2^f by a cubic fitted for this library, and n
added to the exponent field; inputs below -125 are clamped to -125. Its stated bound is a maximum relative error
of 1.01e-4; the test holds it to 1.1e-4 against the fp64 value of 2^x and against CUDA's exp2f (torch.exp2 on the
device), over a dense sweep of [-125, 0] (the range the softmax produces: x = s*c - m <= 0) and the points where
the rounding of n flips (half-integers)."""
import pytest
import torch

from periodicdent42_b200 import _capi

pytestmark = pytest.mark.gpu
BOUND = 1.1e-4


def _sweep(dev):
    dense = torch.linspace(-125.0, 0.0, 4_000_001, dtype=torch.float32)
    g = torch.Generator().manual_seed(3)
    rnd = torch.rand(1_000_000, generator=g) * -125.0
    halves = torch.arange(-250, 1, dtype=torch.float32) * 0.5        # f = +-1/2 at every n
    near = torch.cat([halves + 1e-6 * halves.abs().clamp(min=1), halves - 1e-6 * halves.abs().clamp(min=1)])
    x = torch.cat([dense, rnd, halves, near.clamp(-125.0, 0.0)])
    return x.to(dev)


def _run(x, fma_pipe):
    y = torch.full_like(x, float("nan"))
    _capi.selftest_exp2(x, y, fma_pipe)
    torch.cuda.synchronize()
    return y


def _max_rel(y, ref):
    return ((y.double() - ref.double()).abs() / ref.double().abs()).max().item()


def test_fma_pipe_exp2_within_bound(cuda_dev):
    x = _sweep(cuda_dev)
    y = _run(x, True)
    assert torch.isfinite(y).all()
    ref64 = torch.pow(2.0, x.double())
    err64 = _max_rel(y, ref64)
    assert err64 <= BOUND, err64
    err_cuda = _max_rel(y, torch.exp2(x))
    assert err_cuda <= BOUND, err_cuda


def test_mufu_exp2_matches_cuda(cuda_dev):
    x = _sweep(cuda_dev)
    y = _run(x, False)
    # ex2.approx is accurate to a few ulp for normal results
    assert _max_rel(y, torch.pow(2.0, x.double())) <= 1e-6


def test_fma_pipe_exp2_pairs_and_odd_length(cuda_dev):
    """Both halves of the packed pair and an odd tail element take the same route and agree with the bound."""
    x = torch.tensor([-0.5, -1.5, -3.25, 0.0, -124.75], device=cuda_dev)
    y = _run(x, True)
    assert _max_rel(y, torch.pow(2.0, x.double())) <= BOUND


def test_fma_pipe_exp2_clamps_below_range(cuda_dev):
    """Masked scores reach the exponential as -inf or very negative values: the result is the clamped 2^-125
    (relative to the real value that is garbage, but it is finite, positive and 2^-125 within the bound)."""
    x = torch.tensor([-126.0, -200.0, -1e30, float("-inf")], device=cuda_dev)
    y = _run(x, True)
    ref = torch.full_like(y, 2.0 ** -125, dtype=torch.float64)
    assert torch.isfinite(y).all() and (y > 0).all()
    assert _max_rel(y, ref) <= BOUND


def test_selftest_exp2_rejects_bad_args(cuda_dev):
    x = torch.zeros(4, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.check(_capi.lib().bsk_selftest_exp2(x.data_ptr(), x.data_ptr(), 4, 2, None), "exp2")
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
