"""The reference's archived attention tests, case for case, through the public `attention_forward`
(BlackwellSparseK/.archive/tests/test_kernels.py:23-127): fp16 Q, K, V [B, H, S, D] from
torch.manual_seed(42) on the GPU, dense non-causal attention, compared with torch SDPA under the
reference's own tolerance (allclose rtol=1e-3, atol=2e-3, its utils/validation.py:7-68).

The reference compares with SDPA on the GPU; this file checks against both the GPU SDPA (as the reference
does) and SDPA evaluated in fp32 on the CPU from the same fp16 inputs, which is the more exact of the two."""
import pytest
import torch
import torch.nn.functional as F

import periodicdent42_b200 as bsk
from oracle import reference_path as ref

pytestmark = pytest.mark.gpu


def _inputs(B, H, S, D, dev):
    torch.manual_seed(42)
    Q = torch.randn(B, H, S, D, dtype=torch.float16, device=dev)
    K = torch.randn(B, H, S, D, dtype=torch.float16, device=dev)
    V = torch.randn(B, H, S, D, dtype=torch.float16, device=dev)
    return Q, K, V


@pytest.mark.parametrize("B,H,S,D", [(1, 8, 512, 64), (2, 16, 1024, 64), (4, 32, 2048, 64), (1, 8, 512, 128)])
def test_kernel_correctness(no_device_error, cuda_dev, B, H, S, D):
    Q, K, V = _inputs(B, H, S, D, cuda_dev)
    scale = 1.0 / (D ** 0.5)
    out = bsk.attention_forward(Q, K, V, scale=scale)
    assert out.dtype == torch.float16 and out.shape == (B, H, S, D)
    gpu_ref = F.scaled_dot_product_attention(Q, K, V, scale=scale)
    ok, m = ref.validate_correctness(out, gpu_ref, rtol=1e-3, atol=2e-3)
    assert ok, (B, H, S, D, m)
    cpu_ref = F.scaled_dot_product_attention(Q.cpu().float(), K.cpu().float(), V.cpu().float(), scale=scale)
    ok, m = ref.validate_correctness(out, cpu_ref, rtol=1e-3, atol=2e-3)
    assert ok, (B, H, S, D, m)


def test_kernel_determinism(no_device_error, cuda_dev):
    Q, K, V = _inputs(1, 8, 512, 64, cuda_dev)
    out1 = bsk.attention_forward(Q, K, V)
    out2 = bsk.attention_forward(Q, K, V)
    assert torch.equal(out1, out2)


def test_input_validation(cuda_dev):
    Q, K, V = _inputs(1, 8, 512, 64, cuda_dev)
    bsk.attention_forward(Q, K, V)
    with pytest.raises((ValueError, RuntimeError)):
        bsk.attention_forward(Q.float(), K, V)
    with pytest.raises((ValueError, RuntimeError)):
        bsk.attention_forward(Q.cpu(), K, V)
    with pytest.raises((ValueError, RuntimeError)):
        bsk.attention_forward(Q.unsqueeze(0), K, V)


@pytest.mark.parametrize("D", [32, 256])
def test_unsupported_head_dim(cuda_dev, D):
    Q, K, V = _inputs(1, 8, 512, D, cuda_dev)
    with pytest.raises((ValueError, RuntimeError)):
        bsk.attention_forward(Q, K, V)


def test_large_sequence_length(no_device_error, cuda_dev):
    Q, K, V = _inputs(1, 8, 4096, 64, cuda_dev)
    out = bsk.attention_forward(Q, K, V)
    assert out.shape == (1, 8, 4096, 64)
    assert not torch.isnan(out).any() and not torch.isinf(out).any()
    gpu_ref = F.scaled_dot_product_attention(Q, K, V)
    ok, m = ref.validate_correctness(out, gpu_ref, rtol=1e-3, atol=2e-3)
    assert ok, m


def _stream():
    import ctypes

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,H,S,D", [(1, 8, 512, 64), (1, 4, 512, 128)])
def test_reference_c_launchers(no_device_error, cuda_dev, B, H, S, D, causal):
    """launch_attention_forward / launch_attention_backward with the reference's C signatures (fp16, dense or
    causal): forward vs SDPA under the reference's tolerance; backward vs fp64 autograd (normwise <= 3 x the error
    of torch's fp16 backward + 2e-3)."""
    from periodicdent42_b200 import _capi

    Q, K, V = _inputs(B, H, S, D, cuda_dev)
    scale = 1.0 / (D ** 0.5)
    O = torch.empty_like(Q)
    lib = _capi.lib()
    lib.launch_attention_forward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), B, H, S, D, scale, causal,
                                 _stream())
    torch.cuda.synchronize()
    assert _capi.last_error() == ""
    want = F.scaled_dot_product_attention(Q.cpu().float(), K.cpu().float(), V.cpu().float(), scale=scale,
                                          is_causal=causal)
    ok, m = ref.validate_correctness(O, want, rtol=1e-3, atol=2e-3)
    assert ok, m
    dO = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(2)).half()
    dOd = dO.to(cuda_dev)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    lib.launch_attention_backward(dOd.data_ptr(), Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                  dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), B, H, S, D, scale, causal, _stream())
    torch.cuda.synchronize()
    assert _capi.last_error() == ""

    def grads(dtype):
        q, k, v = (t.cpu().to(dtype).requires_grad_(True) for t in (Q, K, V))
        F.scaled_dot_product_attention(q, k, v, scale=scale, is_causal=causal).backward(dO.to(dtype))
        return q.grad, k.grad, v.grad

    g64, g16 = grads(torch.float64), grads(torch.float16)
    for got, want64, lp in zip((dQ, dK, dV), g64, g16):
        err, base = ref.normwise_rel_err(got.cpu(), want64), ref.normwise_rel_err(lp, want64)
        assert err <= 3 * base + 2e-3, (err, base)
