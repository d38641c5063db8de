"""The split-K GEMM entry point that allocates nothing (bsk_gemm_f16f32_splitk_static), through the C ABI.

It serves callers that cannot allocate device memory -- a fixed C signature with no workspace argument, or an
environment where device allocation is not permitted -- by keeping the split partials in a static device array
inside the library. Its output must match the workspace entry point's (bsk_gemm_f16f32_splitk) on the same
inputs, on two calls in a row (the array keeps the previous call's contents)."""
import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi

pytestmark = pytest.mark.gpu
TOL = 1e-3  # normwise relative error vs fp64, the fp16 GEMM bar of the other GEMM tests


def test_static_scratch_splitk_matches_workspace_entry_point_twice(cuda_dev):
    assert _capi.device_error() == 0
    # calls in a row with different shapes and split counts; none reads an earlier call's partials. The last one
    # lets the library choose the splits (one 256 x 256 output tile and a long K: 32 splits, 8 MiB of partials).
    for seed, (M, N, K, splits) in enumerate([(1024, 1024, 4096, 4), (512, 768, 8192, 8), (256, 256, 65536, 0)]):
        g = torch.Generator().manual_seed(100 + seed)
        A = torch.randn(M, K, generator=g).half()
        Bt = torch.randn(N, K, generator=g).half()
        Ad, Btd = A.to(cuda_dev), Bt.to(cuda_dev)
        c_static = torch.full((M, N), float("nan"), device=cuda_dev)
        c_ws = torch.full((M, N), float("nan"), device=cuda_dev)
        _capi.gemm_f16f32_splitk_static(Ad, Btd, c_static, splits)
        _capi.gemm_f16f32_splitk(Ad, Btd, c_ws, splits)
        torch.cuda.synchronize()
        assert torch.isfinite(c_static).all()
        assert ref.normwise_rel_err(c_static.cpu(), c_ws.cpu()) <= 1e-6
        assert ref.normwise_rel_err(c_static.cpu(), ref.dense_fp64(A, Bt)) <= TOL
    assert _capi.device_error() == 0


def test_static_scratch_rejects_sizes_beyond_its_maximum(cuda_dev):
    A = torch.zeros(2048, 8192, dtype=torch.float16, device=cuda_dev)
    Bt = torch.zeros(2048, 8192, dtype=torch.float16, device=cuda_dev)
    C = torch.empty(2048, 2048, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:  # 4 splits x 2048 x 2048 x 4 B = 64 MiB > 32 MiB
        _capi.gemm_f16f32_splitk_static(A, Bt, C, 4)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG and "static scratch" in str(e.value)
