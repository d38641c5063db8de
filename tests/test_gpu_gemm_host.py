"""Accumulating GEMM (C += A B over a K range) and the host-streaming GEMM (operands and result in host
memory, K streamed in chunks) through the C ABI, against the fp64 recompute of the oracle.
Tolerance: normwise relative error <= 1e-3 against fp64 (the fp16 bar of the dense GEMM)."""
import pytest
import torch

import periodicdent42_b200 as bsk
from oracle import reference_path as ref
from periodicdent42_b200 import _capi

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _operands(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    Bt = (torch.rand(N, K, generator=g) * 2 - 1).half()
    C0 = torch.rand(M, N, generator=g) * 4 - 2
    return A, Bt, C0


@pytest.mark.parametrize("tile", ["single", "pair", "wide"])
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (200, 520, 264), (130, 130, 136), (384, 1024, 8192)])
def test_gemm_acc_adds_to_c(no_device_error, monkeypatch, tile, M, N, K):
    monkeypatch.setenv("BSK_GEMM_TILE", tile)
    A, Bt, C0 = _operands(M, N, K, M + N + K)
    dev = torch.device("cuda", 0)
    C = C0.to(dev)
    _capi.gemm_f16f32_acc(A.to(dev), Bt.to(dev), C)
    torch.cuda.synchronize()
    want = C0.double() + ref.dense_fp64(A, Bt)
    err = ref.normwise_rel_err(C.cpu(), want)
    assert err <= TOL, err


def test_gemm_acc_k_pieces_equal_one_pass(no_device_error):
    """K swept in four accumulated pieces agrees with the single pass to fp32 rounding of the partial sums."""
    M, N, K = 512, 768, 4096
    A, Bt, _ = _operands(M, N, K, 7)
    dev = torch.device("cuda", 0)
    Ad, Btd = A.to(dev), Bt.to(dev)
    C = torch.full((M, N), float("nan"), device=dev)
    _capi.gemm_f16f32(Ad, Btd, C, 0, 1024)
    for k0 in (1024, 2048, 3072):
        _capi.gemm_f16f32_acc(Ad, Btd, C, k0, k0 + 1024)
    one = torch.empty(M, N, device=dev)
    _capi.gemm_f16f32(Ad, Btd, one)
    torch.cuda.synchronize()
    want = ref.dense_fp64(A, Bt)
    assert ref.normwise_rel_err(C.cpu(), want) <= TOL
    assert ref.normwise_rel_err(C.cpu(), one.cpu()) <= 1e-5


def test_gemm_acc_empty_range_leaves_c(no_device_error):
    A, Bt, C0 = _operands(128, 256, 128, 3)
    dev = torch.device("cuda", 0)
    C = C0.to(dev)
    _capi.gemm_f16f32_acc(A.to(dev), Bt.to(dev), C, 64, 64)
    torch.cuda.synchronize()
    assert torch.equal(C.cpu(), C0)


@pytest.mark.parametrize("M,N,K,k_chunk", [(512, 1024, 4096, 1024), (300, 520, 1000, 256), (256, 256, 64, 0),
                                           (1024, 1024, 20000, 0), (130, 136, 72, 64),
                                           # the last chunk goes by row panels (~M/8 rounded up to 256 rows):
                                           # several panels with a ragged last one, and a single-chunk call
                                           (2600, 520, 3000, 1024), (2048, 264, 64, 0), (3000, 384, 9000, 0)])
def test_gemm_from_host(no_device_error, M, N, K, k_chunk):
    A, Bt, _ = _operands(M, N, K, 11 + M)
    A_h, Bt_h = A.pin_memory(), Bt.pin_memory()
    C = bsk.gemm_from_host(A_h, Bt_h.t(), k_chunk=k_chunk)
    assert not C.is_cuda and C.shape == (M, N)
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, err


def test_gemm_from_host_strided_and_pageable(no_device_error):
    """Row strides larger than K on the host side, pageable (not pinned) memory, an explicit `out`."""
    M, N, K = 256, 512, 2048
    A_big, Bt_big, _ = _operands(M, N, K + 64, 5)
    A, Bt = A_big[:, :K], Bt_big[:, :K]
    out = torch.full((M, N + 8), float("nan"))[:, :N]
    C = bsk.gemm_from_host(A, Bt.t(), out=out, k_chunk=512)
    assert C.data_ptr() == out.data_ptr()
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, err


def test_gemm_from_host_repeated_calls_identical(no_device_error):
    A, Bt, _ = _operands(512, 512, 8192, 9)
    A_h, Bt_h = A.pin_memory(), Bt.pin_memory()
    c1 = bsk.gemm_from_host(A_h, Bt_h.t(), k_chunk=2048)
    c2 = bsk.gemm_from_host(A_h, Bt_h.t(), k_chunk=2048)
    assert torch.equal(c1, c2)


def test_gemm_host_workspace_contract(cuda_dev):
    need = _capi.gemm_host_workspace_bytes(512, 512, 4096, 1024)
    assert need == 2 * 512 * 1024 * 2 * 2 + 512 * 512 * 4
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_host_workspace_bytes(512, 512, 4096, 100)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
    A = torch.zeros(512, 4096, dtype=torch.float16)
    C = torch.zeros(512, 512)
    ws = torch.empty(need - 256, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32_host(A, A, C, ws, 1024)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
