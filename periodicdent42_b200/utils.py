"""Sparse-matrix utilities of the reference (BlackwellSparseK/python/utils.py), same signatures."""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def convert_to_bsr(matrix: torch.Tensor, block_size: int = 16, sparsity_threshold: float = 0.5) -> torch.Tensor:
    """Dense / CSR / COO -> BSR with square ``block_size`` blocks (utils.py:10-57). BSR input is returned
    unchanged. Warns (prints, as the reference does) when the matrix is less sparse than the threshold.

    CUDA matrices (fp16 / bf16 / fp32; dense, CSR, or COO) are converted on the GPU by the library's converter
    kernels (one pass over the matrix for the block pattern and the nonzero count, one for the blocks), with
    the result torch's ``to_sparse_bsr`` gives; CPU matrices go through torch as in the reference. The sm_100
    SpMM computes on 128x128 blocks; ``sparse_mm`` re-blocks other sizes itself."""
    if matrix.layout == torch.sparse_bsr:
        return matrix
    if matrix.is_cuda and matrix.dtype in (torch.float16, torch.bfloat16, torch.float32) and matrix.dim() == 2:
        from . import _capi

        M, K = matrix.shape
        if matrix.layout == torch.sparse_coo:
            matrix = matrix.coalesce().to_sparse_csr()
        if matrix.layout == torch.sparse_csr:
            rp, ci, vals, nnz = _capi.csr_to_bsr(matrix.crow_indices(), matrix.col_indices(), matrix.values(),
                                                 (M, K), block_size)
        elif matrix.layout == torch.strided:
            dense = matrix if matrix.stride(1) == 1 or matrix.numel() == 0 else matrix.contiguous()
            rp, ci, vals, nnz = _capi.dense_to_bsr(dense, block_size)
        else:
            raise ValueError(f"Unsupported layout: {matrix.layout}")
        total = M * K
        sparsity = 1.0 - (nnz / total) if total else 0.0
        if sparsity < sparsity_threshold:
            print(f"Warning: Matrix is only {sparsity:.1%} sparse. Dense operations may be faster.")
        return torch.sparse_bsr_tensor(rp, ci, vals, size=(M, K))
    if matrix.layout != torch.strided:
        matrix = matrix.to_dense()
    nnz = torch.count_nonzero(matrix).item()
    total = matrix.numel()
    sparsity = 1.0 - (nnz / total) if total else 0.0
    if sparsity < sparsity_threshold:
        print(f"Warning: Matrix is only {sparsity:.1%} sparse. Dense operations may be faster.")
    return matrix.to_sparse_bsr(blocksize=(block_size, block_size))


def validate_sparse_matrix(matrix: torch.Tensor, expected_sparsity: Optional[float] = None,
                           min_sparsity: float = 0.5) -> Tuple[bool, dict]:
    """(is_valid, info) with the reference's keys and messages (utils.py:60-144). Sparsity counts the
    stored values (``values().numel()``) against the matrix size."""
    info = {}
    if matrix.layout not in (torch.sparse_coo, torch.sparse_csr, torch.sparse_bsr, torch.sparse_csc,
                             torch.sparse_bsc):
        return False, {"message": "Matrix is not sparse", "recommendation": "Convert to sparse format or use dense GEMM"}
    if not matrix.is_cuda:
        return False, {"message": "Matrix is not on CUDA device", "recommendation": "Move to CUDA: matrix.cuda()"}
    if matrix.dtype not in (torch.float16, torch.float32):
        return False, {"message": f"Unsupported dtype: {matrix.dtype}", "recommendation": "Use float16 or float32"}
    nnz = matrix.values().numel() if matrix.layout != torch.sparse_coo else matrix._values().numel()
    total = matrix.shape[0] * matrix.shape[1]
    sparsity = 1.0 - (nnz / total)
    info["sparsity"] = sparsity
    info["nnz"] = nnz
    info["shape"] = tuple(matrix.shape)
    if sparsity < min_sparsity:
        return False, {**info, "message": f"Sparsity {sparsity:.1%} < minimum {min_sparsity:.1%}",
                       "recommendation": f"Use dense GEMM for <{min_sparsity:.0%} sparsity"}
    if expected_sparsity is not None and abs(sparsity - expected_sparsity) > 0.1:
        info["warning"] = f"Sparsity {sparsity:.1%} deviates from expected {expected_sparsity:.1%}"
    if 0.7 <= sparsity <= 0.9:
        info["performance_rating"] = "optimal"
    elif 0.5 <= sparsity < 0.7:
        info["performance_rating"] = "good"
    elif 0.9 < sparsity:
        info["performance_rating"] = "very_sparse"
        info["note"] = "Consider structured sparsity formats"
    return True, info


def get_optimal_block_size(matrix_shape: Tuple[int, int]) -> int:
    """Block size for BSR input on B200 (utils.py:147-172 picked 8/16/32 by size for WMMA kernels): the
    tcgen05 kernel's M tile is 128, so 128x128 blocks avoid any re-blocking."""
    return 128
