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


# BSR SpMM throughput per device at each device's validation workload, in TFLOPS of stored-block FLOPs, with torch's
# sparse path (torch.sparse.mm) and CUTLASS timed on the same device where a figure exists:
#   device: (this operator, torch.sparse.mm, CUTLASS or None, SMs, concurrent output tiles per SM, tile rows x cols,
#            where the figures come from)
# B200 is this build, measured; L4 / A100 / H100 keep the figures the reference's estimator is built on
# (BlackwellSparseK/python/utils.py:195-212: its L4 measurement and its projections from it).
_SPMM_DEVICES = {
    "B200": (1015.0, 3.93, None, 148, 0.5, (128, 512),
             "this build measured on B200 (8192^3, 128x128 blocks, 16 of 64 per block-row; torch.sparse.mm on the "
             "same matrix in CSR fp16)"),
    "H100": (580.0, 9.6, 330.0, 132, 1.0, (256, 128), "the reference's projection from its L4 measurement"),
    "A100": (312.0, 5.2, 180.0, 108, 1.0, (256, 128), "the reference's projection from its L4 measurement"),
    "L4": (52.1, 0.87, 30.0, 58, 1.0, (256, 128), "the reference's L4 measurement (8192^2, 78 % sparse)"),
}


def _wave_efficiency(M: int, N: int, sms: int, per_sm: float, tile) -> float:
    """Fraction of the GPU's tile slots the persistent kernel keeps busy over a shape's output tiles."""
    tiles = -(-max(M, 1) // tile[0]) * -(-max(N, 1) // tile[1])
    slots = max(1, int(sms * per_sm))
    return tiles / (-(-tiles // slots) * slots)


def estimate_speedup(matrix_shape: Tuple[int, int], sparsity: float, device: str = "B200") -> dict:
    """Estimated BSR SpMM throughput for an M x N output on `device`, with the reference's result keys
    (utils.py:172-236). The estimate scales the device's measured throughput at its validation workload by how well
    the shape's output tiles fill the GPU (a shape with few tiles leaves SMs idle in its last wave) relative to
    that workload; ``tflops`` counts the FLOPs of the stored blocks (what the kernel executes), so to first order
    it does not depend on ``sparsity``. Unknown devices raise ``ValueError`` as in the reference."""
    if device not in _SPMM_DEVICES:
        raise ValueError(f"Unknown device: {device}")
    ours, torch_tf, cutlass_tf, sms, per_sm, tile, basis = _SPMM_DEVICES[device]
    M, N = matrix_shape
    f = _wave_efficiency(M, N, sms, per_sm, tile) / _wave_efficiency(8192, 8192, sms, per_sm, tile)
    tflops = ours * f
    return {
        "device": device,
        "matrix_shape": matrix_shape,
        "sparsity": sparsity,
        "tflops": tflops,
        "speedup_vs_pytorch": tflops / torch_tf,
        "speedup_vs_cutlass": (tflops / cutlass_tf) if cutlass_tf else None,
        "note": f"Scaled by output-tile occupancy from {basis}",
    }
