"""The reference's torch CPU path for each operator, plus fp64 recomputes -- TEST INFRASTRUCTURE ONLY.

The reference's CUDA extension never ran (its binding reads int64 BSR indices as int32 and its launcher
references uninstantiated templates), so the path every reference benchmark and test actually checks
against is torch:
  dense GEMM   torch.matmul / torch.mm on fp32-upcast operands
               (BlackwellSparseK/benchmarks/comprehensive_benchmark.py:176-185,
                BlackwellSparseK/benchmarks/compare_all_baselines.py:184-233)
  BSR SpMM     torch.sparse.mm (BlackwellSparseK/python/ops.py:117-120,
               BlackwellSparseK/benchmarks/comprehensive_benchmark.py:133); fp16 BSR is not implemented
               on CPU, hence the fp32 upcast
  attention    F.scaled_dot_product_attention (…/blackwell_sparsek/kernels/sparsek.py:92-98,
               BlackwellSparseK/.archive/tests/test_kernels.py:38-40); the block mask enters as a dense
               boolean attn_mask
  FP8 GEMM     no reference implementation exists; torch._scaled_mm with per-tensor scales is the
               stated semantics (quantisation recipe: docs/validation/FP8_VALIDATION_BLOCKED.txt:64)
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


# ----------------------------------------------------------------------------------------- metrics
def normwise_rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    """||out - ref||_F / ||ref||_F in fp64."""
    o = out.detach().to("cpu", torch.float64)
    r = ref.detach().to("cpu", torch.float64)
    den = torch.linalg.vector_norm(r).item()
    num = torch.linalg.vector_norm(o - r).item()
    return num / den if den > 0 else num


def validate_correctness(output: torch.Tensor, reference: torch.Tensor, rtol: float = 1e-3, atol: float = 2e-3):
    """allclose(rtol, atol) plus difference statistics, as the reference's validation helper reports them
    (BlackwellSparseK/.archive/src_experiments/blackwell_sparsek/utils/validation.py:7-68)."""
    o = output.detach().to("cpu", torch.float64)
    r = reference.detach().to("cpu", torch.float64)
    diff = (o - r).abs()
    metrics = {
        "max_diff": diff.max().item() if diff.numel() else 0.0,
        "mean_diff": diff.mean().item() if diff.numel() else 0.0,
        "num_elements": diff.numel(),
    }
    ok = bool(torch.allclose(o, r, rtol=rtol, atol=atol))
    if not ok:
        bad = diff > (atol + rtol * r.abs())
        metrics["num_mismatches"] = int(bad.sum().item())
        metrics["mismatch_rate"] = float(bad.double().mean().item())
    return ok, metrics


def bf16_storage_floor(ref64: torch.Tensor) -> float:
    """Normwise error of merely rounding the exact result to bf16: the floor any bf16-output kernel sits on."""
    return normwise_rel_err(ref64.to(torch.bfloat16), ref64)


# ----------------------------------------------------------------------------------------- dense GEMM
def dense_ref(A: torch.Tensor, Bt: torch.Tensor) -> torch.Tensor:
    """Reference torch path: torch.matmul on fp32-upcast operands (B column-major given as Bt [N,K])."""
    return torch.matmul(A.float(), Bt.float().t())


def dense_fp64(A: torch.Tensor, Bt: torch.Tensor) -> torch.Tensor:
    return A.double() @ Bt.double().t()


def dense_fp64_sampled(A: torch.Tensor, Bt: torch.Tensor, rows, cols) -> torch.Tensor:
    """fp64 recompute of C[rows][:, cols] only (the full K=237568 product is ~3e16 flop)."""
    return A[rows].double() @ Bt[cols].double().t()


# ----------------------------------------------------------------------------------------- FP8 GEMM
def fp8_ref(Aq: torch.Tensor, Bqt: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor) -> torch.Tensor:
    """torch._scaled_mm(A_q, B_q, scale_a, scale_b, out_dtype=bfloat16) on CPU; B_q column-major = Bqt^T."""
    return torch._scaled_mm(Aq, Bqt.t(), scale_a=sa.reshape(()), scale_b=sb.reshape(()), out_dtype=torch.bfloat16)


def fp8_fp64(Aq: torch.Tensor, Bqt: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor) -> torch.Tensor:
    """fp64 recompute on the dequantised operands (the same e4m3 bytes the kernel reads)."""
    return (Aq.double() @ Bqt.double().t()) * (sa.double().item() * sb.double().item())


# ----------------------------------------------------------------------------------------- BSR SpMM
def bsr_ref(crow, col, vals, B, M: int, K: int) -> torch.Tensor:
    """Reference torch path: torch.sparse.mm(A_bsr.float(), B.float())."""
    A = torch.sparse_bsr_tensor(crow.to(torch.int64), col.to(torch.int64), vals.float(), size=(M, K))
    return torch.sparse.mm(A, B.float())


def bsr_fp64(crow, col, vals, B, M: int, K: int, rows: slice | None = None) -> torch.Tensor:
    """fp64 restatement of C = A_bsr B, block-row by block-row (only nonzero blocks are touched):
    C[bm*br:(bm+1)*br] = sum_j vals[j] @ B[col[j]*bc:(col[j]+1)*bc]  (cpu_bsr semantics,
    BlackwellSparseK/src/bsr_reference.cu:72-93, in fp64 instead of fp32)."""
    nnzb, br, bc = vals.shape
    Mb = crow.numel() - 1
    N = B.shape[1]
    crow_l = crow.tolist()
    col_l = col.tolist()
    Bd = B.double()
    r0, r1 = (0, Mb) if rows is None else (rows.start, rows.stop)
    C = torch.zeros((r1 - r0) * br, N, dtype=torch.float64)
    for bm in range(r0, r1):
        acc = C[(bm - r0) * br:(bm - r0 + 1) * br]
        for j in range(crow_l[bm], crow_l[bm + 1]):
            kb = col_l[j]
            acc += vals[j].double() @ Bd[kb * bc:(kb + 1) * bc]
    return C


def cpu_bsr_numpy(A_blocks: np.ndarray, row_ptr, col_idx, B: np.ndarray, M: int, N: int, K: int,
                  BM: int, BN: int, BK: int) -> np.ndarray:
    """numpy restatement of cpu_bsr (BlackwellSparseK/src/bsr_reference.cu:72-93): fp16 blocks [nnz, BM, BK]
    and fp16 row-major B [K, N]; per output block, per nonzero: a full fp32 partial over that block's k,
    then added to C. Vectorised over i, j (summation order within a block differs from the scalar loop,
    so it agrees with the C restatement to fp32 rounding, not bit-for-bit)."""
    C = np.zeros((M, N), dtype=np.float32)
    Mb = (M + BM - 1) // BM
    for bm in range(Mb):
        i1 = min(BM, M - bm * BM)
        for idx in range(row_ptr[bm], row_ptr[bm + 1]):
            kb = col_idx[idx]
            k1 = min(BK, K - kb * BK)
            a = A_blocks[idx, :i1, :k1].astype(np.float32)
            b = B[kb * BK:kb * BK + k1, :].astype(np.float32)
            C[bm * BM:bm * BM + i1] += a @ b
    return C


# ----------------------------------------------------------------------------------------- attention
def attn_sdpa_ref(q, k, v, dense_mask: torch.Tensor, scale: float) -> torch.Tensor:
    """Reference torch path: scaled_dot_product_attention with a dense boolean mask (True = attend)."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=dense_mask, scale=scale)


def attn_blocksparse_fp64(q, k, v, row_ptr, col_idx, scale: float, causal_diag: bool, block: int = 128,
                          pair_rows=None) -> torch.Tensor:
    """fp64 block-sparse attention for ONE (b,h) pair: q, k, v [S, D]; row_ptr/col_idx the pair's block
    rows (row_ptr rebased so row_ptr[0] is this pair's first entry). Gathers only the nonzero key blocks
    of each query block-row and applies an exact two-pass softmax. Empty rows give zeros.
    ``pair_rows`` restricts the computation to a subset of query block-rows (list of ints)."""
    return attn_blocksparse(q, k, v, row_ptr, col_idx, scale, causal_diag, block, pair_rows, torch.float64)


def attn_blocksparse(q, k, v, row_ptr, col_idx, scale: float, causal_diag: bool, block: int = 128,
                     pair_rows=None, dtype=torch.float32) -> torch.Tensor:
    """Block-sparse attention of one (b,h) pair in `dtype` (the fp64 oracle above, or the fp32 CPU restatement
    of the reference's masked-SDPA path that the benchmark times as its CPU baseline: the same result as
    F.scaled_dot_product_attention with the dense block mask, computed over the nonzero key blocks only)."""
    S, D = q.shape
    nqb = S // block
    qd, kd, vd = q.to(dtype), k.to(dtype), v.to(dtype)
    out = torch.zeros(S, D, dtype=dtype)
    rp = row_ptr.tolist()
    ci = col_idx.tolist()
    base = rp[0]
    rows = range(nqb) if pair_rows is None else pair_rows
    for i in rows:
        cols = ci[rp[i] - base:rp[i + 1] - base]
        if not cols:
            continue
        keys = torch.cat([kd[c * block:(c + 1) * block] for c in cols])
        vals = torch.cat([vd[c * block:(c + 1) * block] for c in cols])
        s = (qd[i * block:(i + 1) * block] @ keys.t()) * scale
        if causal_diag:  # only the diagonal block (key block == query block) is masked elementwise
            kpos = torch.cat([torch.arange(c * block, (c + 1) * block) for c in cols])
            diag = torch.cat([torch.full((block,), c == i) for c in cols])
            qpos = torch.arange(i * block, (i + 1) * block)
            s = s.masked_fill(diag[None, :] & (kpos[None, :] > qpos[:, None]), -math.inf)
        p = torch.softmax(s, dim=1)
        out[i * block:(i + 1) * block] = p @ vals
    return out
