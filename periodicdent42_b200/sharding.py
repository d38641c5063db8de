"""Multi-GPU partition plans for the four operators (one process per GPU).

Every plan is a pure function of the problem and (world, rank), so all ranks agree without communication:
  dense / FP8   N-shard: rank r owns output columns [n0, n1) (tile-aligned), reads all of A and B^T[n0:n1]
  dense         split-K: rank r owns K range [k0, k1) and produces a partial C reduced by reduce-scatter
  BSR           contiguous block-row ranges with balanced cumulative nnz; B replicated
  attention     contiguous (b,h) pair ranges with balanced nnz blocks
"""
from __future__ import annotations

import torch

from .workloads import even_ranges, shard_ranges

GEMM_N_ALIGN = 256  # output-tile width of the GEMM kernels
GEMM_K_ALIGN = 64   # K extent of one pipeline stage (fp16)


def dense_nshard(N: int, world: int, rank: int) -> tuple[int, int]:
    return even_ranges(N, world, align=GEMM_N_ALIGN)[rank]


def dense_ksplit(K: int, world: int, rank: int) -> tuple[int, int]:
    return even_ranges(K, world, align=GEMM_K_ALIGN)[rank]


def splitk_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """Rows of C a rank owns after the reduce-scatter (M must divide evenly)."""
    if M % world:
        raise ValueError(f"split-K reduce-scatter needs M ({M}) divisible by the world size ({world})")
    return rank * M // world, (rank + 1) * M // world


def bsr_block_rows(crow: torch.Tensor, world: int, rank: int) -> tuple[int, int]:
    counts = (crow[1:] - crow[:-1]).tolist()
    return shard_ranges(counts, world)[rank]


def attn_pairs(row_ptr: torch.Tensor, nqb: int, n_pairs: int, world: int, rank: int) -> tuple[int, int]:
    rp = row_ptr.tolist()
    nnz = [rp[(p + 1) * nqb] - rp[p * nqb] for p in range(n_pairs)]
    return shard_ranges(nnz, world)[rank]
