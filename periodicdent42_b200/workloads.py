"""Seeded synthetic workloads for the four operators, and the block-mask / BSR index builders.

The five workloads are the operator family's benchmark configurations:

  dense_small   fp16 GEMM 1024^3, entries uniform[-1, 1), seed 0 (CPU-checkable parity case)
  dense_big     fp16 -> fp32 GEMM M=N=8192, K=237568, entries N(0,1) / K^(1/4) in fp16, seed 1
  fp8           e4m3 GEMM M=N=8192, K=16384: fp32 N(0,1) quantised with per-tensor amax/448 scales, seed 2
  bsr           BSR SpMM M=N=K=8192, 128x128 blocks, exactly 16 nonzero blocks per block-row (25 %),
                columns uniform without replacement, sorted; block values and dense B N(0,1) fp16, seed 3
  attn          block-sparse attention B=2, H=32, S=16384, D=128 bf16, Q/K/V N(0,1); per (b,h) mask over
                128x128 blocks: query block-row i keeps the causal window {i-3..i} (clipped at 0) plus
                min(8, i-3) distinct random blocks from [0, i-4]; diagonal block elementwise-causal; seed 4

Matrix B of the dense GEMMs is column-major [K, N]; it is held as ``Bt`` = B^T, row-major [N, K].
The generators draw on a torch.Generator of the target device, so device inputs come from the device
generator and host (CPU) inputs from the CPU one; each is reproducible on its own device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

E4M3_MAX = 448.0


@dataclass(frozen=True)
class DenseCfg:
    M: int
    N: int
    K: int
    seed: int
    dist: str  # "uniform" | "scaled_normal"

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K


@dataclass(frozen=True)
class Fp8Cfg:
    M: int
    N: int
    K: int
    seed: int

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K


@dataclass(frozen=True)
class BsrCfg:
    M: int
    N: int
    K: int
    block: int
    nnz_per_row: int
    seed: int

    @property
    def nnzb(self) -> int:
        return (self.M // self.block) * self.nnz_per_row

    @property
    def flops(self) -> float:  # nonzero-block FLOPs
        return 2.0 * self.nnzb * self.block * self.block * self.N


@dataclass(frozen=True)
class AttnCfg:
    B: int
    H: int
    S: int
    D: int
    block: int
    window: int
    n_random: int
    seed: int


DENSE_SMALL = DenseCfg(1024, 1024, 1024, 0, "uniform")
DENSE_BIG = DenseCfg(8192, 8192, 237568, 1, "scaled_normal")
FP8 = Fp8Cfg(8192, 8192, 16384, 2)
BSR = BsrCfg(8192, 8192, 8192, 128, 16, 3)
ATTN = AttnCfg(2, 32, 16384, 128, 128, 4, 8, 4)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


# ----------------------------------------------------------------------------------------- dense fp16
def dense_inputs(cfg: DenseCfg, device="cpu", k_slice: int | None = None):
    """A [M, K] fp16 row-major and Bt [N, K] fp16 (column-major B). ``k_slice`` draws only the first
    k_slice columns of K (a bounded sample with the same distribution)."""
    K = cfg.K if k_slice is None else k_slice
    g = _gen(device, cfg.seed)
    if cfg.dist == "uniform":
        A = (torch.rand(cfg.M, K, generator=g, device=device) * 2 - 1).to(torch.float16)
        Bt = (torch.rand(cfg.N, K, generator=g, device=device) * 2 - 1).to(torch.float16)
    else:
        s = cfg.K ** -0.25
        A = torch.empty(cfg.M, K, dtype=torch.float16, device=device)
        Bt = torch.empty(cfg.N, K, dtype=torch.float16, device=device)
        _fill_normal_fp16(A, g, s)
        _fill_normal_fp16(Bt, g, s)
    return A, Bt


def _fill_normal_fp16(t: torch.Tensor, g: torch.Generator, scale: float, chunk_rows: int = 256) -> None:
    """N(0, scale^2) in fp16, drawn in row chunks to bound the fp32 temporary."""
    for r0 in range(0, t.shape[0], chunk_rows):
        r1 = min(r0 + chunk_rows, t.shape[0])
        tmp = torch.randn(r1 - r0, t.shape[1], generator=g, device=t.device)
        tmp.mul_(scale)
        t[r0:r1].copy_(tmp)


# ----------------------------------------------------------------------------------------- fp8
def quantize_e4m3(x: torch.Tensor):
    """Per-tensor amax quantisation: scale = amax / 448, x_q = e4m3(x / scale). Returns (x_q, scale fp32 [1])."""
    amax = x.abs().amax().float()
    scale = (amax / E4M3_MAX).clamp(min=1e-12).reshape(1)
    xq = (x / scale).to(torch.float8_e4m3fn)
    return xq, scale


def fp8_inputs(cfg: Fp8Cfg, device="cpu"):
    """(Aq [M,K] e4m3, Bqt [N,K] e4m3, scale_a [1] fp32, scale_b [1] fp32)."""
    g = _gen(device, cfg.seed)
    A = torch.randn(cfg.M, cfg.K, generator=g, device=device)
    Aq, sa = quantize_e4m3(A)
    del A
    Bt = torch.randn(cfg.N, cfg.K, generator=g, device=device)
    Bqt, sb = quantize_e4m3(Bt)
    return Aq, Bqt, sa, sb


# ----------------------------------------------------------------------------------------- BSR
def bsr_pattern(n_block_rows: int, n_block_cols: int, nnz_per_row: int, g: torch.Generator):
    """Fixed-nnz-per-row block pattern: for each block-row, nnz_per_row distinct columns drawn uniformly
    without replacement (first entries of a random permutation), sorted. Returns int64 (crow, col)."""
    cols = []
    for _ in range(n_block_rows):
        perm = torch.randperm(n_block_cols, generator=g)[:nnz_per_row]
        cols.append(torch.sort(perm).values)
    col = torch.cat(cols) if cols else torch.zeros(0, dtype=torch.int64)
    crow = torch.arange(0, n_block_rows + 1, dtype=torch.int64) * nnz_per_row
    return crow, col


def bsr_inputs(cfg: BsrCfg, device="cpu"):
    """(crow int64 [Mb+1], col int64 [nnzb], vals fp16 [nnzb, bs, bs], B fp16 [K, N]); the index pattern is
    drawn on a CPU generator (same on every device), values and B on the device generator."""
    Mb, Kb = cfg.M // cfg.block, cfg.K // cfg.block
    crow, col = bsr_pattern(Mb, Kb, cfg.nnz_per_row, _gen("cpu", cfg.seed))
    g = _gen(device, cfg.seed)
    vals = torch.randn(crow[-1].item(), cfg.block, cfg.block, generator=g, device=device).to(torch.float16)
    B = torch.empty(cfg.K, cfg.N, dtype=torch.float16, device=device)
    _fill_normal_fp16(B, g, 1.0)
    return crow.to(device), col.to(device), vals, B


def bsr_tensor(crow, col, vals, M: int, K: int) -> torch.Tensor:
    return torch.sparse_bsr_tensor(crow, col, vals, size=(M, K))


# ----------------------------------------------------------------------------------------- attention mask
def attn_block_rows(n_qb: int, window: int, n_random: int, g: torch.Generator) -> list[torch.Tensor]:
    """Key-block lists of one (b,h): row i = {max(0,i-window+1) .. i} plus min(n_random, i-window+1)
    distinct random blocks from [0, i-window], sorted ascending."""
    rows = []
    for i in range(n_qb):
        lo = max(0, i - window + 1)
        win = torch.arange(lo, i + 1, dtype=torch.int64)
        n_pool = max(0, i - window + 1)  # candidates [0, i-window]
        k = min(n_random, n_pool)
        if k > 0:
            rnd = torch.randperm(n_pool, generator=g)[:k]
            rows.append(torch.sort(torch.cat([rnd, win])).values)
        else:
            rows.append(win)
    return rows


def attn_mask_bsr(cfg: AttnCfg, n_pairs: int | None = None):
    """BSR index of the per-(b,h) block masks, pairs in (b, h) order, on the CPU generator seeded cfg.seed.
    Returns (row_ptr int64 [P*nqb + 1], col_idx int64 [nnz]) with within-sequence block indices."""
    nqb = cfg.S // cfg.block
    P = cfg.B * cfg.H if n_pairs is None else n_pairs
    g = _gen("cpu", cfg.seed)
    counts, cols = [], []
    for _ in range(P):
        for r in attn_block_rows(nqb, cfg.window, cfg.n_random, g):
            counts.append(r.numel())
            cols.append(r)
    row_ptr = torch.zeros(len(counts) + 1, dtype=torch.int64)
    row_ptr[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0)
    return row_ptr, torch.cat(cols)


def attn_inputs(cfg: AttnCfg, device="cpu", dtype=torch.bfloat16):
    g = _gen(device, cfg.seed)
    shape = (cfg.B, cfg.H, cfg.S, cfg.D)
    out = []
    for _ in range(3):
        t = torch.empty(shape, dtype=dtype, device=device)
        flat = t.view(-1, cfg.D)
        for r0 in range(0, flat.shape[0], 1 << 16):
            r1 = min(r0 + (1 << 16), flat.shape[0])
            flat[r0:r1].copy_(torch.randn(r1 - r0, cfg.D, generator=g, device=device))
        out.append(t)
    return tuple(out)


def attn_flops(row_ptr: torch.Tensor, block: int, D: int) -> float:
    """Nonzero-block FLOPs: QK^T and PV over every nonzero block, full block counted (4 * blk^2 * D)."""
    nnz = int(row_ptr[-1].item())
    return 4.0 * nnz * block * block * D


def block_mask_dense(row_ptr: torch.Tensor, col_idx: torch.Tensor, n_rows: int, n_cols: int) -> torch.Tensor:
    """Boolean [n_rows, n_cols] block mask of one BSR row range (row_ptr rebased to start at 0)."""
    m = torch.zeros(n_rows, n_cols, dtype=torch.bool)
    rp = row_ptr.tolist()
    ci = col_idx.tolist()
    for i in range(n_rows):
        for j in ci[rp[i] - rp[0]:rp[i + 1] - rp[0]]:
            m[i, j] = True
    return m


def mask_to_bsr(mask: torch.Tensor):
    """Boolean block mask [nr, nc] -> (crow int64, col int64), row-major order, columns ascending.
    Same index layout as torch's ``to_sparse_bsr`` on the expanded mask."""
    nr = mask.shape[0]
    counts = mask.sum(dim=1)
    crow = torch.zeros(nr + 1, dtype=torch.int64)
    crow[1:] = torch.cumsum(counts, 0)
    col = mask.nonzero(as_tuple=False)[:, 1].to(torch.int64)
    return crow, col


def dense_mask_from_blocks(block_mask: torch.Tensor, block: int, causal_diag: bool) -> torch.Tensor:
    """Elementwise boolean mask [S, S] (True = attend) from a [nqb, nkb] block mask."""
    m = block_mask.repeat_interleave(block, 0).repeat_interleave(block, 1)
    if causal_diag:
        S = m.shape[0]
        idx = torch.arange(S)
        qb = idx // block
        same = qb[:, None] == qb[None, :]
        m &= ~(same & (idx[None, :] > idx[:, None]))
    return m


def shard_ranges(weights: list[int], n: int) -> list[tuple[int, int]]:
    """Contiguous partition of len(weights) units into n ranges with balanced cumulative weight
    (greedy on prefix sums; every unit lands in exactly one range)."""
    total = sum(weights)
    L = len(weights)
    bounds = [0]
    acc = 0
    i = 0
    for r in range(1, n):
        target = total * r / n
        while i < L and acc + weights[i] / 2 <= target:
            acc += weights[i]
            i += 1
        bounds.append(max(i, bounds[-1]))
    bounds.append(L)
    return [(bounds[r], bounds[r + 1]) for r in range(n)]


def even_ranges(L: int, n: int, align: int = 1) -> list[tuple[int, int]]:
    """Split [0, L) into n contiguous ranges of near-equal size, boundaries multiples of `align`."""
    units = math.ceil(L / align)
    out = []
    for r in range(n):
        a = (units * r // n) * align
        b = min(L, (units * (r + 1) // n) * align)
        out.append((min(a, L), b))
    return out
