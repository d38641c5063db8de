"""Parity at the benchmark sizes: every operator run once on its full benchmark workload, through the C ABI, on
the same code paths the benchmark times (tile kind, rasterisation group, split policy), then checked two ways:

  * sampled fp64 recompute: rows and columns (or block-rows, or query block-rows of (b,h) pairs) chosen so that
    every output tile of the launch holds at least one checked element, against the fp64 oracle;
  * size-independent checksums over the WHOLE output, in fp64 on the device: C 1 = A (B 1) and 1^T C = (1^T A) B
    for the linear operators (a wrong, missing or misplaced tile anywhere moves a row or column sum).

Tolerances are the operator family's: normwise relative error <= 1e-3 against fp64 for fp16 inputs, <= 3e-2 for
e4m3, and for bf16 attention output the bf16 storage floor of the checked rows + 1e-3.

Workloads (seeded, as the benchmark generates them):
  dense   M = N = 8192, K = 237568, fp16 N(0,1)/K^(1/4), seed 1; plus 4096 x 1024 x 65536 (long-K raster)
  fp8     8192 x 8192 x 16384 e4m3 with per-tensor amax scales, bf16 out, seed 2
  bsr     8192^3, 128 x 128 blocks, 16 of 64 per block-row, seed 3, on both tile kinds
  attn    B = 2, H = 32, S = 16384, D = 128 bf16, window 4 + 8 random blocks per row, seed 4
"""
import math

import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 1e-3
TOL_FP8 = 3e-2


def _tile_sample(extent: int, tile: int, per_tile: int, g: torch.Generator) -> torch.Tensor:
    """`per_tile` distinct random indices inside every `tile`-wide slice of [0, extent), sorted."""
    out = []
    for t0 in range(0, extent, tile):
        w = min(tile, extent - t0)
        out.append(t0 + torch.randperm(w, generator=g)[:min(per_tile, w)])
    return torch.sort(torch.cat(out)).values


def _rowsum_fp64(X: torch.Tensor, v: torch.Tensor, chunk: int = 256) -> torch.Tensor:
    """X (fp16 / e4m3, [R, K], device) @ v (fp64 [K]) in fp64, in row chunks (bounded fp64 temporaries)."""
    out = torch.empty(X.shape[0], dtype=torch.float64, device=X.device)
    for r0 in range(0, X.shape[0], chunk):
        out[r0:r0 + chunk] = X[r0:r0 + chunk].double() @ v
    return out


def _colsum_fp64(X: torch.Tensor, chunk: int = 256) -> torch.Tensor:
    """1^T X in fp64 ([K]) for X [R, K] on the device."""
    out = torch.zeros(X.shape[1], dtype=torch.float64, device=X.device)
    for r0 in range(0, X.shape[0], chunk):
        out += X[r0:r0 + chunk].double().sum(0)
    return out


def _dense_checksums(A, Bt, C, scale: float = 1.0):
    """(row-sum error, column-sum error) of C = scale * A B (B given as Bt = B^T) over the whole output."""
    v = _colsum_fp64(Bt)                       # B 1 (sum over the N columns of B)
    row_ref = _rowsum_fp64(A, v) * scale       # A (B 1)
    u = _colsum_fp64(A)                        # 1^T A
    col_ref = _rowsum_fp64(Bt, u) * scale      # (1^T A) B, as Bt u
    Cd = C.double()
    return (ref.normwise_rel_err(Cd.sum(1), row_ref), ref.normwise_rel_err(Cd.sum(0), col_ref))


@pytest.fixture
def big_mem(cuda_dev):
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- dense fp16 -> fp32
def test_dense_headline_8192x8192x237568(no_device_error, big_mem, monkeypatch):
    """The headline shape on its default launch: CTA-pair 256 x 512 tiles, all 32 M tiles per raster group
    (K >= 65536), 3712 K blocks accumulated in TMEM per output tile."""
    monkeypatch.delenv("BSK_GEMM_TILE", raising=False)
    dev = torch.device("cuda", 0)
    cfg = wl.DENSE_BIG
    A, Bt = wl.dense_inputs(cfg, dev)
    C = torch.full((cfg.M, cfg.N), float("nan"), device=dev)
    _capi.gemm_f16f32(A, Bt, C)
    torch.cuda.synchronize()
    assert torch.isfinite(C).all()
    g = torch.Generator().manual_seed(11)
    rows = _tile_sample(cfg.M, 256, 2, g)      # every 256-row tile
    cols = _tile_sample(cfg.N, 512, 4, g)      # every 512-column tile
    c64 = ref.dense_fp64_sampled(A[rows.to(dev)].cpu(), Bt[cols.to(dev)].cpu(), slice(None), slice(None))
    err = ref.normwise_rel_err(C[rows.to(dev)][:, cols.to(dev)].cpu(), c64)
    assert err <= TOL, err
    e_row, e_col = _dense_checksums(A, Bt, C)
    assert e_row <= TOL and e_col <= TOL, (e_row, e_col)


def test_dense_long_k_wide_tile_4096x1024x65536(no_device_error, big_mem, monkeypatch):
    """A plain (no split-K) wide-tile GEMM at K = 65536, where the long-K raster group applies, checked on 4 rows
    of every M tile against all 1024 columns."""
    monkeypatch.delenv("BSK_GEMM_TILE", raising=False)
    dev = torch.device("cuda", 0)
    cfg = wl.DenseCfg(4096, 1024, 65536, 21, "scaled_normal")
    A, Bt = wl.dense_inputs(cfg, dev)
    C = torch.full((cfg.M, cfg.N), float("nan"), device=dev)
    _capi.gemm_f16f32(A, Bt, C)
    torch.cuda.synchronize()
    rows = _tile_sample(cfg.M, 256, 4, torch.Generator().manual_seed(12))
    c64 = ref.dense_fp64(A[rows.to(dev)].cpu(), Bt.cpu())
    err = ref.normwise_rel_err(C[rows.to(dev)].cpu(), c64)
    assert err <= TOL, err
    e_row, e_col = _dense_checksums(A, Bt, C)
    assert e_row <= TOL and e_col <= TOL, (e_row, e_col)


# ----------------------------------------------------------------------------------------- FP8 e4m3 -> bf16
def test_fp8_8192x8192x16384(no_device_error, big_mem):
    dev = torch.device("cuda", 0)
    cfg = wl.FP8
    Aq, Bqt, sa, sb = wl.fp8_inputs(cfg, dev)
    D = torch.full((cfg.M, cfg.N), float("nan"), dtype=torch.bfloat16, device=dev)
    _capi.gemm_e4m3_bf16(Aq, Bqt, sa, sb, D)
    torch.cuda.synchronize()
    assert torch.isfinite(D).all()
    g = torch.Generator().manual_seed(13)
    rows = _tile_sample(cfg.M, 256, 2, g).to(dev)
    cols = _tile_sample(cfg.N, 512, 4, g).to(dev)
    d64 = ref.fp8_fp64(Aq[rows].cpu(), Bqt[cols].cpu(), sa.cpu(), sb.cpu())
    err = ref.normwise_rel_err(D[rows][:, cols].cpu(), d64)
    assert err <= TOL_FP8, err
    # the reference path's own call (torch._scaled_mm, here on the device) over the whole output
    d_ref = torch._scaled_mm(Aq, Bqt.t(), scale_a=sa.reshape(()), scale_b=sb.reshape(()), out_dtype=torch.bfloat16)
    err_full = ref.normwise_rel_err(D.float(), d_ref.float())
    assert err_full <= TOL_FP8, err_full
    s = float(sa.item()) * float(sb.item())
    e_row, e_col = _dense_checksums(Aq, Bqt, D, s)
    assert e_row <= TOL_FP8 and e_col <= TOL_FP8, (e_row, e_col)


# ----------------------------------------------------------------------------------------- BSR SpMM
@pytest.mark.parametrize("tile", ["pair", "single"])
def test_bsr_8192cube_16_per_row(no_device_error, big_mem, monkeypatch, tile):
    """The BSR workload on both tile kinds (the CTA pair is the default at N = 8192): 4 whole block-rows against
    the fp64 restatement, and the row / column checksums of the whole output."""
    monkeypatch.setenv("BSK_SPMM_TILE", tile)
    dev = torch.device("cuda", 0)
    cfg = wl.BSR
    crow, col, vals, B = wl.bsr_inputs(cfg, dev)
    C = torch.full((cfg.M, cfg.N), float("nan"), device=dev)
    _capi.spmm_bsr_f16f32(crow.to(torch.int32), col.to(torch.int32), vals, B, C, cfg.M)
    torch.cuda.synchronize()
    assert torch.isfinite(C).all()
    crow_h, col_h, vals_h, B_h = crow.cpu(), col.cpu(), vals.cpu(), B.cpu()
    Mb = cfg.M // cfg.block
    for r in (0, 21, 42, Mb - 1):
        c64 = ref.bsr_fp64(crow_h, col_h, vals_h, B_h, cfg.M, cfg.K, rows=slice(r, r + 1))
        err = ref.normwise_rel_err(C[r * 128:(r + 1) * 128].cpu(), c64)
        assert err <= TOL, (r, err)
    # C 1 = A (B 1): per stored block, its rows dotted with the matching slice of B 1
    w = _rowsum_fp64(B, torch.ones(cfg.N, dtype=torch.float64, device=dev))       # B 1, [K]
    blk_rows = torch.repeat_interleave(torch.arange(Mb, device=dev), (crow[1:] - crow[:-1]))
    wb = w.view(-1, 128)[col]                                                       # [nnzb, 128]
    part = torch.bmm(vals.double(), wb.unsqueeze(2)).squeeze(2)                     # [nnzb, 128]
    row_ref = torch.zeros(Mb, 128, dtype=torch.float64, device=dev).index_add_(0, blk_rows, part).reshape(-1)
    # 1^T C = (1^T A) B
    u = torch.zeros(cfg.K // 128, 128, dtype=torch.float64, device=dev).index_add_(0, col, vals.double().sum(1))
    col_ref = _bsr_colsum(u.reshape(-1), B)
    Cd = C.double()
    e_row = ref.normwise_rel_err(Cd.sum(1), row_ref)
    e_col = ref.normwise_rel_err(Cd.sum(0), col_ref)
    assert e_row <= TOL and e_col <= TOL, (e_row, e_col)


def _bsr_colsum(u: torch.Tensor, B: torch.Tensor, chunk: int = 1024) -> torch.Tensor:
    """u^T B in fp64 for B [K, N] fp16 on the device, in K chunks."""
    out = torch.zeros(B.shape[1], dtype=torch.float64, device=B.device)
    for k0 in range(0, B.shape[0], chunk):
        out += u[k0:k0 + chunk] @ B[k0:k0 + chunk].double()
    return out


# ----------------------------------------------------------------------------------------- attention
def test_attention_2x32x16384x128(no_device_error, big_mem):
    """The attention workload (64 (b,h) pairs, 128 query block-rows each): 8 query block-rows of 3 pairs, and the
    first, last and one random block-row of every pair, against the fp64 block-sparse restatement."""
    dev = torch.device("cuda", 0)
    cfg = wl.ATTN
    q, k, v = wl.attn_inputs(cfg, dev)
    rp, ci = wl.attn_mask_bsr(cfg)
    O = torch.full_like(q, float("nan"))
    scale = 1.0 / math.sqrt(cfg.D)
    _capi.bsattn_fwd_bf16(q, k, v, O, rp.to(torch.int32).to(dev), ci.to(torch.int32).to(dev), scale, True)
    torch.cuda.synchronize()
    assert torch.isfinite(O.float()).all()
    nqb, P = cfg.S // cfg.block, cfg.B * cfg.H
    g = torch.Generator().manual_seed(14)
    plan = {}
    for p in (0, 31, P - 1):
        plan[p] = sorted(set([0, nqb - 1] + torch.randperm(nqb, generator=g)[:6].tolist()))
    for p in range(P):
        plan.setdefault(p, sorted({0, nqb - 1, int(torch.randint(nqb, (1,), generator=g))}))
    Oh = O.cpu()
    qh, kh, vh = q.cpu(), k.cpu(), v.cpu()
    for p, rows in plan.items():
        b, h = divmod(p, cfg.H)
        r0, r1 = p * nqb, (p + 1) * nqb
        o64 = ref.attn_blocksparse_fp64(qh[b, h], kh[b, h], vh[b, h], rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], scale, True,
                                        pair_rows=rows)
        sel = torch.cat([torch.arange(r * 128, (r + 1) * 128) for r in rows])
        floor = ref.bf16_storage_floor(o64[sel])
        err = ref.normwise_rel_err(Oh[b, h][sel], o64[sel])
        assert err <= floor + 1e-3, (p, rows, err, floor)
