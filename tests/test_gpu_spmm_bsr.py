"""BSR x dense SpMM through the C ABI vs the reference's torch path (torch.sparse.mm on fp32 BSR) and the
fp64 block restatement. Tolerance: normwise relative error <= 1e-3; index handling exact. Every case runs on both
kernels: the one-CTA 128 x 256 tile and the CTA-pair 128 x 512 transposed tile (BSK_SPMM_TILE)."""
import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(autouse=True, params=["single", "pair"])
def tile(request, monkeypatch):
    monkeypatch.setenv("BSK_SPMM_TILE", request.param)
    return request.param


def _case(Mb, Kb, N, per_row, seed, empty_rows=()):
    g = torch.Generator().manual_seed(seed)
    crow, col = wl.bsr_pattern(Mb, Kb, per_row, g)
    if empty_rows:  # drop the nonzeros of some block-rows
        keep_rows = [r for r in range(Mb) if r not in empty_rows]
        cols, counts = [], []
        for r in range(Mb):
            seg = col[crow[r]:crow[r + 1]]
            cols.append(seg if r in keep_rows else seg[:0])
            counts.append(len(cols[-1]))
        col = torch.cat(cols)
        crow = torch.zeros(Mb + 1, dtype=torch.int64)
        crow[1:] = torch.cumsum(torch.tensor(counts), 0)
    vals = torch.randn(col.numel(), 128, 128, generator=g).half()
    B = torch.randn(Kb * 128, N, generator=g).half()
    return crow, col, vals, B


def _run(crow, col, vals, B, M, row_begin=0, row_end=None, C=None):
    dev = torch.device("cuda", 0)
    if C is None:
        C = torch.full((M, B.shape[1]), float("nan"), device=dev)
    _capi.spmm_bsr_f16f32(crow.to(torch.int32).to(dev), col.to(torch.int32).to(dev), vals.to(dev), B.to(dev), C, M,
                          row_begin, row_end)
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("Mb,Kb,N,per_row", [(2, 2, 256, 1), (4, 8, 512, 3), (3, 5, 200, 5), (8, 8, 1024, 8),
                                             (16, 16, 520, 4), (5, 12, 1544, 6), (3, 4, 24, 2)])
def test_bsr_shapes(no_device_error, Mb, Kb, N, per_row):
    crow, col, vals, B = _case(Mb, Kb, N, per_row, Mb * 100 + N)
    M, K = Mb * 128, Kb * 128
    C = _run(crow, col, vals, B, M).cpu()
    assert torch.isfinite(C).all()
    err = ref.normwise_rel_err(C, ref.bsr_fp64(crow, col, vals, B, M, K))
    assert err <= TOL, err
    ok, m = ref.validate_correctness(C, ref.bsr_ref(crow, col, vals, B, M, K), rtol=1e-3, atol=1e-2)
    assert ok, m


def test_bsr_empty_rows_are_zero(no_device_error):
    crow, col, vals, B = _case(6, 6, 256, 2, 11, empty_rows=(1, 4))
    C = _run(crow, col, vals, B, 6 * 128).cpu()
    assert torch.count_nonzero(C[128:256]) == 0 and torch.count_nonzero(C[512:640]) == 0
    err = ref.normwise_rel_err(C, ref.bsr_fp64(crow, col, vals, B, 768, 768))
    assert err <= TOL, err


def test_bsr_row_range_shards(no_device_error):
    crow, col, vals, B = _case(8, 8, 512, 3, 21)
    M = 8 * 128
    dev = torch.device("cuda", 0)
    C = torch.full((M, 512), 7.0, device=dev)
    _run(crow, col, vals, B, M, 2, 5, C=C)
    C = C.cpu()
    assert torch.all(C[:256] == 7.0) and torch.all(C[640:] == 7.0)  # rows outside the range untouched
    full = ref.bsr_fp64(crow, col, vals, B, M, M)
    err = ref.normwise_rel_err(C[256:640], full[256:640])
    assert err <= TOL, err


def test_bsr_unsorted_columns(no_device_error):
    crow, col, vals, B = _case(4, 8, 256, 4, 5)
    perm = torch.cat([torch.randperm(4, generator=torch.Generator().manual_seed(r)) + 4 * r for r in range(4)])
    col2, vals2 = col[perm], vals[perm]
    C = _run(crow, col2, vals2, B, 512).cpu()
    err = ref.normwise_rel_err(C, ref.bsr_fp64(crow, col, vals, B, 512, 1024))
    assert err <= TOL, err


def test_bsr_bad_index_flagged_not_faulted(cuda_dev):
    crow, col, vals, B = _case(2, 2, 256, 1, 1)
    col = col.clone()
    col[0] = 1 << 20  # out of range: the kernel flags it and reads zero fill instead of faulting
    _capi.device_error()
    _run(crow, col, vals, B, 256)
    word = _capi.device_error()
    assert (word & 0xFF) == 2, hex(word)


def test_bsr_rejects_block_shape(cuda_dev):
    vals = torch.zeros(1, 64, 64, dtype=torch.float16, device=cuda_dev)
    rp = torch.tensor([0, 1], dtype=torch.int32, device=cuda_dev)
    ci = torch.tensor([0], dtype=torch.int32, device=cuda_dev)
    B = torch.zeros(64, 64, dtype=torch.float16, device=cuda_dev)
    C = torch.zeros(64, 64, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.spmm_bsr_f16f32(rp, ci, vals, B, C, 64)
    assert e.value.code == _capi.BSK_ERR_UNSUPPORTED
