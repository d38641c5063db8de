"""Device dense -> BSR and CSR -> BSR conversion through the C ABI, bit-exact against the reference's
convert_to_bsr path (torch's to_sparse_bsr; the golden fixtures hold its outputs) and against torch on the CPU
for the edge cases: block sizes 128 / 16 / 2, fp16 / bf16 / fp32, -0.0 (zero) and NaN (nonzero), empty and
all-zero matrices, strided rows, int32 / int64 indices, explicit zeros in CSR, out-of-range column indices."""
import os

import numpy as np
import pytest
import torch

from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _assert_same(got, want_bsr):
    rp, ci, vals = (x.cpu() for x in got[:3])
    assert torch.equal(rp.long(), want_bsr.crow_indices()), (rp, want_bsr.crow_indices())
    assert torch.equal(ci.long(), want_bsr.col_indices())
    assert vals.shape == want_bsr.values().shape
    assert torch.equal(_bits(vals), _bits(want_bsr.values()))


def _sparse_dense(M, K, bs, dtype, seed, block_density=0.3, elem_density=0.5):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    keep_blocks = torch.rand(M // bs, K // bs, generator=g) < block_density
    x = x * keep_blocks.repeat_interleave(bs, 0).repeat_interleave(bs, 1)
    x = x * (torch.rand(M, K, generator=g) < elem_density)
    return x.to(dtype)


def test_dense_golden_matches_reference_convert(no_device_error, cuda_dev):
    z = np.load(GOLDEN)
    crow, col, vals = (torch.from_numpy(z[k]) for k in ("bsr_ref_crow", "bsr_ref_col", "bsr_ref_vals"))
    dense = torch.sparse_bsr_tensor(crow, col, vals, size=(512, 768)).to_dense()
    rp, ci, v, _ = _capi.dense_to_bsr(dense.to(cuda_dev), 128)
    assert torch.equal(rp.cpu(), crow) and torch.equal(ci.cpu(), col)
    assert torch.equal(_bits(v.cpu()), _bits(vals))


def test_dense_golden_masks(no_device_error, cuda_dev):
    z = np.load(GOLDEN)
    cfg = wl.AttnCfg(1, 2, 2048, 128, 128, 4, 8, 4)
    rp_m, ci_m = wl.attn_mask_bsr(cfg)
    off = 0
    for p in range(2):
        bm = wl.block_mask_dense(rp_m[p * 16:(p + 1) * 16 + 1], ci_m[rp_m[p * 16]:rp_m[(p + 1) * 16]], 16, 16)
        expanded = bm.repeat_interleave(128, 0).repeat_interleave(128, 1).to(torch.float16)
        rp, ci, _, nnz = _capi.dense_to_bsr(expanded.to(cuda_dev), 128)
        want_rp = torch.from_numpy(z["mask_ref_crow"][p])
        n = int(want_rp[-1])
        assert torch.equal(rp.cpu(), want_rp)
        assert torch.equal(ci.cpu(), torch.from_numpy(z["mask_ref_col"][off:off + n]))
        assert nnz == n * 128 * 128
        off += n


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,K,bs", [(512, 768, 128), (256, 320, 16), (48, 40, 8), (12, 10, 2), (130, 390, 13)])
def test_dense_matches_torch(no_device_error, cuda_dev, dtype, M, K, bs):
    x = _sparse_dense(M, K, bs, dtype, M + K + bs)
    got = _capi.dense_to_bsr(x.to(cuda_dev), bs, index_dtype=torch.int32)
    _assert_same(got, x.to_sparse_bsr((bs, bs)))
    assert got[3] == int(torch.count_nonzero(x))


def test_dense_negative_zero_and_nan(no_device_error, cuda_dev):
    x = torch.zeros(64, 64, dtype=torch.float16)
    x[0, 0] = -0.0        # block (0,0): only a negative zero -> not stored
    x[20, 40] = float("nan")  # block (1,2): NaN -> stored
    x[63, 17] = -0.0
    x[60, 18] = 1.0       # block (3,1): stored, keeps the -0.0 bits
    got = _capi.dense_to_bsr(x.to(cuda_dev), 16)
    _assert_same(got, x.to_sparse_bsr((16, 16)))


def test_dense_empty_and_all_zero(no_device_error, cuda_dev):
    z = torch.zeros(256, 384, dtype=torch.float16, device=cuda_dev)
    rp, ci, v, nnz = _capi.dense_to_bsr(z, 128)
    assert rp.tolist() == [0, 0, 0] and ci.numel() == 0 and v.shape == (0, 128, 128) and nnz == 0
    e = torch.zeros(0, 256, dtype=torch.float16, device=cuda_dev)
    rp, ci, v, nnz = _capi.dense_to_bsr(e, 128)
    assert rp.tolist() == [0] and ci.numel() == 0


def test_dense_strided_rows(no_device_error, cuda_dev):
    big = _sparse_dense(256, 520, 8, torch.float16, 3)
    x = big[:, :512]  # row stride 520: vector path (520 % 8 == 0)
    got = _capi.dense_to_bsr(big.to(cuda_dev)[:, :512], 8)
    _assert_same(got, x.contiguous().to_sparse_bsr((8, 8)))
    big2 = _sparse_dense(64, 67, 1, torch.float16, 4)
    x2 = big2[:, :64]     # row stride 67: element path
    got = _capi.dense_to_bsr(big2.to(cuda_dev)[:, :64], 16)
    _assert_same(got, x2.contiguous().to_sparse_bsr((16, 16)))


def test_dense_bsr_workload_round_trip(no_device_error, cuda_dev):
    """The 8192 x 8192 BSR workload (16 of 64 blocks per block-row): device dense -> BSR reproduces the
    generator's pattern and values exactly."""
    crow, col, vals, _ = wl.bsr_inputs(wl.BSR, cuda_dev)
    A = torch.sparse_bsr_tensor(crow.long(), col.long(), vals, size=(wl.BSR.M, wl.BSR.K)).to_dense()
    rp, ci, v, nnz = _capi.dense_to_bsr(A, 128)
    assert torch.equal(rp.cpu(), crow.long().cpu()) and torch.equal(ci.cpu(), col.long().cpu())
    assert torch.equal(_bits(v), _bits(vals))
    assert nnz == int(torch.count_nonzero(A))


@pytest.mark.parametrize("idx", [torch.int32, torch.int64])
@pytest.mark.parametrize("dtype,bs", [(torch.float16, 128), (torch.float16, 16), (torch.float32, 4), (torch.bfloat16, 8)])
def test_csr_matches_to_dense_path(no_device_error, cuda_dev, idx, dtype, bs):
    M, K = 256, 512
    x = _sparse_dense(M, K, bs, dtype, 17 + bs, block_density=0.2, elem_density=0.1)
    csr = x.to_sparse_csr()
    crow, col, vals = csr.crow_indices().to(idx), csr.col_indices().to(idx), csr.values()
    got = _capi.csr_to_bsr(crow.to(cuda_dev), col.to(cuda_dev), vals.to(cuda_dev), (M, K), bs, index_dtype=idx)
    _assert_same(got, csr.to_dense().to_sparse_bsr((bs, bs)))
    assert got[0].dtype == idx


def _shifted(t: torch.Tensor, k: int) -> torch.Tensor:
    """A copy of t whose storage starts k elements into a larger buffer (a pointer off the vector alignment)."""
    buf = torch.zeros(t.numel() + k, dtype=t.dtype, device=t.device)
    buf[k:] = t
    return buf[k:]


# The CSR passes take a quad path (4 entries per vector load) when col is 16-byte aligned and vals 4-element
# aligned, with one 4-element store per quad when the values output is 4-element aligned and bs % 4 == 0; these
# cases cover both paths and the quad path's boundaries: entries outside [crow[0], crow[M]) at either end (partial
# quads, out-of-range junk that must be ignored), rows shorter than a quad (row changes inside a quad, empty rows),
# columns unsorted within rows, block sizes that are not powers of two or not multiples of 4, an unaligned output.
@pytest.mark.parametrize("idx", [torch.int32, torch.int64])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("case", ["aligned", "offset_inputs", "junk_ends", "short_rows", "unsorted", "bs6", "bs12",
                                  "offset_output"])
def test_csr_quad_and_scalar_paths(no_device_error, cuda_dev, idx, dtype, case):
    M, K, bs, ed = {"short_rows": (1024, 64, 8, 0.03), "bs6": (96, 120, 6, 0.5),
                    "bs12": (240, 96, 12, 0.5)}.get(case, (384, 256, 16, 0.4))
    x = _sparse_dense(M, K, bs, dtype, 101 + len(case), block_density=0.4, elem_density=ed)
    csr = x.to_sparse_csr()
    crow, col, vals = csr.crow_indices().to(idx), csr.col_indices().to(idx), csr.values()
    want = csr.to_dense().to_sparse_bsr((bs, bs))
    if case == "junk_ends":  # 3 entries before crow[0], 5 after crow[M]; their columns are out of range
        col = torch.cat([torch.tensor([-5, K + 7, 2], dtype=idx), col, torch.tensor([K, -1, 0, 1, K + 3], dtype=idx)])
        vals = torch.cat([torch.ones(3, dtype=dtype), vals, torch.ones(5, dtype=dtype)])
        crow = crow + 3
    elif case == "unsorted":
        for r in range(M):
            a, b = int(crow[r]), int(crow[r + 1])
            col[a:b] = col[a:b].flip(0).clone()
            vals[a:b] = vals[a:b].flip(0).clone()
    crow, col, vals = crow.to(cuda_dev), col.to(cuda_dev), vals.to(cuda_dev)
    if case == "offset_inputs":
        col, vals = _shifted(col, 1), _shifted(vals, 1)
    if case != "offset_output":
        got = _capi.csr_to_bsr(crow, col, vals, (M, K), bs, index_dtype=idx)
        _assert_same(got, want)
        assert got[3] == int(torch.count_nonzero(x))
        return
    nnzb = want.col_indices().numel()
    ws = torch.empty(_capi.bsr_convert_workspace_bytes(M, K, bs), dtype=torch.uint8, device=cuda_dev)
    rp = torch.empty(M // bs + 1, dtype=idx, device=cuda_dev)
    ci = torch.empty(nnzb, dtype=idx, device=cuda_dev)
    v = torch.empty(nnzb * bs * bs + 1, dtype=dtype, device=cuda_dev)[1:].view(nnzb, bs, bs)
    _capi.csr_to_bsr_bounded(crow, col, vals, (M, K), bs, rp, ci, v, ws)
    _assert_same((rp, ci, v), want)


def test_csr_explicit_zeros_drop_blocks(no_device_error, cuda_dev):
    crow = torch.tensor([0, 2, 3, 3, 3])
    col = torch.tensor([0, 3, 5])
    vals = torch.tensor([2.0, 0.0, -0.0], dtype=torch.float16)  # block (0,1) and (0,2) hold only zeros
    csr = torch.sparse_csr_tensor(crow, col, vals, (4, 6))
    got = _capi.csr_to_bsr(crow.to(cuda_dev), col.to(cuda_dev), vals.to(cuda_dev), (4, 6), 2)
    _assert_same(got, csr.to_dense().to_sparse_bsr((2, 2)))
    assert got[3] == 1


def test_csr_out_of_range_column_is_an_error(cuda_dev):
    crow = torch.tensor([0, 1, 2], dtype=torch.int32, device=cuda_dev)
    col = torch.tensor([1, 9], dtype=torch.int32, device=cuda_dev)
    vals = torch.ones(2, dtype=torch.float16, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.csr_to_bsr(crow, col, vals, (2, 4), 2)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
    assert _capi.device_error() == 0


def test_convert_rejects_bad_arguments(cuda_dev):
    x = torch.zeros(100, 128, dtype=torch.float16, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.dense_to_bsr(x, 128)  # 100 not divisible by 128
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
    with pytest.raises(_capi.BskError) as e:
        _capi.dense_to_bsr(torch.zeros(128, 128, dtype=torch.float64, device=cuda_dev), 128)
    assert e.value.code == _capi.BSK_ERR_UNSUPPORTED


def test_public_convert_to_bsr_on_cuda(no_device_error, cuda_dev, capsys):
    import periodicdent42_b200 as bsk

    x = _sparse_dense(512, 512, 16, torch.float16, 21, block_density=0.3, elem_density=0.5)
    want = x.to_sparse_bsr((16, 16))
    got = bsk.convert_to_bsr(x.to(cuda_dev), block_size=16)
    assert got.layout == torch.sparse_bsr and got.is_cuda
    assert torch.equal(got.crow_indices().cpu(), want.crow_indices())
    assert torch.equal(got.col_indices().cpu(), want.col_indices())
    assert torch.equal(_bits(got.values().cpu()), _bits(want.values()))
    assert "Warning" not in capsys.readouterr().out  # ~85 % sparse: no warning
    csr = x.to_sparse_csr()  # drops the -0.0 entries the masking left, so compare with its own dense form
    want_csr = csr.to_dense().to_sparse_bsr((16, 16))
    got_csr = bsk.convert_to_bsr(csr.to(cuda_dev), block_size=16)
    assert torch.equal(got_csr.col_indices().cpu(), want_csr.col_indices())
    assert torch.equal(_bits(got_csr.values().cpu()), _bits(want_csr.values()))
    dense = torch.randn(256, 256).half().to(cuda_dev)
    bsk.convert_to_bsr(dense, block_size=128)
    assert "Warning: Matrix is only" in capsys.readouterr().out


def test_sparse_mm_with_csr_input(no_device_error, cuda_dev):
    import periodicdent42_b200 as bsk
    from oracle import reference_path as ref

    x = _sparse_dense(512, 768, 128, torch.float16, 8, block_density=0.4, elem_density=0.3)
    B = torch.randn(768, 256).half()
    C = bsk.sparse_mm(x.to_sparse_csr().to(cuda_dev), B.to(cuda_dev))
    err = ref.normwise_rel_err(C.cpu(), x.double() @ B.double())
    assert err <= 1e-3, err


@pytest.mark.parametrize("kind", ["dense", "csr"])
# 32 x 48 blocks: the one-CTA index pass; 1024 x 1024 blocks (more than 2^18): the three-launch index pass
@pytest.mark.parametrize("M,K,bs", [(512, 768, 16), (4096, 4096, 4)])
@pytest.mark.parametrize("idx", [torch.int64, torch.int32])
def test_bounded_single_call_matches_two_phase(no_device_error, cuda_dev, kind, M, K, bs, idx):
    x = _sparse_dense(M, K, bs, torch.float16, 31, block_density=0.3, elem_density=0.4)
    csr = x.to_sparse_csr()
    want = (csr.to_dense() if kind == "csr" else x).to_sparse_bsr((bs, bs))
    nnzb = want.col_indices().numel()
    ws = torch.empty(_capi.bsr_convert_workspace_bytes(M, K, bs), dtype=torch.uint8, device=cuda_dev)
    for cap in (nnzb, nnzb + 50, nnzb - 7, 0):  # exact, roomy, too small (truncated in BSR order), none
        rp = torch.full((M // bs + 1,), -1, dtype=idx, device=cuda_dev)
        ci = torch.full((cap,), -1, dtype=idx, device=cuda_dev)
        v = torch.full((cap, bs, bs), 7.0, dtype=torch.float16, device=cuda_dev)
        if kind == "dense":
            _capi.dense_to_bsr_bounded(x.to(cuda_dev), bs, rp, ci, v, ws)
        else:
            _capi.csr_to_bsr_bounded(csr.crow_indices().to(cuda_dev), csr.col_indices().to(cuda_dev),
                                     csr.values().to(cuda_dev), (M, K), bs, rp, ci, v, ws)
        torch.cuda.synchronize()
        n = min(cap, nnzb)
        assert torch.equal(rp.cpu().long(), want.crow_indices())
        assert torch.equal(ci.cpu().long()[:n], want.col_indices()[:n])
        assert torch.equal(_bits(v.cpu()[:n]), _bits(want.values()[:n]))
        if cap > nnzb:  # untouched beyond the true count
            assert torch.all(ci.cpu()[nnzb:] == -1) and torch.all(v.cpu()[nnzb:] == 7.0)
