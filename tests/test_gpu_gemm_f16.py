"""Dense fp16 -> fp32 GEMM through the C ABI vs the reference's torch path and an fp64 recompute.
Tolerance: normwise relative error <= 1e-3 against fp64 (operator family's fp16/bf16 bar)."""
import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _run(A, Bt, k_begin=0, k_end=None):
    dev = torch.device("cuda", 0)
    Ad, Btd = A.to(dev), Bt.to(dev)
    C = torch.full((A.shape[0], Bt.shape[0]), float("nan"), device=dev)
    _capi.gemm_f16f32(Ad, Btd, C, k_begin, k_end)
    torch.cuda.synchronize()
    return C.cpu()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (384, 768, 1024), (200, 136, 72), (1, 8, 8),
                                   (130, 260, 136), (1000, 520, 264)])
def test_gemm_shapes(no_device_error, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    Bt = (torch.rand(N, K, generator=g) * 2 - 1).half()
    C = _run(A, Bt)
    assert torch.isfinite(C).all()
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, err
    ok, m = ref.validate_correctness(C, ref.dense_ref(A, Bt), rtol=1e-4, atol=1e-4)
    assert ok, m


def test_gemm_config1_1024(no_device_error):
    A, Bt = wl.dense_inputs(wl.DENSE_SMALL, "cpu")
    C = _run(A, Bt)
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, err
    ok, m = ref.validate_correctness(C, ref.dense_ref(A, Bt), rtol=1e-4, atol=1e-3)
    assert ok, m


def test_gemm_split_k_range(no_device_error):
    g = torch.Generator().manual_seed(5)
    A = torch.randn(256, 1024, generator=g).half()
    Bt = torch.randn(512, 1024, generator=g).half()
    parts = [_run(A, Bt, a, b) for a, b in [(0, 384), (384, 1000), (1000, 1024)]]
    C = sum(parts)
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, err
    # one shard alone equals the product over its K range
    err0 = ref.normwise_rel_err(parts[1], ref.dense_fp64(A[:, 384:1000], Bt[:, 384:1000]))
    assert err0 <= TOL, err0


def test_gemm_deterministic(no_device_error):
    g = torch.Generator().manual_seed(9)
    A = torch.randn(512, 2048, generator=g).half()
    Bt = torch.randn(1024, 2048, generator=g).half()
    assert torch.equal(_run(A, Bt), _run(A, Bt))


def test_gemm_rejects_bad_args(cuda_dev):
    A = torch.zeros(128, 100, dtype=torch.float16, device=cuda_dev)  # lda 100 not a multiple of 8
    Bt = torch.zeros(128, 100, dtype=torch.float16, device=cuda_dev)
    C = torch.zeros(128, 128, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32(A, Bt, C)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG


@pytest.mark.parametrize("tile", ["pair", "wide", "single"])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 640), (300, 520, 200), (1024, 1024, 1024),
                                   (768, 1536, 4160)])
def test_gemm_tile_variants(no_device_error, monkeypatch, tile, M, N, K):
    """The CTA-pair 256x256 and 256x512 kernels and the single-CTA 128x256 kernel against fp64."""
    monkeypatch.setenv("BSK_GEMM_TILE", tile)
    g = torch.Generator().manual_seed(M + 3 * N + 7 * K)
    A = torch.randn(M, K, generator=g).half()
    Bt = torch.randn(N, K, generator=g).half()
    C = _run(A, Bt)
    err = ref.normwise_rel_err(C, ref.dense_fp64(A, Bt))
    assert err <= TOL, (tile, err)


def test_gemm_pair_and_single_agree_bitwise(no_device_error, monkeypatch):
    """Same K order of accumulation in both kernels: identical fp32 results."""
    g = torch.Generator().manual_seed(77)
    A = torch.randn(512, 1024, generator=g).half()
    Bt = torch.randn(512, 1024, generator=g).half()
    outs = []
    for tile in ("pair", "wide", "single"):
        monkeypatch.setenv("BSK_GEMM_TILE", tile)
        outs.append(_run(A, Bt))
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


@pytest.mark.parametrize("M,N,K,splits", [(1024, 1024, 1024, 0), (256, 512, 8192, 4), (300, 520, 4160, 3),
                                          (512, 1024, 65536, 0), (200, 136, 2048, 5), (2048, 2048, 512, 0)])
def test_gemm_splitk(no_device_error, M, N, K, splits):
    """Split-K (fp32 partial slabs in a workspace, deterministic reduction) against fp64."""
    g = torch.Generator().manual_seed(M + N + K + splits)
    A = torch.randn(M, K, generator=g).half()
    Bt = torch.randn(N, K, generator=g).half()
    dev = torch.device("cuda", 0)
    C = torch.full((M, N), float("nan"), device=dev)
    _capi.gemm_f16f32_splitk(A.to(dev), Bt.to(dev), C, splits)
    torch.cuda.synchronize()
    err = ref.normwise_rel_err(C.cpu(), ref.dense_fp64(A, Bt))
    assert err <= TOL, err


def test_gemm_splitk_workspace_contract(cuda_dev):
    assert _capi.gemm_splitk_workspace_bytes(1024, 1024, 1024, 4) == 4 * 1024 * 1024 * 4
    assert _capi.gemm_splitk_workspace_bytes(8192, 8192, 237568, 0) == 0  # enough tiles: no split chosen
    A = torch.zeros(256, 8192, dtype=torch.float16, device=cuda_dev)
    Bt = torch.zeros(256, 8192, dtype=torch.float16, device=cuda_dev)
    C = torch.empty(256, 256, device=cuda_dev)
    small = torch.empty(16, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32_splitk(A, Bt, C, 4, workspace=small)
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG and "workspace" in str(e.value)


def test_gemm_splitk_deterministic_and_matches_single_pass(no_device_error):
    g = torch.Generator().manual_seed(31)
    A = torch.randn(512, 16384, generator=g).half()
    Bt = torch.randn(768, 16384, generator=g).half()
    dev = torch.device("cuda", 0)
    Ad, Btd = A.to(dev), Bt.to(dev)
    c1 = torch.empty(512, 768, device=dev)
    c2 = torch.empty(512, 768, device=dev)
    _capi.gemm_f16f32_splitk(Ad, Btd, c1, 8)
    _capi.gemm_f16f32_splitk(Ad, Btd, c2, 8)
    c3 = torch.empty(512, 768, device=dev)
    _capi.gemm_f16f32(Ad, Btd, c3)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)  # deterministic split reduction
    # A different K partition rounds the tensor core's fp32 accumulation differently (~1e-5 normwise at
    # K = 16384); both must sit well inside the 1e-3 bar against fp64.
    c64 = ref.dense_fp64(A, Bt)
    assert ref.normwise_rel_err(c1.cpu(), c64) < 1e-4
    assert ref.normwise_rel_err(c3.cpu(), c64) < 1e-4
