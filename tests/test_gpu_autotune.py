"""Autotuner on the GPU: every candidate launch configuration computes the same product (parity with fp64 for each
tile kind and rasterisation group, ragged shape), tuning registers and caches the fastest, the cache restores it,
and the public autotune switches (gemm, sparse_mm) run through it.
Tolerance: normwise relative error <= 1e-3 against fp64."""
import pytest
import torch

import periodicdent42_b200 as bsk
from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import autotune as at
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(autouse=True)
def _clean_table():
    at.clear()
    yield
    at.clear()


def test_every_gemm_candidate_is_correct(no_device_error, cuda_dev):
    M, N, K = 700, 900, 520
    g = torch.Generator().manual_seed(3)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    Bt = (torch.rand(N, K, generator=g) * 2 - 1).half()
    want = ref.dense_fp64(A, Bt)
    Ad, Btd = A.to(cuda_dev), Bt.to(cuda_dev)
    for tile, group in at.candidates("gemm_f16f32", M, N, K):
        at.register("gemm_f16f32", M, N, K, tile, group)
        C = torch.full((M, N), float("nan"), device=cuda_dev)
        _capi.gemm_f16f32(Ad, Btd, C)
        torch.cuda.synchronize()
        err = ref.normwise_rel_err(C.cpu(), want)
        assert err <= TOL, (tile, group, err)


def test_every_spmm_candidate_is_correct(no_device_error, cuda_dev):
    cfg = wl.BsrCfg(1024, 768, 1280, 128, 3, 9)
    crow, col, vals, B = wl.bsr_inputs(cfg, "cpu")
    want = wl.bsr_tensor(crow, col, vals, cfg.M, cfg.K).to_dense().double() @ B.double()
    rp, ci = crow.to(torch.int32).to(cuda_dev), col.to(torch.int32).to(cuda_dev)
    for tile, group in at.candidates("spmm_bsr", cfg.M, cfg.N, cfg.K):
        at.register("spmm_bsr", cfg.M, cfg.N, cfg.K, tile, group)
        C = torch.full((cfg.M, cfg.N), float("nan"), device=cuda_dev)
        _capi.spmm_bsr_f16f32(rp, ci, vals.to(cuda_dev), B.to(cuda_dev), C, cfg.M)
        torch.cuda.synchronize()
        assert ref.normwise_rel_err(C.cpu(), want) <= TOL, group


def test_tune_registers_caches_and_restores(no_device_error, cuda_dev, tmp_path):
    path = str(tmp_path / "cache.json")
    cache = at.AutotuneCache(path)
    e = at.tune_gemm(1024, 2048, 4096, warmup=1, runs=3, rounds=1, settle_ms=5, cache=cache, save=True)
    assert e["tile"] in (-1, 0, 1, 2) and e["ms"] <= e["default_ms"]
    assert at.registered("gemm_f16f32", 1024, 2048, 4096) == (e["tile"], e["group_m"])
    at.clear()
    assert at.load_cache(path) == 1
    assert at.registered("gemm_f16f32", 1024, 2048, 4096) == (e["tile"], e["group_m"])


def test_public_autotune_switches(no_device_error, cuda_dev, tmp_path, monkeypatch):
    monkeypatch.setenv("BSK_AUTOTUNE_CACHE", str(tmp_path / "c.json"))
    g = torch.Generator().manual_seed(4)
    A = torch.randn(512, 1024, generator=g).half()
    B = torch.randn(1024, 768, generator=g).half()
    C = bsk.gemm(A.to(cuda_dev), B.to(cuda_dev), autotune=True)
    assert at.registered("gemm_f16f32", 512, 768, 1024) is not None
    assert ref.normwise_rel_err(C.cpu(), A.double() @ B.double()) <= TOL
    cfg = wl.BsrCfg(512, 512, 768, 128, 2, 5)
    crow, col, vals, Bs = wl.bsr_inputs(cfg, "cpu")
    Abs = wl.bsr_tensor(crow, col, vals, cfg.M, cfg.K).to(cuda_dev)
    Cs = bsk.sparse_mm(Abs, Bs.to(cuda_dev), autotune=True)
    assert at.registered("spmm_bsr", cfg.M, cfg.N, cfg.K) is not None
    want = wl.bsr_tensor(crow, col, vals, cfg.M, cfg.K).to_dense().double() @ Bs.double()
    assert ref.normwise_rel_err(Cs.cpu(), want) <= TOL
    assert (tmp_path / "c.json").exists()
