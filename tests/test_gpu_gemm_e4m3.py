"""FP8 e4m3 GEMM (per-tensor scales, bf16 out) through the C ABI vs torch._scaled_mm on CPU (the stated
semantics) and an fp64 recompute on the same e4m3 bytes. Tolerance: normwise relative error <= 3e-2."""
import pytest
import torch

from oracle import reference_path as ref
from periodicdent42_b200 import _capi
from periodicdent42_b200 import workloads as wl

pytestmark = pytest.mark.gpu
TOL = 3e-2


def _run(Aq, Bqt, sa, sb):
    dev = torch.device("cuda", 0)
    D = torch.full((Aq.shape[0], Bqt.shape[0]), float("nan"), dtype=torch.bfloat16, device=dev)
    _capi.gemm_e4m3_bf16(Aq.to(dev), Bqt.to(dev), sa.to(dev), sb.to(dev), D)
    torch.cuda.synchronize()
    return D.cpu()


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 512), (200, 136, 144), (1024, 1024, 2048)])
def test_fp8_shapes(no_device_error, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    Aq, sa = wl.quantize_e4m3(torch.randn(M, K, generator=g))
    Bqt, sb = wl.quantize_e4m3(torch.randn(N, K, generator=g))
    D = _run(Aq, Bqt, sa, sb)
    assert torch.isfinite(D.float()).all()
    err = ref.normwise_rel_err(D, ref.fp8_fp64(Aq, Bqt, sa, sb))
    assert err <= TOL, err
    err_ref = ref.normwise_rel_err(D, ref.fp8_ref(Aq, Bqt, sa, sb))
    assert err_ref <= 1e-2, err_ref


def test_fp8_scales_applied(no_device_error):
    g = torch.Generator().manual_seed(3)
    Aq, sa = wl.quantize_e4m3(torch.randn(256, 256, generator=g) * 50)
    Bqt, sb = wl.quantize_e4m3(torch.randn(256, 256, generator=g) * 0.01)
    D = _run(Aq, Bqt, sa, sb)
    err = ref.normwise_rel_err(D, ref.fp8_fp64(Aq, Bqt, sa, sb))
    assert err <= TOL, err


@pytest.mark.parametrize("tile", ["pair", "wide", "single"])
def test_fp8_tile_variants(no_device_error, monkeypatch, tile):
    monkeypatch.setenv("BSK_GEMM_TILE", tile)
    g = torch.Generator().manual_seed(17)
    Aq, sa = wl.quantize_e4m3(torch.randn(640, 1024, generator=g))
    Bqt, sb = wl.quantize_e4m3(torch.randn(768, 1024, generator=g))
    D = _run(Aq, Bqt, sa, sb)
    err = ref.normwise_rel_err(D, ref.fp8_fp64(Aq, Bqt, sa, sb))
    assert err <= TOL, (tile, err)
