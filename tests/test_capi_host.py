"""The C-ABI library loads without a GPU, exports every symbol include/bsk_capi.h declares, validates
arguments on the host, and fails loudly (never falls back) when no sm_100 device is present."""
import os
import re

import pytest
import torch

from periodicdent42_b200 import _capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "bsk_capi.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for s in ["bsk_gemm_f16f32", "bsk_gemm_e4m3_bf16", "bsk_spmm_bsr_f16f32", "bsk_bsattn_fwd_bf16", "bsk_bsattn_fwd_f16",
              "bsk_device_error", "launch_bsr_spmm_async", "bsk_last_error"]:
        assert s in syms, s


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), f"libbsk_sm100.so does not export {s}"
    assert set(declared_symbols()) == set(_capi.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version():
    assert _capi.lib().bsk_version() == 0x000100


def _fake(shape, dtype=torch.float16):
    return torch.empty(shape, dtype=dtype)  # host tensors: only their pointers/strides are used before validation fails


def test_gemm_argument_validation_on_host():
    A, Bt, C = _fake((64, 100)), _fake((64, 100)), _fake((64, 64), torch.float32)
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32(A, Bt, C, stream=0)  # lda = 100 is not a multiple of 8
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG
    A, Bt = _fake((64, 128)), _fake((64, 128))
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32(A, Bt, C, 8, 200, stream=0)  # k_end beyond K
    assert e.value.code == _capi.BSK_ERR_INVALID_ARG


def test_spmm_rejects_unsupported_block_shape_on_host():
    rp = torch.zeros(2, dtype=torch.int32)
    ci = torch.zeros(1, dtype=torch.int32)
    with pytest.raises(_capi.BskError) as e:
        _capi.spmm_bsr_f16f32(rp, ci, _fake((1, 16, 16)), _fake((16, 16)), _fake((16, 16), torch.float32), 16,
                              stream=0)
    assert e.value.code == _capi.BSK_ERR_UNSUPPORTED


@pytest.mark.parametrize("D", [32, 256])
def test_attention_rejects_head_dim_on_host(D):
    rp = torch.zeros(2, dtype=torch.int32)
    for dt, fn in [(torch.bfloat16, _capi.bsattn_fwd_bf16), (torch.float16, _capi.bsattn_fwd_f16)]:
        q = _fake((1, 1, 128, D), dt)
        with pytest.raises(_capi.BskError) as e:
            fn(q, q, q, q, rp, rp, 0.1, stream=0)
        assert e.value.code == _capi.BSK_ERR_UNSUPPORTED


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_fails_loudly():
    A, Bt, C = _fake((128, 64)), _fake((128, 64)), _fake((128, 128), torch.float32)
    with pytest.raises(_capi.BskError) as e:
        _capi.gemm_f16f32(A, Bt, C, stream=0)
    assert e.value.code == _capi.BSK_ERR_NO_DEVICE
    assert _capi.lib().bsk_device_sm_count() == _capi.BSK_ERR_NO_DEVICE


def test_bsr_validate_host():
    ok_rp = torch.tensor([0, 2, 2, 3], dtype=torch.int32)
    ok_ci = torch.tensor([0, 3, 1], dtype=torch.int32)
    _capi.bsr_validate_host(ok_rp, ok_ci, 4)
    bad = [
        (torch.tensor([1, 2, 2, 3], dtype=torch.int32), ok_ci, "row_ptr[0]"),
        (torch.tensor([0, 2, 1, 3], dtype=torch.int32), ok_ci, "decreases"),
        (torch.tensor([0, 2, 2, 2], dtype=torch.int32), ok_ci, "nnzb"),
        (ok_rp, torch.tensor([0, 4, 1], dtype=torch.int32), "outside"),
        (ok_rp, torch.tensor([0, -1, 1], dtype=torch.int32), "outside"),
    ]
    for rp, ci, msg in bad:
        with pytest.raises(_capi.BskError) as e:
            _capi.bsr_validate_host(rp, ci, 4)
        assert e.value.code == _capi.BSK_ERR_INVALID_ARG and msg in str(e.value)


def test_wait_timeout_bounds_validated():
    with pytest.raises(_capi.BskError):
        _capi.set_wait_timeout_ns(10)
    _capi.set_wait_timeout_ns(2_000_000_000)


def test_reference_launcher_signature_reports_errors():
    # block counts that do not divide M: recorded in bsk_last_error, nothing launched
    _capi.lib().launch_bsr_spmm_async(None, None, None, 3, 1, 0, None, None, None, 1, 1, 1, None, 256, 128, 128, 128,
                                      256, 128, 32, None)
    assert "divisible" in _capi.last_error()
