"""Python API surface (no GPU): reference names and signatures exist, CPU tensors are rejected (no CPU
fallback), and block-mask normalisation is exact."""
import inspect

import pytest
import torch

import periodicdent42_b200 as bsk
from periodicdent42_b200 import ops


def test_reference_surface_present():
    for name in ["sparse_mm", "sparse_mm_benchmark", "convert_to_bsr", "validate_sparse_matrix", "attention_forward",
                 "__version__"]:
        assert hasattr(bsk, name)
    sig = inspect.signature(bsk.sparse_mm)
    assert list(sig.parameters) == ["A", "B", "block_size", "autotune"]
    assert sig.parameters["block_size"].default == 16 and sig.parameters["autotune"].default is False
    sig = inspect.signature(bsk.attention_forward)
    assert list(sig.parameters)[:4] == ["Q", "K", "V", "scale"]
    assert ops._default_config(8192, 8192, 8192) == {"BM": 256, "BN": 128, "BK": 32}
    assert ops._autotune_config(20000, 1, 1)["BM"] == 512


def test_extension_surface():
    from periodicdent42_b200 import _C

    for name in ["sparse_mm_bsr", "gemm_f16f32", "gemm_e4m3", "bsattn_fwd", "device_error"]:
        assert hasattr(_C, name)


def test_cpu_inputs_rejected():
    A = torch.eye(256, dtype=torch.float16).to_sparse_bsr((128, 128))
    B = torch.zeros(256, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        bsk.sparse_mm(A, B)
    with pytest.raises(ValueError, match="sparse"):
        bsk.sparse_mm(torch.zeros(4, 4), B)
    with pytest.raises(ValueError):
        bsk.gemm(torch.zeros(4, 8, dtype=torch.float16), torch.zeros(8, 4, dtype=torch.float16))
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        bsk.attention_forward(q, q, q)


def test_block_mask_forms():
    nqb = 3
    m = torch.tensor([[1, 0, 0], [1, 1, 0], [0, 1, 1]], dtype=torch.bool)
    rp, ci = ops.block_mask_to_bsr(m, 2, 1, nqb, False, "cpu")
    assert rp.tolist() == [0, 1, 3, 5, 6, 8, 10] and ci.tolist() == [0, 0, 1, 1, 2, 0, 0, 1, 1, 2]
    m4 = m.expand(2, 1, 3, 3)
    rp4, ci4 = ops.block_mask_to_bsr(m4, 2, 1, nqb, False, "cpu")
    assert torch.equal(rp, rp4) and torch.equal(ci, ci4)
    rp_c, ci_c = ops.block_mask_to_bsr(None, 1, 1, nqb, True, "cpu")
    assert rp_c.tolist() == [0, 1, 3, 6] and ci_c.tolist() == [0, 0, 1, 0, 1, 2]


def test_validate_sparse_matrix_messages():
    dense = torch.zeros(8, 8)
    ok, info = bsk.validate_sparse_matrix(dense)
    assert not ok and info["message"] == "Matrix is not sparse"
    ok, info = bsk.validate_sparse_matrix(dense.to_sparse_csr())
    assert not ok and info["message"] == "Matrix is not on CUDA device"


def test_convert_to_bsr_cpu():
    d = torch.zeros(256, 256)
    d[:128, 128:] = 1.0
    b = bsk.convert_to_bsr(d, block_size=128, sparsity_threshold=0.0)
    assert b.layout == torch.sparse_bsr and b.crow_indices().tolist() == [0, 1, 1] and b.col_indices().tolist() == [1]
    assert bsk.get_optimal_block_size((8192, 8192)) == 128
