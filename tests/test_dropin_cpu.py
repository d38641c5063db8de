"""The reference's import name (no GPU): ``blackwellsparsek`` and ``blackwellsparsek._C`` resolve to this build's
package and extension, with the reference package's public names (BlackwellSparseK/python/__init__.py:27-39) and
submodules (python/ops.py, python/utils.py)."""
import importlib
import inspect

import periodicdent42_b200 as impl


def test_package_surface_matches_reference():
    bsk = importlib.import_module("blackwellsparsek")
    assert set(bsk.__all__) >= {"sparse_mm", "sparse_mm_benchmark", "convert_to_bsr", "validate_sparse_matrix"}
    for name in ["sparse_mm", "sparse_mm_benchmark", "convert_to_bsr", "validate_sparse_matrix", "attention_forward",
                 "get_optimal_block_size", "estimate_speedup"]:
        assert getattr(bsk, name) is getattr(impl.ops, name, None) or getattr(bsk, name) is getattr(impl.utils, name), name
    assert bsk.__version__ == impl.__version__
    assert list(inspect.signature(bsk.sparse_mm).parameters) == ["A", "B", "block_size", "autotune"]


def test_extension_module_name():
    import blackwellsparsek
    from periodicdent42_b200 import _C as ext

    mod = importlib.import_module("blackwellsparsek._C")
    assert mod is ext and blackwellsparsek._C is ext
    assert hasattr(mod, "sparse_mm_bsr")


def test_submodules():
    from blackwellsparsek import ops, utils

    assert ops.HAS_CUDA_EXT is True
    assert ops._default_config(8192, 8192, 8192) == {"BM": 256, "BN": 128, "BK": 32}
    assert callable(ops._convert_csr_to_bsr)
    assert utils.convert_to_bsr is impl.convert_to_bsr


def test_estimate_speedup_keys():
    import blackwellsparsek as bsk

    for dev in ("B200", "H100", "A100", "L4"):
        est = bsk.utils.estimate_speedup((8192, 8192), 0.75, device=dev)
        assert set(est) >= {"device", "matrix_shape", "sparsity", "tflops", "speedup_vs_pytorch", "note"}
        assert est["tflops"] > 0 and est["speedup_vs_pytorch"] > 0
    try:
        bsk.utils.estimate_speedup((8192, 8192), 0.75, device="TPU")
    except ValueError:
        pass
    else:
        raise AssertionError("unknown device accepted")
