"""blackwellsparsek -- the reference package's import name, served by the B200 (sm_100a) build.

Existing callers keep ``import blackwellsparsek as bsk`` and ``bsk._C.sparse_mm_bsr(...)`` unchanged
(BlackwellSparseK/python/__init__.py:27-39, setup.py:18); every name resolves to ``periodicdent42_b200``, whose
operators run the hand-written tcgen05/TMA kernels of ``libbsk_sm100.so``. Nothing here computes: this package
only re-exports, so the two import names always run the same code.

    >>> import blackwellsparsek as bsk
    >>> C = bsk.sparse_mm(A_bsr, B)                  # BSR (or CSR) x dense, fp16 -> fp32
    >>> O = bsk.attention_forward(Q, K, V)           # the archived attention API
    >>> C = bsk._C.sparse_mm_bsr(rp, ci, vals, brp, bci, bvals, M, N, K, 256, 128, 32)
"""
from periodicdent42_b200 import __version__
from periodicdent42_b200.ops import attention_forward, gemm, gemm_fp8, quantize_e4m3, sparse_mm, sparse_mm_benchmark
from periodicdent42_b200.utils import convert_to_bsr, estimate_speedup, get_optimal_block_size, validate_sparse_matrix

from . import ops, utils  # noqa: E402  (the reference's submodules: bsk.ops, bsk.utils)

__all__ = [
    "sparse_mm",
    "sparse_mm_benchmark",
    "convert_to_bsr",
    "validate_sparse_matrix",
    "attention_forward",
    "__version__",
]


def __getattr__(name):
    # `bsk._C` without an explicit `import blackwellsparsek._C`, as the reference's package makes it available
    if name == "_C":
        import importlib

        return importlib.import_module(__name__ + "._C")
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
