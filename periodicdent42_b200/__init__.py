"""periodicdent42_b200 -- B200-native (sm_100a) BlackwellSparseK operator family.

Drop-in for the reference package ``blackwellsparsek`` (BlackwellSparseK/python/__init__.py): same
functions and signatures, backed by hand-written tcgen05/TMA kernels behind a C ABI
(include/bsk_capi.h, libbsk_sm100.so) and the torch extension ``periodicdent42_b200._C``.

    >>> import periodicdent42_b200 as bsk
    >>> C = bsk.sparse_mm(A_bsr, B)          # BSR x dense, fp16 -> fp32
    >>> C = bsk.gemm(A, B)                   # dense fp16 -> fp32
    >>> D = bsk.gemm_fp8(Aq, Bq, sa, sb)     # e4m3 -> bf16, per-tensor scales
    >>> O = bsk.attention_forward(Q, K, V, block_mask=mask, causal=True)
"""

__version__ = "0.9.0+sm100a"

from .ops import (attention_forward, gemm, gemm_fp8, gemm_from_host, has_cuda_ext, quantize_e4m3, sparse_mm,
                  sparse_mm_benchmark, synchronize_and_check)
from .utils import convert_to_bsr, get_optimal_block_size, validate_sparse_matrix

__all__ = [
    "sparse_mm",
    "sparse_mm_benchmark",
    "convert_to_bsr",
    "validate_sparse_matrix",
    "get_optimal_block_size",
    "gemm",
    "gemm_fp8",
    "gemm_from_host",
    "quantize_e4m3",
    "attention_forward",
    "has_cuda_ext",
    "synchronize_and_check",
    "__version__",
]
