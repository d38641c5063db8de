"""blackwellsparsek.ops -- the reference's operator module (BlackwellSparseK/python/ops.py), re-exported from
``periodicdent42_b200.ops``. ``HAS_CUDA_EXT`` keeps its meaning (ops.py:13-22): whether the extension imports."""
from periodicdent42_b200.ops import (_autotune_config, _convert_csr_to_bsr, _default_config, has_cuda_ext,
                                     sparse_mm, sparse_mm_benchmark)

HAS_CUDA_EXT = has_cuda_ext()

__all__ = ["sparse_mm", "sparse_mm_benchmark", "HAS_CUDA_EXT", "_convert_csr_to_bsr", "_default_config",
           "_autotune_config"]
