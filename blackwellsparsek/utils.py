"""blackwellsparsek.utils -- the reference's helper module (BlackwellSparseK/python/utils.py), re-exported from
``periodicdent42_b200.utils``."""
from periodicdent42_b200.utils import convert_to_bsr, estimate_speedup, get_optimal_block_size, validate_sparse_matrix

__all__ = ["convert_to_bsr", "validate_sparse_matrix", "get_optimal_block_size", "estimate_speedup"]
