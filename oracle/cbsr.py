"""ctypes access to the C restatement of cpu_bsr and to the reference's compiled cpu_bsr -- TEST
INFRASTRUCTURE ONLY."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .build import ORACLE_LIB, REF_LIB

_c = {}


def _load(path: str):
    if path not in _c:
        _c[path] = ctypes.CDLL(path)
    return _c[path]


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def oracle_cpu_bsr(A_blocks_f16: np.ndarray, row_ptr: np.ndarray, col_idx: np.ndarray, B_f16: np.ndarray,
                   M: int, N: int, K: int, BM: int, BN: int, BK: int) -> np.ndarray:
    """C restatement (oracle/bsr_oracle.c). A_blocks [nnz, BM, BK] float16, B [K, N] float16."""
    lib = _load(ORACLE_LIB)
    A = np.ascontiguousarray(A_blocks_f16, dtype=np.float16).view(np.uint16)
    B = np.ascontiguousarray(B_f16, dtype=np.float16).view(np.uint16)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    C = np.empty((M, N), dtype=np.float32)
    f = lib.oracle_cpu_bsr
    f.restype = None
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 6
    f(_p(A), _p(rp), _p(ci), _p(B), _p(C), M, N, K, BM, BN, BK)
    return C


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_block_dims() -> tuple[int, int, int]:
    lib = _load(REF_LIB)
    bm, bn, bk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    lib.ref_block_dims(ctypes.byref(bm), ctypes.byref(bn), ctypes.byref(bk))
    return bm.value, bn.value, bk.value


def ref_cpu_bsr(A_blocks_f16: np.ndarray, row_ptr: np.ndarray, col_idx: np.ndarray, B_f16: np.ndarray,
                M: int, N: int, K: int) -> np.ndarray:
    """The reference's own cpu_bsr (BlackwellSparseK/src/bsr_reference.cu:72-93), compiled from source."""
    lib = _load(REF_LIB)
    A = np.ascontiguousarray(A_blocks_f16, dtype=np.float16).view(np.uint16)
    B = np.ascontiguousarray(B_f16, dtype=np.float16).view(np.uint16)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    C = np.empty((M, N), dtype=np.float32)
    f = lib.ref_cpu_bsr
    f.restype = None
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    f(_p(A), A.size, _p(rp), rp.size - 1, _p(ci), ci.size, _p(B), B.size, _p(C), M, N, K)
    return C
