"""ctypes binding of the C ABI in include/bsk_capi.h (libbsk_sm100.so).

This is the path the parity tests and the benchmark use to call the kernels exactly as a foreign
caller would (plain pointers, sizes and a cudaStream_t). There is no fallback: if the library is
missing or the device is not an sm_100 part, calls raise ``BskError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

# BSK_CAPI_LIB selects another build of the library (e.g. one compiled with different tuning macros).
LIB_PATH = os.environ.get("BSK_CAPI_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                          "libbsk_sm100.so")

BSK_OK = 0
BSK_ERR_INVALID_ARG = -1
BSK_ERR_UNSUPPORTED = -2
BSK_ERR_CUDA = -3
BSK_ERR_DEVICE_TIMEOUT = -4
BSK_ERR_NO_DEVICE = -5

# Every symbol include/bsk_capi.h declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float
SIGNATURES = {
    "bsk_version": (_i32, []),
    "bsk_last_error": (ctypes.c_char_p, []),
    "bsk_device_sm_count": (_i32, []),
    "bsk_config_set": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "bsk_config_get": (_i32, [_i32, _i32, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "bsk_config_clear": (_i32, []),
    "bsk_gemm_f16f32": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp]),
    "bsk_gemm_f16f32_acc": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp]),
    "bsk_gemm_f16f32_host": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp]),
    "bsk_gemm_host_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "bsk_gemm_host_chunk": (_i32, [_i32, _i32]),
    "bsk_copy_2d_async": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "bsk_gemm_f16f32_splitk": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp]),
    "bsk_gemm_splitk_workspace_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "bsk_gemm_f16f32_splitk_static": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp]),
    "bsk_gemm_f16f32_splitk_scatter": (_i32, [_vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                               ctypes.POINTER(ctypes.c_void_p), _i64, _vp]),
    "bsk_splitk_slots_reduce": (_i32, [_vp, _i32, _i32, _i32, _i64, _vp, _i64, _vp]),
    "bsk_peer_buffer_alloc": (_i32, [_i64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "bsk_peer_buffer_open": (_i32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "bsk_peer_buffer_close": (_i32, [_vp]),
    "bsk_peer_buffer_free": (_i32, [_vp]),
    "bsk_gemm_e4m3_bf16": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp]),
    "bsk_spmm_bsr_f16f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _i32, _i32, _i32,
                                   _i32, _i32, _vp]),
    "bsk_bsr_validate_host": (_i32, [_vp, _vp, _i32, _i32, _i32]),
    "bsk_spmm_bsr_bsr_f16f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _i32, _i32, _i32,
                                       _i32, _i32, _vp]),
    "bsk_bsr_convert_workspace_bytes": (_i64, [_i32, _i32, _i32]),
    "bsk_dense_to_bsr_pattern": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _vp, _i64,
                                        ctypes.POINTER(_i64), ctypes.POINTER(_i64), _vp]),
    "bsk_dense_to_bsr_fill": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _i64,
                                     _vp]),
    "bsk_csr_to_bsr_pattern": (_i32, [_vp, _vp, _i32, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _i32, _vp, _i64,
                                      ctypes.POINTER(_i64), ctypes.POINTER(_i64), _vp]),
    "bsk_csr_to_bsr_fill": (_i32, [_vp, _vp, _i32, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _i32, _vp, _i64, _vp,
                                   _i64, _vp]),
    "bsk_dense_to_bsr_bounded": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _i64,
                                        _vp]),
    "bsk_csr_to_bsr_bounded": (_i32, [_vp, _vp, _i32, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _i32, _vp, _i64,
                                      _vp, _i64, _vp]),
    "bsk_bsattn_fwd_bf16": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32,
                                   _i32, _vp]),
    "bsk_bsattn_fwd_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32,
                                  _i32, _vp]),
    "bsk_bsattn_fwd_ex": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _i32,
                                 _i32, _i32, _vp]),
    "bsk_bsattn_mask_transpose": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _i64, _vp]),
    "bsk_bsattn_bwd": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                              _i32, _i32, _f32, _i32, _vp, _vp]),
    "launch_attention_forward": (None, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, ctypes.c_bool, _vp]),
    "launch_attention_backward": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32,
                                         ctypes.c_bool, _vp]),
    "launch_bsr_spmm_async": (None, [_vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _i32,
                                     _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "bsk_device_error": (_i32, [ctypes.POINTER(ctypes.c_uint32)]),
    "bsk_set_wait_timeout_ns": (_i32, [_u64]),
    "bsk_selftest_wait_timeout": (_i32, [_u64, _vp]),
    "bsk_selftest_exp2": (_i32, [_vp, _vp, _i32, _i32, _vp]),
}


class BskError(RuntimeError):
    def __init__(self, code: int, what: str, msg: str):
        super().__init__(f"{what} failed with code {code}: {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libbsk_sm100.so once and attach the declared signatures."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m periodicdent42_b200.build`")
                l = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(l, name)
                    f.restype = res
                    f.argtypes = args
                _lib = l
    return _lib


def last_error() -> str:
    return lib().bsk_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != BSK_OK:
        raise BskError(rc, what, last_error())


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return int(stream) if isinstance(stream, int) else stream.cuda_stream


def gemm_f16f32(A, Bt, C, k_begin: int = 0, k_end: int | None = None, stream=None) -> None:
    """C[M,N] fp32 = A[M,K] fp16 @ B[K,N], B passed as Bt = B^T row-major [N,K] (column-major B)."""
    M, K = A.shape
    N = Bt.shape[0]
    k_end = K if k_end is None else k_end
    check(lib().bsk_gemm_f16f32(_ptr(A), A.stride(0), _ptr(Bt), Bt.stride(0), _ptr(C), C.stride(0), M, N, K,
                                k_begin, k_end, _stream(stream)), "bsk_gemm_f16f32")


def gemm_f16f32_acc(A, Bt, C, k_begin: int = 0, k_end: int | None = None, stream=None) -> None:
    """C[M,N] += A[M, k_begin:k_end] @ B[k_begin:k_end, N] (fp32 C read and updated in place)."""
    M, K = A.shape
    N = Bt.shape[0]
    k_end = K if k_end is None else k_end
    check(lib().bsk_gemm_f16f32_acc(_ptr(A), A.stride(0), _ptr(Bt), Bt.stride(0), _ptr(C), C.stride(0), M, N, K,
                                    k_begin, k_end, _stream(stream)), "bsk_gemm_f16f32_acc")


def gemm_host_workspace_bytes(M: int, N: int, K: int, k_chunk: int = 0) -> int:
    n = lib().bsk_gemm_host_workspace_bytes(M, N, K, k_chunk)
    if n < 0:
        raise BskError(n, "bsk_gemm_host_workspace_bytes", last_error())
    return n


def gemm_host_chunk(K: int, k_chunk: int = 0) -> int:
    """K elements per chunk of the host-streaming GEMM for this K and request (0 = automatic)."""
    n = lib().bsk_gemm_host_chunk(K, k_chunk)
    if n < 0:
        raise BskError(n, "bsk_gemm_host_chunk", last_error())
    return n


def copy_2d_async(dst: int, dpitch: int, src: int, spitch: int, width_bytes: int, rows: int, stream=None) -> None:
    """cudaMemcpy2DAsync between raw addresses (host or device, direction by unified addressing)."""
    check(lib().bsk_copy_2d_async(dst, dpitch, src, spitch, width_bytes, rows, _stream(stream)), "bsk_copy_2d_async")


def gemm_f16f32_host(A_h, Bt_h, C_h, workspace, k_chunk: int = 0, stream=None) -> None:
    """C_h = A_h @ B for HOST tensors (pinned for overlap), streamed through the GPU in K chunks; `workspace` is
    a CUDA uint8 tensor of gemm_host_workspace_bytes(M, N, K, k_chunk) bytes. Asynchronous on `stream`."""
    M, K = A_h.shape
    N = Bt_h.shape[0]
    nbytes = workspace.numel() * workspace.element_size()
    check(lib().bsk_gemm_f16f32_host(_ptr(A_h), A_h.stride(0), _ptr(Bt_h), Bt_h.stride(0), _ptr(C_h), C_h.stride(0),
                                     M, N, K, k_chunk, _ptr(workspace), nbytes, _stream(stream)),
          "bsk_gemm_f16f32_host")


def gemm_splitk_workspace_bytes(M: int, N: int, K: int, splits: int = 0) -> int:
    n = lib().bsk_gemm_splitk_workspace_bytes(M, N, K, splits)
    if n < 0:
        raise BskError(n, "bsk_gemm_splitk_workspace_bytes", last_error())
    return n


def gemm_f16f32_splitk(A, Bt, C, splits: int = 0, workspace=None, stream=None) -> None:
    """C = A @ B with K split across CTA pairs; `workspace` (a CUDA tensor) defaults to a fresh uint8 buffer of
    the queried size."""
    import torch

    M, K = A.shape
    N = Bt.shape[0]
    need = gemm_splitk_workspace_bytes(M, N, K, splits)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=A.device)
    nbytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().bsk_gemm_f16f32_splitk(_ptr(A), A.stride(0), _ptr(Bt), Bt.stride(0), _ptr(C), C.stride(0), M, N, K,
                                       splits, _ptr(workspace), nbytes, _stream(stream)), "bsk_gemm_f16f32_splitk")


def gemm_f16f32_splitk_static(A, Bt, C, splits: int = 0, stream=None) -> None:
    """Split-K GEMM that allocates nothing: the partials live in the library's static 32 MiB device array
    (for callers that cannot allocate device memory). Concurrent calls on the GPU race on that array."""
    M, K = A.shape
    N = Bt.shape[0]
    check(lib().bsk_gemm_f16f32_splitk_static(_ptr(A), A.stride(0), _ptr(Bt), Bt.stride(0), _ptr(C), C.stride(0), M,
                                              N, K, splits, _stream(stream)), "bsk_gemm_f16f32_splitk_static")


def gemm_e4m3_bf16(Aq, Bqt, scale_a, scale_b, D, stream=None) -> None:
    """D[M,N] bf16 = (Aq[M,K] @ Bq[K,N]) * scale_a * scale_b, Bq passed as Bqt [N,K] (column-major B)."""
    M, K = Aq.shape
    N = Bqt.shape[0]
    check(lib().bsk_gemm_e4m3_bf16(_ptr(Aq), Aq.stride(0), _ptr(Bqt), Bqt.stride(0), _ptr(scale_a), _ptr(scale_b),
                                   _ptr(D), D.stride(0), M, N, K, _stream(stream)), "bsk_gemm_e4m3_bf16")


def spmm_bsr_f16f32(row_ptr, col_idx, vals, B, C, M: int, row_begin: int = 0, row_end: int | None = None,
                    stream=None) -> None:
    """C = A_bsr @ B for block-rows [row_begin, row_end); int32 indices, vals [nnzb, br, bc] fp16."""
    nnzb, br, bc = vals.shape
    Mb = row_ptr.numel() - 1
    K, N = B.shape
    row_end = Mb if row_end is None else row_end
    check(lib().bsk_spmm_bsr_f16f32(_ptr(row_ptr), _ptr(col_idx), _ptr(vals), br, bc, Mb, nnzb, _ptr(B), B.stride(0),
                                    _ptr(C), C.stride(0), M, N, K, row_begin, row_end, _stream(stream)),
          "bsk_spmm_bsr_f16f32")


def spmm_bsr_bsr_f16f32(a_row_ptr, a_col_idx, a_vals, b_row_ptr, b_col_idx, b_vals, C, M: int, N: int, K: int,
                        row_begin: int = 0, row_end: int | None = None, stream=None) -> None:
    """C = A_bsr @ B_bsr (both 128x128 blocks, int32 indices, fp16 values [nnzb, 128, 128]) into fp32 C."""
    Mb = M // 128
    row_end = Mb if row_end is None else row_end
    check(lib().bsk_spmm_bsr_bsr_f16f32(_ptr(a_row_ptr), _ptr(a_col_idx), _ptr(a_vals), Mb, a_col_idx.numel(),
                                        _ptr(b_row_ptr), _ptr(b_col_idx), _ptr(b_vals), b_col_idx.numel(), _ptr(C),
                                        C.stride(0), M, N, K, row_begin, row_end, _stream(stream)),
          "bsk_spmm_bsr_bsr_f16f32")


def bsattn_fwd_bf16(Q, K, V, O, row_ptr, col_idx, scale: float, causal_diag: bool = True, bh_begin: int = 0,
                    bh_end: int | None = None, blk: int = 128, stream=None) -> None:
    """O = block-sparse softmax(scale * Q K^T) V over the BSR block mask (row_ptr, col_idx)."""
    B, H, S, D = Q.shape
    bh_end = B * H if bh_end is None else bh_end
    check(lib().bsk_bsattn_fwd_bf16(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(row_ptr), _ptr(col_idx), B, H, S, D, blk,
                                    float(scale), int(bool(causal_diag)), bh_begin, bh_end, _stream(stream)),
          "bsk_bsattn_fwd_bf16")


def bsattn_fwd_f16(Q, K, V, O, row_ptr, col_idx, scale: float, causal_diag: bool = True, bh_begin: int = 0,
                   bh_end: int | None = None, blk: int = 128, stream=None) -> None:
    """fp16 form of bsattn_fwd_bf16 (same arguments)."""
    B, H, S, D = Q.shape
    bh_end = B * H if bh_end is None else bh_end
    check(lib().bsk_bsattn_fwd_f16(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(row_ptr), _ptr(col_idx), B, H, S, D, blk,
                                   float(scale), int(bool(causal_diag)), bh_begin, bh_end, _stream(stream)),
          "bsk_bsattn_fwd_f16")


def bsr_convert_workspace_bytes(M: int, K: int, bs: int) -> int:
    n = lib().bsk_bsr_convert_workspace_bytes(M, K, bs)
    if n < 0:
        raise BskError(n, "bsk_bsr_convert_workspace_bytes", last_error())
    return n


def _index_bytes(dtype) -> int:
    import torch

    if dtype not in (torch.int32, torch.int64):
        raise ValueError("index tensors must be int32 or int64")
    return 4 if dtype == torch.int32 else 8


def dense_to_bsr(A, bs: int, index_dtype=None, stream=None):
    """Device dense [M, K] (fp16 / bf16 / fp32, unit column stride) -> (row_ptr, col_idx, values, nnz_elems), the
    block pattern and blocks torch's A.to_sparse_bsr((bs, bs)) stores. Synchronises the stream once (to size
    the outputs)."""
    import torch

    index_dtype = torch.int64 if index_dtype is None else index_dtype
    ib = _index_bytes(index_dtype)
    M, K = A.shape
    if A.stride(1) != 1 and A.numel() > 0:
        raise ValueError("dense_to_bsr: A needs unit column stride")
    eb = A.element_size()
    ws = torch.empty(bsr_convert_workspace_bytes(M, K, bs), dtype=torch.uint8, device=A.device)
    row_ptr = torch.empty(M // bs + 1, dtype=index_dtype, device=A.device)
    nnzb, nnz = ctypes.c_int64(0), ctypes.c_int64(0)
    lda = A.stride(0) if A.numel() > 0 else max(K, 1)
    s = _stream(stream)
    check(lib().bsk_dense_to_bsr_pattern(_ptr(A), lda, eb, M, K, bs, _ptr(row_ptr), ib, _ptr(ws), ws.numel(),
                                         ctypes.byref(nnzb), ctypes.byref(nnz), s), "bsk_dense_to_bsr_pattern")
    col_idx = torch.empty(nnzb.value, dtype=index_dtype, device=A.device)
    values = torch.empty(nnzb.value, bs, bs, dtype=A.dtype, device=A.device)
    check(lib().bsk_dense_to_bsr_fill(_ptr(A), lda, eb, M, K, bs, _ptr(row_ptr), _ptr(col_idx), ib, _ptr(values),
                                      nnzb.value, _ptr(ws), ws.numel(), s), "bsk_dense_to_bsr_fill")
    return row_ptr, col_idx, values, nnz.value


def csr_to_bsr(crow, col, vals, shape, bs: int, index_dtype=None, stream=None):
    """Device CSR (crow [M+1], col [nnz], vals [nnz]) of `shape` (M, K) -> (row_ptr, col_idx, values, nnz_elems),
    the result of to_dense().to_sparse_bsr((bs, bs)). Synchronises the stream once."""
    import torch

    index_dtype = torch.int64 if index_dtype is None else index_dtype
    ib = _index_bytes(index_dtype)
    ib_in = _index_bytes(crow.dtype)
    if col.dtype != crow.dtype:
        raise ValueError("crow and col indices must have one dtype")
    M, K = shape
    nnz_in = vals.numel()
    eb = vals.element_size()
    dev = vals.device
    ws = torch.empty(bsr_convert_workspace_bytes(M, K, bs), dtype=torch.uint8, device=dev)
    row_ptr = torch.empty(M // bs + 1, dtype=index_dtype, device=dev)
    nnzb, nnz = ctypes.c_int64(0), ctypes.c_int64(0)
    s = _stream(stream)
    check(lib().bsk_csr_to_bsr_pattern(_ptr(crow), _ptr(col), ib_in, _ptr(vals), eb, nnz_in, M, K, bs, _ptr(row_ptr),
                                       ib, _ptr(ws), ws.numel(), ctypes.byref(nnzb), ctypes.byref(nnz), s),
          "bsk_csr_to_bsr_pattern")
    col_idx = torch.empty(nnzb.value, dtype=index_dtype, device=dev)
    values = torch.empty(nnzb.value, bs, bs, dtype=vals.dtype, device=dev)
    check(lib().bsk_csr_to_bsr_fill(_ptr(crow), _ptr(col), ib_in, _ptr(vals), eb, nnz_in, M, K, bs, _ptr(row_ptr),
                                    _ptr(col_idx), ib, _ptr(values), nnzb.value, _ptr(ws), ws.numel(), s),
          "bsk_csr_to_bsr_fill")
    return row_ptr, col_idx, values, nnz.value


def dense_to_bsr_bounded(A, bs: int, row_ptr, col_idx, values, workspace, stream=None) -> None:
    """Single-call dense -> BSR into preallocated outputs (capacity = len(col_idx) blocks); no host sync.
    row_ptr[-1] holds the true block count once the stream gets there."""
    M, K = A.shape
    cap = col_idx.numel()
    if values.shape[0] < cap:
        raise ValueError("values must hold as many blocks as col_idx")
    check(lib().bsk_dense_to_bsr_bounded(_ptr(A), A.stride(0) if A.numel() else max(K, 1), A.element_size(), M, K, bs,
                                         _ptr(row_ptr), _ptr(col_idx), _index_bytes(col_idx.dtype), _ptr(values), cap,
                                         _ptr(workspace), workspace.numel(), _stream(stream)),
          "bsk_dense_to_bsr_bounded")


def csr_to_bsr_bounded(crow, col, vals, shape, bs: int, row_ptr, col_idx, values, workspace, stream=None) -> None:
    """Single-call CSR -> BSR into preallocated outputs (capacity = len(col_idx) blocks); no host sync."""
    M, K = shape
    cap = col_idx.numel()
    if values.shape[0] < cap:
        raise ValueError("values must hold as many blocks as col_idx")
    check(lib().bsk_csr_to_bsr_bounded(_ptr(crow), _ptr(col), _index_bytes(crow.dtype), _ptr(vals),
                                       vals.element_size(), vals.numel(), M, K, bs, _ptr(row_ptr), _ptr(col_idx),
                                       _index_bytes(col_idx.dtype), _ptr(values), cap, _ptr(workspace),
                                       workspace.numel(), _stream(stream)), "bsk_csr_to_bsr_bounded")


def _attn_dtype(t) -> int:
    import torch

    if t.dtype == torch.bfloat16:
        return 0
    if t.dtype == torch.float16:
        return 1
    raise ValueError("attention tensors must be bfloat16 or float16")


def bsattn_fwd_ex(Q, K, V, O, lse, row_ptr, col_idx, scale: float, causal_diag: bool = True, bh_begin: int = 0,
                  bh_end: int | None = None, blk: int = 128, stream=None) -> None:
    """Forward (bf16 or fp16 by Q's dtype) that also writes the natural-log LSE per query row (lse may be None)."""
    B, H, S, D = Q.shape
    bh_end = B * H if bh_end is None else bh_end
    check(lib().bsk_bsattn_fwd_ex(_attn_dtype(Q), _ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(lse), _ptr(row_ptr),
                                  _ptr(col_idx), B, H, S, D, blk, float(scale), int(bool(causal_diag)), bh_begin,
                                  bh_end, _stream(stream)), "bsk_bsattn_fwd_ex")


def bsattn_mask_transpose(row_ptr, col_idx, pairs: int, nqb: int, stream=None):
    """(col_ptr, row_idx) int32 column lists of the block mask, on row_ptr's device."""
    import torch

    dev = row_ptr.device
    col_ptr = torch.empty(pairs * nqb + 1, dtype=torch.int32, device=dev)
    row_idx = torch.empty(max(col_idx.numel(), 1), dtype=torch.int32, device=dev)
    ws = torch.empty(pairs * nqb * 4 + 16, dtype=torch.uint8, device=dev)
    check(lib().bsk_bsattn_mask_transpose(_ptr(row_ptr), _ptr(col_idx), pairs, nqb, _ptr(col_ptr), _ptr(row_idx),
                                          _ptr(ws), ws.numel(), _stream(stream)), "bsk_bsattn_mask_transpose")
    return col_ptr, row_idx


def bsattn_bwd(dO, Q, K, V, O, lse, dQ, dK, dV, row_ptr, col_idx, col_ptr, row_idx, scale: float,
               causal_diag: bool = True, delta=None, blk: int = 128, stream=None) -> None:
    """Backward of the block-sparse attention into dQ, dK, dV (same shape and dtype as Q)."""
    import torch

    B, H, S, D = Q.shape
    if delta is None:  # per row: rowsum(dO * O) and -lse * log2(e)
        delta = torch.empty(2 * B * H * S, dtype=torch.float32, device=Q.device)
    elif delta.numel() < 2 * B * H * S:
        raise ValueError("delta scratch needs 2 * B * H * S floats")
    check(lib().bsk_bsattn_bwd(_attn_dtype(Q), _ptr(dO), _ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(lse), _ptr(dQ),
                               _ptr(dK), _ptr(dV), _ptr(row_ptr), _ptr(col_idx), _ptr(col_ptr), _ptr(row_idx), B, H, S,
                               D, blk, float(scale), int(bool(causal_diag)), _ptr(delta), _stream(stream)),
          "bsk_bsattn_bwd")


def device_error() -> int:
    """Read and clear the device error word (synchronises the device)."""
    w = ctypes.c_uint32(0)
    check(lib().bsk_device_error(ctypes.byref(w)), "bsk_device_error")
    return w.value


def set_wait_timeout_ns(ns: int) -> None:
    check(lib().bsk_set_wait_timeout_ns(int(ns)), "bsk_set_wait_timeout_ns")


def selftest_wait_timeout(ns: int, stream=None) -> int:
    """Returns the status code of the failure-detection probe (BSK_ERR_DEVICE_TIMEOUT is the expected one)."""
    return lib().bsk_selftest_wait_timeout(int(ns), _stream(stream))


def selftest_exp2(x, y, fma_pipe: bool, stream=None) -> None:
    """y = 2^x elementwise (fp32 device tensors) by the softmax's FMA-pipe polynomial or its MUFU route."""
    check(lib().bsk_selftest_exp2(_ptr(x), _ptr(y), x.numel(), int(bool(fma_pipe)), _stream(stream)),
          "bsk_selftest_exp2")


def bsr_validate_host(row_ptr, col_idx, Kb: int) -> None:
    """Validate a BSR index structure held in host (CPU, int32, contiguous) tensors."""
    Mb = row_ptr.numel() - 1
    nnzb = col_idx.numel()
    check(lib().bsk_bsr_validate_host(_ptr(row_ptr), _ptr(col_idx) if nnzb else None, Mb, Kb, nnzb),
          "bsk_bsr_validate_host")
