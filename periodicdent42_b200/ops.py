"""Operator API: the reference's ``blackwellsparsek`` functions (BlackwellSparseK/python/ops.py) re-pointed
at the sm_100a kernels, plus the operators the reference never exposed (dense GEMM, FP8 GEMM,
block-sparse attention).

Every operator runs through the torch extension ``periodicdent42_b200._C``, which calls the C ABI of
libbsk_sm100.so. There is no CPU fallback: CPU tensors raise ``ValueError`` (as the reference's
``sparse_mm`` does, ops.py:64-65) and a missing extension raises ``ImportError`` on first use.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _capi

from . import workloads as _wl

_C_MOD = None


def _C():
    global _C_MOD
    if _C_MOD is None:
        try:
            from . import _C as mod  # noqa: N814
        except ImportError as e:  # pragma: no cover - exercised on broken installs only
            raise ImportError(
                "periodicdent42_b200._C is not built: run `python -m periodicdent42_b200.build` "
                "(no CPU fallback exists for these operators)") from e
        _C_MOD = mod
    return _C_MOD


def has_cuda_ext() -> bool:
    """Whether the extension imports (the reference's HAS_CUDA_EXT, ops.py:13-22)."""
    try:
        _C()
        return True
    except ImportError:
        return False


KERNEL_BLOCK = 128  # block edge of the sm_100 BSR kernel (tcgen05 M = 128)


# ----------------------------------------------------------------------------------------- BSR SpMM
def sparse_mm(A: torch.Tensor, B: torch.Tensor, block_size: int = 16, autotune: bool = False) -> torch.Tensor:
    """C = A @ B for sparse A (BSR or CSR, fp16, CUDA) and B dense or BSR / CSR (fp16, CUDA); returns fp32 [M, N].

    Same signature and argument checks as the reference (BlackwellSparseK/python/ops.py:25-69).
    ``block_size`` and ``autotune`` keep their meaning for the tile-config dicts
    (``_default_config`` / ``_autotune_config``) but the sm_100 kernel always computes on 128x128 blocks:
    inputs in another layout (CSR, or BSR with another block size) are re-blocked on the device first.
    A B in BSR or CSR layout takes the BSR x BSR kernel (B's blocks looked up per A block, as the reference's
    sparse-B kernel path does, src/sparse_h100_async.cu:105-119); a COO B is rejected as in the reference.
    """
    if not A.is_sparse and A.layout not in (torch.sparse_csr, torch.sparse_bsr):
        raise ValueError("A must be a sparse tensor")
    if B.is_sparse:
        raise ValueError("B must be a dense tensor")
    if A.device != B.device:
        raise ValueError("A and B must be on the same device")
    if not A.is_cuda:
        raise ValueError("CUDA tensors required (CPU not supported)")
    M, K1 = A.shape
    K2, N = B.shape
    if K1 != K2:
        raise ValueError(f"Dimension mismatch: A is {M}×{K1}, B is {K2}×{N}")
    config = _autotune_config(M, N, K1) if autotune else _default_config(M, N, K1)
    A_bsr = _to_kernel_bsr(A)
    if B.dtype != torch.float16:
        raise ValueError("B must be float16")
    if autotune and B.layout == torch.strided:
        _ensure_tuned("spmm_bsr", M, N, K1, lambda: _tune_spmm(A_bsr, B.contiguous(), M))
    if B.layout in (torch.sparse_bsr, torch.sparse_csr):
        if N % KERNEL_BLOCK:
            raise ValueError(f"a sparse B needs N divisible by {KERNEL_BLOCK}, got {N}")
        B_bsr = _to_kernel_bsr(B)
        crow, col = B_bsr.crow_indices(), B_bsr.col_indices()
        if col.numel() == (K2 // KERNEL_BLOCK) * (N // KERNEL_BLOCK):  # every block stored: plain dense product
            Bc = B_bsr.to_dense()
        else:
            return _C().sparse_mm_bsr(A_bsr.crow_indices(), A_bsr.col_indices(), A_bsr.values(), crow, col,
                                      B_bsr.values(), M, N, K1, config["BM"], config["BN"], config["BK"])
    else:
        Bc = B.contiguous()
    dummy = torch.zeros(1, dtype=torch.int32, device=A.device)
    return _C().sparse_mm_bsr(A_bsr.crow_indices(), A_bsr.col_indices(), A_bsr.values(), dummy, dummy, Bc, M, N, K1,
                              config["BM"], config["BN"], config["BK"])


def _ensure_tuned(op: str, M: int, N: int, K: int, tune_fn) -> None:
    """Registers the cached launch configuration of (op, M, N, K) for this device, tuning (and caching) it on
    first use -- the reference's ``autotune=True`` switch, backed by measurements instead of size buckets."""
    from . import autotune as at

    if at.registered(op, M, N, K) is not None:
        return
    cache = at.AutotuneCache()
    e = cache.get(at.device_key(), at.shape_key(op, M, N, K))
    if e is not None:
        at.register(op, M, N, K, int(e["tile"]), int(e["group_m"]))
    else:
        tune_fn()


def _tune_spmm(A_bsr: torch.Tensor, B: torch.Tensor, M: int) -> None:
    from . import autotune as at

    rp = A_bsr.crow_indices().to(torch.int32)
    ci = A_bsr.col_indices().to(torch.int32)
    at.tune_spmm_bsr(rp, ci, A_bsr.values().contiguous(), B, M)


def _to_kernel_bsr(A: torch.Tensor) -> torch.Tensor:
    """BSR with 128x128 blocks, on A's device: CSR / COO input through the device converter; BSR with another
    block size re-blocked through its dense form (the reference left CSR -> BSR unimplemented,
    ops.py:193-197)."""
    if A.layout == torch.sparse_bsr and tuple(A.values().shape[1:]) == (KERNEL_BLOCK, KERNEL_BLOCK):
        return A
    if A.layout not in (torch.sparse_csr, torch.sparse_bsr, torch.sparse_coo):
        raise ValueError(f"Unsupported sparse layout: {A.layout}")
    M, K = A.shape
    if M % KERNEL_BLOCK or K % KERNEL_BLOCK:
        raise ValueError(f"A's shape must be a multiple of {KERNEL_BLOCK} in both dimensions, got {M}x{K}")
    return _convert_csr_to_bsr(A, KERNEL_BLOCK)


def _convert_csr_to_bsr(A_csr: torch.Tensor, block_size: int) -> torch.Tensor:
    """Sparse (CSR / COO / BSR) -> BSR with square blocks, keeping only blocks that hold a nonzero (the
    reference's stub, ops.py:193-197). On CUDA: CSR / COO by the device CSR converter, BSR of another block size
    by the device dense converter on its dense form; on the CPU through torch's dense form."""
    if A_csr.is_cuda and A_csr.dtype in (torch.float16, torch.bfloat16, torch.float32):
        from .utils import convert_to_bsr

        src = A_csr.to_dense() if A_csr.layout == torch.sparse_bsr else A_csr
        return convert_to_bsr(src, block_size, sparsity_threshold=0.0)
    return A_csr.to_dense().to_sparse_bsr((block_size, block_size))


def _default_config(M: int, N: int, K: int) -> dict:
    """Tile configuration dict of the reference (ops.py:200-206); the sm_100 kernel's own tile is
    128 x 256 with 128-wide K slabs, independent of these values."""
    return {"BM": 256, "BN": 128, "BK": 32}


def _autotune_config(M: int, N: int, K: int) -> dict:
    """Size-bucketed tile dict of the reference (ops.py:209-217); informational for the sm_100 kernel."""
    if M < 4096:
        return {"BM": 128, "BN": 64, "BK": 32}
    elif M < 16384:
        return {"BM": 256, "BN": 128, "BK": 32}
    return {"BM": 512, "BN": 256, "BK": 64}


def sparse_mm_benchmark(A: torch.Tensor, B: torch.Tensor,
                        implementations: Tuple[str, ...] = ("blackwellsparsek", "pytorch", "cutlass"),
                        num_iterations: int = 100, warmup_iterations: int = 5) -> dict:
    """Timing dict with the reference's keys (ops.py:123-190): ``blackwellsparsek_ms``,
    ``blackwellsparsek_tflops``, ``pytorch_ms``, ``pytorch_tflops``, ``speedup_vs_pytorch``.
    Times are CUDA-event times on the current stream. FLOPs = 2 * (stored nonzero values) * N: the
    reference's ``2 * A._nnz() * N`` counts blocks, not values, for BSR input. "cutlass" has no
    implementation on this path and is ignored."""
    M, K = A.shape
    _, N = B.shape
    nnz = A.values().numel()
    flops = 2 * nnz * N
    results = {}

    def _time(fn) -> float:
        for _ in range(warmup_iterations):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(num_iterations):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / num_iterations

    if "blackwellsparsek" in implementations:
        ms = _time(lambda: sparse_mm(A, B))
        results["blackwellsparsek_ms"] = ms
        results["blackwellsparsek_tflops"] = flops / (ms * 1e-3) / 1e12
    if "pytorch" in implementations:
        ms = _time(lambda: torch.sparse.mm(A, B))
        results["pytorch_ms"] = ms
        results["pytorch_tflops"] = flops / (ms * 1e-3) / 1e12
    if "blackwellsparsek_tflops" in results and "pytorch_tflops" in results:
        results["speedup_vs_pytorch"] = results["blackwellsparsek_tflops"] / results["pytorch_tflops"]
    return results


# ----------------------------------------------------------------------------------------- dense GEMM
def gemm(A: torch.Tensor, B: torch.Tensor, out_dtype: torch.dtype = torch.float32, k_range=None,
         split_k: Optional[int] = None, autotune: bool = False) -> torch.Tensor:
    """C = A @ B, fp16 inputs, fp32 output. A [M, K] row-major; B [K, N], column-major preferred
    (``B = Bt.t()`` with Bt contiguous costs nothing; a row-major B is transposed once). ``k_range``
    = (k_begin, k_end) restricts the contraction (split-K shards across ranks). ``split_k``: None = one pass;
    0 = split K across CTA pairs automatically when the output has too few tiles to fill the GPU; n > 0 =
    n splits (partials in a torch-allocated workspace, summed deterministically). ``autotune``: use the tuned
    tile / rasterisation for this shape (measured and cached on first use, see ``autotune``)."""
    _check_cuda_f16(A, B)
    if out_dtype != torch.float32:
        raise ValueError("gemm computes fp16 x fp16 -> fp32; out_dtype must be torch.float32")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"gemm: shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    A = A if A.stride(1) == 1 else A.contiguous()
    Bt = B.t()
    Bt = Bt if Bt.stride(1) == 1 else Bt.contiguous()
    if split_k is not None:
        if k_range is not None:
            raise ValueError("gemm: k_range and split_k are exclusive")
        return _C().gemm_f16f32_splitk(A, Bt, int(split_k))
    kb, ke = (0, -1) if k_range is None else k_range
    if autotune:
        from . import autotune as at

        M, K = A.shape
        kr = (K if ke < 0 else ke) - kb
        _ensure_tuned("gemm_f16f32", M, Bt.shape[0], kr, lambda: at.tune_gemm(M, Bt.shape[0], kr))
    return _C().gemm_f16f32(A, Bt, kb, ke)


def gemm_from_host(A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None, k_chunk: int = 0,
                   device=None, sync: bool = True) -> torch.Tensor:
    """C = A @ B for fp16 operands in HOST memory, fp32 result in host memory, computed on the GPU with the
    K dimension streamed in chunks: the PCIe copy of chunk i+1 overlaps the tensor-core work on chunk i and C
    accumulates on the device (the last chunk by row panels, each panel's C rows copied back while the next
    panel uploads). A [M, K] row-major; B [K, N], column-major preferred
    (``B = Bt.t()``). Use page-locked tensors (``pin_memory=True``) for A, B and ``out``: pageable memory works
    but its copies do not overlap. ``k_chunk``: K per chunk (multiple of 64), 0 = automatic. ``sync``: wait for
    the result (False leaves it pending on the current stream of ``device``)."""
    for t in (A, B):
        if t.is_cuda:
            raise ValueError("gemm_from_host takes host tensors (use gemm for device tensors)")
        if t.dtype != torch.float16:
            raise ValueError("float16 tensors required")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"gemm_from_host: shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    A = A if A.stride(1) == 1 else A.contiguous()
    Bt = B.t()
    Bt = Bt if Bt.stride(1) == 1 else Bt.contiguous()
    M, K = A.shape
    N = Bt.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, pin_memory=True)
    elif out.is_cuda or out.dtype != torch.float32 or tuple(out.shape) != (M, N) or out.stride(1) != 1:
        raise ValueError(f"out must be a host float32 [{M}, {N}] tensor with unit column stride")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        ws = torch.empty(_capi.gemm_host_workspace_bytes(M, N, K, k_chunk), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        _capi.gemm_f16f32_host(A, Bt, out, ws, k_chunk, stream)
        if sync:
            stream.synchronize()
    return out


def quantize_e4m3(x: torch.Tensor):
    """Per-tensor amax quantisation to e4m3: (x_q, scale) with scale = amax / 448, x_q = e4m3(x / scale)."""
    return _wl.quantize_e4m3(x)


def gemm_fp8(A_q: torch.Tensor, B_q: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
             out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """D = (A_q @ B_q) * scale_a * scale_b in bf16; A_q e4m3 [M, K] row-major, B_q e4m3 [K, N]
    (column-major preferred), per-tensor fp32 scales. Same semantics as
    ``torch._scaled_mm(A_q, B_q, scale_a, scale_b, out_dtype=torch.bfloat16)``."""
    if not (A_q.is_cuda and B_q.is_cuda):
        raise ValueError("CUDA tensors required (CPU not supported)")
    if out_dtype != torch.bfloat16:
        raise ValueError("gemm_fp8 produces bfloat16")
    Bt = B_q.t()
    Bt = Bt if Bt.stride(1) == 1 else Bt.contiguous()
    A = A_q if A_q.stride(1) == 1 else A_q.contiguous()
    sa = scale_a.to(device=A.device, dtype=torch.float32).reshape(1)
    sb = scale_b.to(device=A.device, dtype=torch.float32).reshape(1)
    return _C().gemm_e4m3(A, Bt, sa, sb)


def _check_cuda_f16(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("CUDA tensors required (CPU not supported)")
        if t.dtype != torch.float16:
            raise ValueError("float16 tensors required")


# ----------------------------------------------------------------------------------------- attention
def attention_forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: Optional[float] = None,
                      block_mask=None, block_size: int = 128, causal: bool = False) -> torch.Tensor:
    """O = softmax(scale * Q K^T) V, optionally restricted to a 128x128 block mask.

    Keeps the reference's signature ``attention_forward(Q, K, V, scale=None)``
    (.archive/src_experiments/blackwell_sparsek/__init__.py:52-109) and its checks (CUDA, 4-D, equal
    shapes, fp16, D in {64, 128}), and also accepts bf16; S must be a multiple of 128.
      block_mask: None (all blocks), a bool tensor [S/128, S/128] shared by every (b, h) or
                  [B, H, S/128, S/128], or a BSR tuple (row_ptr, col_idx) over the B*H*(S/128) block
                  rows (pairs in (b, h) order, within-sequence block indices).
      causal:     mask the diagonal block elementwise-causally; with block_mask=None it also restricts
                  to the lower-triangular blocks (standard causal attention).
    """
    if not (Q.is_cuda and K.is_cuda and V.is_cuda):
        raise ValueError("All tensors must be on CUDA device")
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise ValueError("All tensors must be 4D [B, H, S, D]")
    Bsz, H, S, D = Q.shape
    if K.shape != (Bsz, H, S, D) or V.shape != (Bsz, H, S, D):
        raise ValueError("Q, K, V must have the same shape")
    if Q.dtype not in (torch.float16, torch.bfloat16) or K.dtype != Q.dtype or V.dtype != Q.dtype:
        raise ValueError("All tensors must be FP16 (torch.float16) or all BF16 (torch.bfloat16)")
    if D not in (64, 128):
        raise ValueError(f"Head dimension must be 64 or 128, got {D}")
    if block_size != 128:
        raise ValueError("block_size must be 128")
    if S % 128:
        raise ValueError(f"Sequence length must be a multiple of 128, got {S}")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    row_ptr, col_idx = block_mask_to_bsr(block_mask, Bsz, H, S // 128, causal, Q.device)
    if torch.is_grad_enabled() and (Q.requires_grad or K.requires_grad or V.requires_grad):
        return _BlockSparseAttention.apply(Q, K, V, row_ptr, col_idx, float(scale), bool(causal))
    return _C().bsattn_fwd(Q, K, V, row_ptr, col_idx, float(scale), bool(causal))


class _BlockSparseAttention(torch.autograd.Function):
    """Autograd for block-sparse attention on the sm_100 kernels: the forward also keeps the row log-sum-exp,
    the backward recomputes the scores block by block (dK/dV per key block, dQ per query block). Replaces the
    reference's SparseKAttentionFunction (.archive/.../kernels/sparsek.py:100-142), whose CUDA backward was a
    stub."""

    @staticmethod
    def forward(ctx, Q, K, V, row_ptr, col_idx, scale, causal):
        Qc, Kc, Vc = Q.contiguous(), K.contiguous(), V.contiguous()
        B, H, S, _ = Qc.shape
        O = torch.empty_like(Qc)
        lse = torch.empty(B * H * S, dtype=torch.float32, device=Qc.device)
        _capi.bsattn_fwd_ex(Qc, Kc, Vc, O, lse, row_ptr, col_idx, scale, causal)
        ctx.save_for_backward(Qc, Kc, Vc, O, lse, row_ptr, col_idx)
        ctx.scale, ctx.causal = scale, causal
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, lse, row_ptr, col_idx = ctx.saved_tensors
        B, H, S, _ = Q.shape
        col_ptr, row_idx = _capi.bsattn_mask_transpose(row_ptr, col_idx, B * H, S // 128)
        dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
        _capi.bsattn_bwd(dO.to(Q.dtype).contiguous(), Q, K, V, O, lse, dQ, dK, dV, row_ptr, col_idx, col_ptr,
                         row_idx, ctx.scale, ctx.causal)
        return dQ, dK, dV, None, None, None, None


def block_mask_to_bsr(block_mask, B: int, H: int, nqb: int, causal: bool, device):
    """Normalise the accepted block-mask forms to (row_ptr, col_idx) int32 on `device`."""
    if isinstance(block_mask, tuple):
        rp, ci = block_mask
        return rp.to(device=device, dtype=torch.int32), ci.to(device=device, dtype=torch.int32)
    if block_mask is None:
        m = torch.ones(nqb, nqb, dtype=torch.bool)
        if causal:
            m = torch.tril(m)
        block_mask = m
    m = block_mask.to("cpu", torch.bool)
    if m.dim() == 2:
        if m.shape != (nqb, nqb):
            raise ValueError(f"block_mask must be [{nqb}, {nqb}]")
        crow, col = _wl.mask_to_bsr(m)
        P = B * H
        nnz = crow[-1]
        row_ptr = torch.cat([crow[:-1] + p * nnz for p in range(P)] + [torch.tensor([P * nnz])])
        col_idx = col.repeat(P)
    elif m.dim() == 4:
        if m.shape != (B, H, nqb, nqb):
            raise ValueError(f"block_mask must be [{B}, {H}, {nqb}, {nqb}]")
        crow, col = _wl.mask_to_bsr(m.reshape(B * H * nqb, nqb))
        row_ptr, col_idx = crow, col
    else:
        raise ValueError("block_mask must be 2-D or 4-D")
    return row_ptr.to(device=device, dtype=torch.int32), col_idx.to(device=device, dtype=torch.int32)


def synchronize_and_check() -> None:
    """Synchronise and raise if any kernel recorded a device-side error (bounded-wait timeout or an
    out-of-range BSR index)."""
    word = _C().device_error()
    if word:
        kind = {1: "device wait timed out", 2: "out-of-range index"}.get(word & 0xFF, "device error")
        raise RuntimeError(f"{kind} (error word 0x{word:08x})")
