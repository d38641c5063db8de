"""Multi-GPU dense GEMM with K split across ranks and the reduce-scatter fused into the GEMM kernel.

One process per GPU (torchrun), a torch.distributed process group (NCCL) for rendezvous and a stream-ordered
barrier. Rank r computes the partial product over its K range; the GEMM's epilogue stores every partial row
straight into the receive buffer of the rank that owns the row (CUDA IPC peer memory over NVLink), so the
transfer overlaps the remaining tiles' tensor work. A one-element all-reduce on the current stream orders
"every rank's GEMM has completed" before each rank sums its `world` slots (fixed rank order: deterministic).
The receive buffers are double-buffered by call parity, so the next call's stores never race this call's sum.

This replaces the split-K + NCCL reduce-scatter plan of the dense GEMM (in the reference the multi-GPU layer
is only a roadmap item).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _capi
from . import sharding


class SplitKReduceScatterGemm:
    """C_shard[M/world, N] (fp32) of C = A @ B for fp16 A [M, K] and B^T [N, K] replicated on every rank."""

    def __init__(self, M: int, N: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one NVLink domain)")
        if M % self.world:
            raise ValueError(f"M ({M}) must be divisible by the world size ({self.world})")
        self.M, self.N = M, N
        self.rows = M // self.world
        self.ld = (N + 3) // 4 * 4
        nbytes = self.world * self.rows * self.ld * 4
        lib = _capi.lib()
        self._own = []
        handles = []
        for _ in range(2):
            p = ctypes.c_void_p()
            h = ctypes.create_string_buffer(64)
            _capi.check(lib.bsk_peer_buffer_alloc(nbytes, ctypes.byref(p), h), "bsk_peer_buffer_alloc")
            self._own.append(p.value)
            handles.append(h.raw)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        self._opened = []
        self._tables = []
        for b in range(2):
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._own[b])
                else:
                    q = ctypes.c_void_p()
                    _capi.check(lib.bsk_peer_buffer_open(gathered[r][b], ctypes.byref(q)), "bsk_peer_buffer_open")
                    self._opened.append(q.value)
                    ptrs.append(q.value)
            self._tables.append((ctypes.c_void_p * self.world)(*ptrs))
        self._flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))
        self._calls = 0

    def __call__(self, A: torch.Tensor, Bt: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        M, K = A.shape
        N = Bt.shape[0]
        if (M, N) != (self.M, self.N):
            raise ValueError(f"built for {self.M}x{self.N}, called with {M}x{N}")
        if out is None:
            out = torch.empty(self.rows, N, dtype=torch.float32, device=A.device)
        k0, k1 = sharding.dense_ksplit(K, self.world, self.rank)
        b = self._calls & 1
        s = _capi._stream(stream)
        lib = _capi.lib()
        if k1 > k0:
            _capi.check(lib.bsk_gemm_f16f32_splitk_scatter(A.data_ptr(), A.stride(0), Bt.data_ptr(), Bt.stride(0), M, N,
                                                           K, k0, k1, self.world, self.rank, self._tables[b], self.ld,
                                                           s), "bsk_gemm_f16f32_splitk_scatter")
        else:  # no K for this rank: its slot in every owner's buffer must still be defined
            raise ValueError("K too small to give every rank a non-empty K range")
        dist.all_reduce(self._flag, group=self.group)  # every rank's GEMM (and its peer stores) has completed
        _capi.check(lib.bsk_splitk_slots_reduce(self._own[b], self.world, self.rows, N, self.ld, out.data_ptr(),
                                                out.stride(0), s), "bsk_splitk_slots_reduce")
        self._calls += 1
        return out

    def close(self) -> None:
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still writes into a buffer that is about to go away
        lib = _capi.lib()
        for q in self._opened:
            lib.bsk_peer_buffer_close(q)
        self._opened = []
        for p in self._own:
            lib.bsk_peer_buffer_free(p)
        self._own = []
