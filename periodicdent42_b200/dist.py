"""Multi-GPU dense GEMM: K split across ranks with the reduce-scatter fused into the GEMM kernel
(SplitKReduceScatterGemm), and the N-sharded GEMM fed from host memory (HostShardedGemm).

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
        strm = _as_stream(stream, A.device)
        s = strm.cuda_stream
        lib = _capi.lib()
        if k1 > k0:
            _capi.check(lib.bsk_gemm_f16f32_splitk_scatter(A.data_ptr(), A.stride(0), Bt.data_ptr(), Bt.stride(0), M, N,
                                                           K, k0, k1, self.world, self.rank, self._tables[b], self.ld,
                                                           s), "bsk_gemm_f16f32_splitk_scatter")
        else:  # no K for this rank: its slot in every owner's buffer must still be defined
            raise ValueError("K too small to give every rank a non-empty K range")
        # The barrier goes on the GEMM's stream: NCCL then starts only after this rank's peer stores were issued
        # and completed, and the slot sum below (same stream) starts only after every rank's have.
        with torch.cuda.stream(strm):
            dist.all_reduce(self._flag, group=self.group)
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


def _as_stream(stream, device) -> torch.cuda.Stream:
    """The torch stream object for `stream`: None = the current stream of `device`, an int = a raw cudaStream_t
    handle (wrapped, not owned), else a torch.cuda.Stream."""
    if stream is None:
        return torch.cuda.current_stream(device)
    if isinstance(stream, int):
        return torch.cuda.ExternalStream(stream, device=device)
    return stream


def host_rows(M: int, world: int, rank: int) -> tuple[int, int, int]:
    """Rows of A that `rank` stages from host memory in HostShardedGemm: (r0, r1, rows_per_rank). Every rank
    owns a padded block of rows_per_rank = ceil(M / world) rows of the gathered chunk; the last blocks may hold
    fewer (or no) real rows."""
    mr = -(-M // world)
    r0 = min(rank * mr, M)
    return r0, min(r0 + mr, M), mr


class HostShardedGemm:
    """C[:, n0:n1] = A @ B[:, n0:n1] on every rank, fp16 A [M, K] and B^T [N, K] in HOST memory (each rank holds
    its own host copy of A and its shard B^T[n0:n1]; page-locked for overlap), fp32 result to host.

    N-sharding needs all of A on every GPU. Instead of every rank pulling all of A over its own PCIe link, K is
    streamed in chunks and, per chunk, each rank copies only its 1/world slice of A's rows (plus its own B^T
    rows) and an NCCL all-gather over NVLink assembles the full A chunk on every GPU, so a rank's PCIe traffic
    is (M / world + N / world) x K x 2 bytes rather than (M + N / world) x K x 2. Chunk i+1's copies and gather
    overlap the tensor-core work on chunk i (bsk_gemm_f16f32 for the first chunk, bsk_gemm_f16f32_acc after).
    Collectives are issued in the same order on every rank; world = 1 degenerates to the host-streaming GEMM
    without the gather."""

    def __init__(self, M: int, N_local: int, K: int, k_chunk: int = 0, group=None, device=None):
        import torch.cuda

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.M, self.N, self.K = M, N_local, K
        self.kc = _capi.gemm_host_chunk(K, k_chunk)
        self.r0, self.r1, self.mr = host_rows(M, self.world, self.rank)
        rows = self.mr * self.world
        self.abuf = [torch.empty(rows * self.kc, dtype=torch.float16, device=self.dev) for _ in range(2)]
        # this rank's slice lands in `stage` and is gathered from there into every rank's `abuf`
        self.stage = ([torch.empty(self.mr * self.kc, dtype=torch.float16, device=self.dev) for _ in range(2)]
                      if self.world > 1 else None)
        self.bbuf = [torch.empty(max(N_local, 1) * self.kc, dtype=torch.float16, device=self.dev) for _ in range(2)]
        self.ldc = (N_local + 3) // 4 * 4
        self.C = torch.empty(M, self.ldc, dtype=torch.float32, device=self.dev)
        self.copy_stream = torch.cuda.Stream(self.dev)
        self.freed = [torch.cuda.Event() for _ in range(2)]

    def __call__(self, A_h: torch.Tensor, Bt_h: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        M, N, K, kc = self.M, self.N, self.K, self.kc
        if tuple(A_h.shape) != (M, K) or tuple(Bt_h.shape) != (N, K) or tuple(out.shape) != (M, N):
            raise ValueError("HostShardedGemm: operand shapes differ from the ones it was built for")
        for t in (A_h, Bt_h, out):
            if t.is_cuda or t.stride(1) != 1:
                raise ValueError("HostShardedGemm: host tensors with unit column stride required")
        if A_h.dtype != torch.float16 or Bt_h.dtype != torch.float16 or out.dtype != torch.float32:
            raise ValueError("HostShardedGemm: fp16 A, B^T and fp32 out required")
        s = torch.cuda.current_stream(self.dev) if stream is None else stream
        cs = self.copy_stream
        cs.wait_stream(s)  # earlier work on `s` (a previous call still reading the buffers) precedes the copies
        nchunks = (K + kc - 1) // kc if K else 0
        for i in range(nchunks):
            b = i & 1
            k0 = i * kc
            kw = min(kc, K - k0)
            if i >= 2:
                cs.wait_event(self.freed[b])
            a_dst = self.stage[b].data_ptr() if self.world > 1 else self.abuf[b].data_ptr()
            _capi.copy_2d_async(a_dst, kc * 2, A_h.data_ptr() + (self.r0 * A_h.stride(0) + k0) * 2,
                                A_h.stride(0) * 2, kw * 2, self.r1 - self.r0, cs)
            _capi.copy_2d_async(self.bbuf[b].data_ptr(), kc * 2, Bt_h.data_ptr() + k0 * 2, Bt_h.stride(0) * 2,
                                kw * 2, N, cs)
            if self.world > 1:
                with torch.cuda.stream(cs):  # the gather starts after this rank's slice has landed
                    work = dist.all_gather_into_tensor(self.abuf[b], self.stage[b], group=self.group, async_op=True)
                with torch.cuda.stream(s):
                    work.wait()
            s.wait_stream(cs)
            A_view = self.abuf[b][:M * kc].view(M, kc)
            Bt_view = self.bbuf[b][:N * kc].view(N, kc)
            if N > 0:
                fn = _capi.gemm_f16f32 if i == 0 else _capi.gemm_f16f32_acc
                fn(A_view, Bt_view, self.C, 0, kw, stream=s)
            self.freed[b].record(s)
        if nchunks == 0:
            with torch.cuda.stream(s):
                self.C.zero_()
        _capi.copy_2d_async(out.data_ptr(), out.stride(0) * 4, self.C.data_ptr(), self.ldc * 4, N * 4, M, s)
        return out
