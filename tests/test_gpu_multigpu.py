"""Multi-GPU paths on 2 GPUs (child processes, one per GPU, NCCL), each rank's shard against the fp64 oracle:
the fused split-K GEMM + reduce-scatter (peer-memory epilogue; on the current stream and on an explicit side
stream), the N-sharded GEMM, the N-sharded GEMM fed from host memory (row slices staged per rank, NCCL
all-gather), the FP8 GEMM sharded by N, the BSR SpMM sharded by balanced block-row nnz and the block-sparse
attention sharded by (b,h) pairs -- the partitions the benchmark uses at N > 1. Tolerances: 1e-3 normwise for
fp16 inputs, 3e-2 for e4m3, the bf16 storage floor + 1e-3 for attention. Skipped with fewer than 2 GPUs."""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _sharded_ops(rank, dev):
    """FP8 (N-shard), BSR (block-row shard) and attention ((b,h) shard) on this rank's part, as the benchmark
    partitions them; returns {name: (error, tolerance)}."""
    import math

    from oracle import reference_path as ref
    from periodicdent42_b200 import _capi, sharding
    from periodicdent42_b200 import workloads as wl

    out = {}
    g = torch.Generator().manual_seed(17)
    # FP8 e4m3 -> bf16, N-sharded
    M, N, K = 512, 1024, 2048
    Aq, sa = wl.quantize_e4m3(torch.randn(M, K, generator=g))
    Bqt, sb = wl.quantize_e4m3(torch.randn(N, K, generator=g))
    n0, n1 = sharding.dense_nshard(N, WORLD, rank)
    D = torch.full((M, n1 - n0), float("nan"), dtype=torch.bfloat16, device=dev)
    _capi.gemm_e4m3_bf16(Aq.to(dev), Bqt[n0:n1].contiguous().to(dev), sa.to(dev), sb.to(dev), D)
    torch.cuda.synchronize()
    out["fp8_nshard"] = (ref.normwise_rel_err(D.cpu(), ref.fp8_fp64(Aq, Bqt[n0:n1], sa, sb)), 3e-2)
    # BSR, balanced block-row shards (uneven nnz per row so the plan is not trivially half and half)
    Mb, Kb, Nn = 16, 16, 1024
    crow, col = wl.bsr_pattern(Mb, Kb, 4, g)
    keep = torch.cat([col[crow[r]:crow[r + 1]][: 1 + (r % 4)] for r in range(Mb)])
    counts = torch.tensor([1 + (r % 4) for r in range(Mb)])
    crow = torch.zeros(Mb + 1, dtype=torch.int64)
    crow[1:] = torch.cumsum(counts, 0)
    col = keep
    vals = torch.randn(col.numel(), 128, 128, generator=g).half()
    B = torch.randn(Kb * 128, Nn, generator=g).half()
    b0, b1 = sharding.bsr_block_rows(crow, WORLD, rank)
    C = torch.full((Mb * 128, Nn), float("nan"), device=dev)
    _capi.spmm_bsr_f16f32(crow.to(torch.int32).to(dev), col.to(torch.int32).to(dev), vals.to(dev), B.to(dev), C,
                          Mb * 128, b0, b1)
    torch.cuda.synchronize()
    c64 = ref.bsr_fp64(crow, col, vals, B, Mb * 128, Kb * 128, rows=slice(b0, b1))
    out["bsr_block_rows"] = (ref.normwise_rel_err(C[b0 * 128:b1 * 128].cpu(), c64), 1e-3)
    # block-sparse attention, (b,h) pairs balanced by nnz
    cfg = wl.AttnCfg(1, 4, 1024, 128, 128, 4, 8, 4)
    q, k, v = wl.attn_inputs(cfg, "cpu")
    rp, ci = wl.attn_mask_bsr(cfg)
    nqb, P = cfg.S // 128, cfg.B * cfg.H
    p0, p1 = sharding.attn_pairs(rp, nqb, P, WORLD, rank)
    O = torch.full(q.shape, float("nan"), dtype=q.dtype, device=dev)
    scale = 1.0 / math.sqrt(cfg.D)
    _capi.bsattn_fwd_bf16(q.to(dev), k.to(dev), v.to(dev), O, rp.to(torch.int32).to(dev),
                          ci.to(torch.int32).to(dev), scale, True, p0, p1)
    torch.cuda.synchronize()
    Oh = O.cpu()
    for p in range(p0, p1):
        r0, r1 = p * nqb, (p + 1) * nqb
        o64 = ref.attn_blocksparse_fp64(q[0, p], k[0, p], v[0, p], rp[r0:r1 + 1], ci[rp[r0]:rp[r1]], scale, True)
        out[f"attn_pair_{p}"] = (ref.normwise_rel_err(Oh[0, p], o64), ref.bf16_storage_floor(o64) + 1e-3)
    out["attn_pairs_owned"] = (0.0 if p1 > p0 else 1.0, 0.5)
    return out


def _worker(rank, port, q):
    try:
        import torch.distributed as dist

        from oracle import reference_path as ref
        from periodicdent42_b200 import _capi, sharding
        from periodicdent42_b200.dist import HostShardedGemm, SplitKReduceScatterGemm

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60), device_id=dev)
        g = torch.Generator().manual_seed(5)
        M, N, K = 512, 1024, 8192
        A = torch.randn(M, K, generator=g).half()
        Bt = torch.randn(N, K, generator=g).half()
        Ad, Btd = A.to(dev), Bt.to(dev)
        full64 = ref.dense_fp64(A, Bt)
        errs = {}
        op = SplitKReduceScatterGemm(M, N)
        r0, r1 = rank * M // WORLD, (rank + 1) * M // WORLD
        for call in range(3):  # odd and even calls use the two receive buffers
            shard = op(Ad, Btd)
            torch.cuda.synchronize()
            errs[f"splitk_rs_{call}"] = ref.normwise_rel_err(shard.cpu(), full64[r0:r1])
        # an explicit side stream (object and raw handle): the barrier and the slot sum follow the GEMM on it
        side = torch.cuda.Stream(dev)
        outs = [torch.full((M // WORLD, N), float("nan"), device=dev) for _ in range(3)]
        side.wait_stream(torch.cuda.current_stream(dev))
        for call in range(3):
            op(Ad, Btd, outs[call], stream=side if call != 1 else side.cuda_stream)
        side.synchronize()
        for call in range(3):
            errs[f"splitk_rs_side_stream_{call}"] = ref.normwise_rel_err(outs[call].cpu(), full64[r0:r1])
        op.close()
        errs.update(_sharded_ops(rank, dev))
        n0, n1 = sharding.dense_nshard(N, WORLD, rank)
        C = torch.empty(M, n1 - n0, device=dev)
        _capi.gemm_f16f32(Ad, Btd[n0:n1], C)
        torch.cuda.synchronize()
        errs["nshard"] = ref.normwise_rel_err(C.cpu(), full64[:, n0:n1])
        # host-resident operands: each rank stages half of A's rows per K chunk, NCCL gathers the chunk
        A_h, Bt_h = A.pin_memory(), Bt[n0:n1].contiguous().pin_memory()
        C_h = torch.empty(M, n1 - n0, pin_memory=True)
        hsg = HostShardedGemm(M, n1 - n0, K, k_chunk=1024)
        for call in range(2):
            C_h.fill_(float("nan"))
            hsg(A_h, Bt_h, C_h)
            torch.cuda.synchronize()
            errs[f"host_sharded_{call}"] = ref.normwise_rel_err(C_h, full64[:, n0:n1])
        # ragged: M not divisible by the world size, K not a multiple of the chunk
        Mr, Kr = 301, 3000
        hs2 = HostShardedGemm(Mr, n1 - n0, Kr, k_chunk=512)
        C2 = torch.empty(Mr, n1 - n0, pin_memory=True)
        hs2(A_h[:Mr, :Kr], Bt_h[:, :Kr], C2)
        torch.cuda.synchronize()
        errs["host_sharded_ragged"] = ref.normwise_rel_err(C2, ref.dense_fp64(A[:Mr, :Kr], Bt[n0:n1, :Kr]))
        errs["device_error"] = _capi.device_error()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_splitk_reduce_scatter_and_nshard_on_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    for rank, res in results.items():
        assert isinstance(res, dict), f"rank {rank} failed:\n{res}"
        assert res["device_error"] == 0
        for k, v in res.items():
            if k == "device_error":
                continue
            err, tol = v if isinstance(v, tuple) else (v, 1e-3)
            assert err <= tol, (rank, k, err, tol)
