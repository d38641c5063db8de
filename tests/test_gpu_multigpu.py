"""Multi-GPU paths on 2 GPUs (child processes, one per GPU, NCCL): the fused split-K GEMM + reduce-scatter
(peer-memory epilogue), the N-sharded GEMM and the N-sharded GEMM fed from host memory (row slices staged
per rank, NCCL all-gather), each rank's shard against fp64. Skipped with fewer than 2 GPUs."""
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
        op.close()
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
            if k != "device_error":
                assert v <= 1e-3, (rank, k, v)
