"""Multi-rank host logic on CPU ranks (gloo, world_size 2): every shard plan, computed with the oracle on each
rank's shard and reassembled with collectives, reproduces the unsharded oracle result; failures (a rank that
raises, a rank that never joins) end the job with an error on the host instead of a hang."""
import math
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_path as ref
from periodicdent42_b200 import sharding
from periodicdent42_b200 import workloads as wl

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=timeout_s))


def _worker_plans(rank, port, errq):
    try:
        _init(rank, port)
        torch.manual_seed(0)
        g = torch.Generator().manual_seed(11)
        # dense N-shard
        A = torch.randn(96, 128, generator=g).half()
        Bt = torch.randn(1000, 128, generator=g).half()
        n0, n1 = sharding.dense_nshard(1000, WORLD, rank)
        part = ref.dense_fp64(A, Bt[n0:n1])
        bufs = [None] * WORLD
        dist.all_gather_object(bufs, part)  # ragged shards: gathered as objects
        full = torch.cat(bufs, dim=1)
        assert torch.equal(full, ref.dense_fp64(A, Bt)), "N-shard reassembly"
        # dense split-K + reduce (gloo: all_reduce then keep the owned rows = reduce-scatter semantics)
        k0, k1 = sharding.dense_ksplit(128, WORLD, rank)
        partial = ref.dense_fp64(A[:, k0:k1], Bt[:, k0:k1])
        dist.all_reduce(partial)
        r0, r1 = sharding.splitk_rows(96, WORLD, rank)
        assert ref.normwise_rel_err(partial[r0:r1], ref.dense_fp64(A, Bt)[r0:r1]) < 1e-12, "split-K"
        # BSR block rows balanced by nnz
        crow, col = wl.bsr_pattern(7, 5, 2, g)
        vals = torch.randn(int(crow[-1]), 128, 128, generator=g).half()
        B = torch.randn(640, 64, generator=g).half()
        a, b = sharding.bsr_block_rows(crow, WORLD, rank)
        mine = ref.bsr_fp64(crow, col, vals, B, 7 * 128, 640, rows=slice(a, b))
        bufs = [None] * WORLD
        dist.all_gather_object(bufs, mine)
        assert torch.equal(torch.cat(bufs), ref.bsr_fp64(crow, col, vals, B, 7 * 128, 640)), "BSR rows"
        # attention (b,h) pairs balanced by nnz
        cfg = wl.AttnCfg(1, 3, 384, 128, 128, 2, 1, 4)
        q, k, v = wl.attn_inputs(cfg, "cpu")
        rp, ci = wl.attn_mask_bsr(cfg)
        p0, p1 = sharding.attn_pairs(rp, 3, 3, WORLD, rank)
        outs = []
        for p in range(3):
            o = torch.zeros(384, 128, dtype=torch.float64)
            if p0 <= p < p1:
                o = ref.attn_blocksparse_fp64(q[0, p], k[0, p], v[0, p], rp[p * 3:p * 3 + 4], ci[rp[p * 3]:rp[p * 3 + 3]],
                                              1 / math.sqrt(128), True)
            outs.append(o)
        mine = torch.stack(outs)
        dist.all_reduce(mine)  # disjoint pairs: the sum is the union
        for p in range(3):
            full = ref.attn_blocksparse_fp64(q[0, p], k[0, p], v[0, p], rp[p * 3:p * 3 + 4], ci[rp[p * 3]:rp[p * 3 + 3]],
                                             1 / math.sqrt(128), True)
            assert torch.equal(mine[p], full), f"attention pair {p}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))
        raise


def test_shard_plans_reassemble_to_the_unsharded_oracle():
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    mp.start_processes(_worker_plans, args=(port, errq), nprocs=WORLD, start_method="spawn", join=True)
    assert errq.empty()


def _worker_rank_raises(rank, port, resq):
    _init(rank, port, timeout_s=5)
    if rank == 1:
        dist.destroy_process_group()
        raise RuntimeError("rank 1 failed before its collective")
    t = torch.ones(4)
    try:
        dist.all_reduce(t)  # rank 1 never arrives
        resq.put("completed")
    except Exception as e:  # noqa: BLE001  (gloo raises on timeout / closed peer)
        resq.put(f"error: {type(e).__name__}")


def test_rank_that_raises_ends_the_collective_with_an_error():
    ctx = mp.get_context("spawn")
    resq = ctx.Queue()
    port = _free_port()
    with pytest.raises(Exception):
        mp.start_processes(_worker_rank_raises, args=(port, resq), nprocs=WORLD, start_method="spawn", join=True)
    msg = resq.get(timeout=60)
    assert msg.startswith("error"), msg


def _worker_never_joins(rank, port, resq):
    if rank == 1:
        return  # never initialises the process group
    try:
        _init(rank, port, timeout_s=3)
        resq.put("joined")
    except Exception as e:  # noqa: BLE001  (rendezvous times out)
        resq.put(f"error: {type(e).__name__}")


def test_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    resq = ctx.Queue()
    port = _free_port()
    mp.start_processes(_worker_never_joins, args=(port, resq), nprocs=WORLD, start_method="spawn", join=True)
    msg = resq.get(timeout=60)
    assert msg.startswith("error"), msg


@pytest.mark.parametrize("M,world", [(8192, 8), (10, 4), (2, 4), (301, 2), (1, 1), (0, 3)])
def test_host_rows_cover_m_contiguously(M, world):
    from periodicdent42_b200.dist import host_rows

    spans = [host_rows(M, world, r) for r in range(world)]
    mr = spans[0][2]
    assert all(s[2] == mr for s in spans) and mr * world >= M
    assert spans[0][0] == 0 and spans[-1][1] == M
    for r in range(world):
        r0, r1, _ = spans[r]
        assert r0 == min(r * mr, M) and 0 <= r1 - r0 <= mr  # rank r's real rows sit at the start of its block
        if r:
            assert r0 == spans[r - 1][1]
