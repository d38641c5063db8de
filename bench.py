#!/usr/bin/env python
"""Benchmark of the BlackwellSparseK operator family on B200.

Headline (the JSON line's metric/value): dense fp16 x fp16 -> fp32 GEMM, M = N = 8192, K = 237568,
A row-major, B column-major, entries N(0,1)/K^(1/4) from seed 1, TFLOPS for the whole job.
The line also carries the other three operators at their workloads under "ops":
  fp8   e4m3 GEMM 8192 x 8192 x 16384, per-tensor scales, bf16 out
  bsr   BSR SpMM 8192^3, 128x128 blocks, 16 nonzero blocks per block-row (nonzero-block FLOPs)
  attn  block-sparse attention fwd B=2, H=32, S=16384, D=128, sliding window 4 + 8 random blocks
Multi-GPU (torchrun, one rank per GPU, NCCL): total work is fixed ("scaling": "strong"):
  dense / fp8 sharded by N (no communication), bsr by balanced block-row nnz, attn by (b,h) pairs.
  ``--dense-mode splitk`` shards the dense GEMM by K and reduces with reduce_scatter instead.
The reference arm (``--impl reference``) times the reference's CPU torch path on the host cores.

Timing: W warm-up steps, then K steps between a barrier + synchronize on both sides, CUDA events on the
launching stream, max over ranks. Inputs (7.8 GB for the headline) are far larger than L2.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from periodicdent42_b200 import _capi  # noqa: E402
from periodicdent42_b200 import sharding  # noqa: E402
from periodicdent42_b200 import workloads as wl  # noqa: E402

METRIC = "fp16/fp8 GEMM & BSR TFLOPS per B200, % tensor peak, 1-8 GPU scaling"
UNIT = "TFLOPS"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------------------------------- plumbing
def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--ops", default="dense,fp8,bsr,attn,attn_bwd,convert,bsr_bsr",
                   help="comma list; dense is the headline; opt-in: autotune, cublas (same-box library yardstick)")
    p.add_argument("--dense-mode", choices=["nshard", "splitk", "splitk_nccl"], default="nshard",
                   help="nshard: N-sharded, no communication; splitk: K split across ranks, reduce-scatter fused "
                        "into the GEMM (peer-memory epilogue); splitk_nccl: K split + NCCL reduce_scatter")
    p.add_argument("--shape", default=None, help="M,N,K override of the dense GEMM (profiling a small case)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--tune-cache-out", default=None, metavar="PATH",
                   help="write the autotune op's results as a cache file at PATH")
    p.add_argument("--e2e-k-chunk", type=int, default=0, help="K per streamed chunk of the e2e GEMM (0 = auto)")
    p.add_argument("--nshard-k-splits", type=int, default=0,
                   help="K splits of each rank's N-shard GEMM (0 = automatic: nshard_k_splits)")
    p.add_argument("--op-steps", type=int, default=20,
                   help="timed steps of the fp8 / bsr / attn / ... measurements: short regions (~5-40 ms) that run "
                        "at the full clock, like the burst peak they are compared with (100 steps: the clock sags "
                        "under the load and FP8 / attention read 7-8 %% lower)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    return p.parse_args()


class Ctx:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None
        self.stream = None

    def init_gpu(self):
        # NCCL prints a version banner on stdout at INFO/VERSION level; the bench's stdout is one JSON line.
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        torch.cuda.set_device(self.local_rank)
        self.dev = torch.device("cuda", self.local_rank)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)
        self.stream = torch.cuda.current_stream()

    def barrier(self):
        if self.world > 1:
            dist.barrier(device_ids=[self.local_rank])

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1 and dist.is_initialized():
            dist.destroy_process_group()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes of each kernel from the committed ncu summaries (profiles/traffic.json)."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


class Clocks:
    """SM clock, power and clock-event reasons of the GPUs in use, sampled every ~10 ms from a thread through NVML
    (queries only; falls back to `nvidia-smi -lms 100` when NVML cannot be loaded). Each timed region records its
    host-time window; summaries are taken over the samples inside a window, so even a ~50 ms region (the 8-GPU
    headline) gets a handful of samples. The headline summary falls back to all samples under load only when its
    window holds fewer than 3."""
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_indices, period_s: float = 0.01):
        self.idx = sorted(set(gpu_indices))
        self.period = period_s
        self.windows = {}
        self.rows = []  # (time, gpu, sm_mhz, max_mhz, power_w, {reason: bool})
        self.source = None
        self._stop = None
        self._thread = None
        self._proc = None
        self._path = os.path.join("/tmp", f"bsk_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [(i, pynvml.nvmlDeviceGetHandleByIndex(i)) for i in self.idx]
            maxes = {i: pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for i, h in handles}
        except Exception:  # noqa: BLE001 - no NVML: the nvidia-smi sampler instead
            self._start_smi()
            return
        import threading

        self.source = "nvml"
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                for i, h in handles:
                    try:
                        t = time.time()
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:  # noqa: BLE001
                        continue
                    self.rows.append((t, i, float(sm), float(maxes[i]), pw,
                                      {n: bool(rs & b) for n, b in self.REASONS}))
                self._stop.wait(self.period)
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def _start_smi(self):
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                           "-lms", "100"], stdout=open(self._path, "w"), stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi"
        except OSError:
            self._proc = None

    def _read_smi(self):
        import datetime as _dt

        def f(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")
        with open(self._path) as fh:
            for line in fh:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 10:
                    continue
                try:
                    gpu = int(p[1])
                    ts = _dt.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                if gpu in self.idx:
                    self.rows.append((ts, gpu, f(p[2]), f(p[3]), f(p[4]),
                                      {n: v.lower().startswith("active") for (n, _), v in zip(self.REASONS, p[6:10])}))
        os.unlink(self._path)

    def mark(self, name, t0, t1):
        self.windows[name] = (t0, t1)

    @staticmethod
    def summary(rows):
        reasons = sorted({n for r in rows for n, on in r[5].items() if on})
        sm = [r[2] for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm), "sm_max_mhz": max(r[3] for r in rows),
                "power_w_max": max(r[4] for r in rows), "power_w_median": statistics.median(r[4] for r in rows),
                "samples": len(rows), "reasons": reasons}

    def stop(self, headline="dense"):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._read_smi()
        rows = self.rows
        if not rows:
            return None
        out = {}
        for name, (t0, t1) in self.windows.items():
            win = [x for x in rows if t0 <= x[0] <= t1]
            if win:
                out[name] = self.summary(win)
        head = out.get(headline)
        if head is None or head["samples"] < 3:
            load = [x for x in rows if x[4] > 200.0] or rows
            head = dict(self.summary(load), window="all samples under load")
        else:
            head = dict(head, window=f"{headline} timed region")
        head["source"] = self.source
        head["per_region"] = out
        return head


CLOCKS = None


def time_region(ctx: Ctx, fn, steps: int, warmup: int, name: str = ""):
    """Warm-up, then `steps` calls between barrier+synchronize; returns (max-over-ranks ms per step)."""
    for _ in range(warmup):
        fn()
    ctx.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(ctx.stream)
    for _ in range(steps):
        fn()
    e.record(ctx.stream)
    torch.cuda.synchronize()
    if CLOCKS is not None and name:
        CLOCKS.mark(name, t0, time.time())
    ctx.barrier()
    return ctx.max(s.elapsed_time(e) / steps)


# ----------------------------------------------------------------------------------------- output self-checks
# After each timed region, every rank checks a sample of its own output against an fp64 recompute on the device
# (rows and columns drawn from a fixed seed; the max error over ranks is reported), so the 2-8 GPU runs carry
# evidence that the sharded results are right, not only fast.
def _rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.double(), ref.double()
    den = torch.linalg.vector_norm(r).item()
    return torch.linalg.vector_norm(o - r).item() / den if den > 0 else torch.linalg.vector_norm(o).item()


def _pick(n: int, k: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.sort(torch.randperm(n, generator=g)[:min(k, n)]).values


def _check_entry(ctx: Ctx, err: float, tol: float, sample: str) -> dict:
    err = ctx.max(err)
    return {"err": err, "tol": tol, "ok": bool(err <= tol), "sample": sample, "ranks": ctx.world,
            "reference": "fp64 recompute on the device"}


# ----------------------------------------------------------------------------------------- dense GEMM
def nshard_k_splits(M: int, n_local: int, K: int, sm_count: int) -> int:
    """K splits for one rank's N-shard of the headline GEMM: 2 when the shard has at least two waves of 256 x 512
    tiles on the CTA pairs and splitting K in two fills the last wave markedly better (the 2-rank shard
    8192 x 4096: 256 tiles on 74 pairs fill 86.5 % of the pairs' slots, 512 (tile, split) units 98.8 %; measured
    1208 vs 1146 TFLOPS on one B200), else 1. Narrower shards measured no gain (8192 x 2048 with 4 splits) or a
    loss (8192 x 1024 with 8), and long K is needed so each split keeps the long-K raster."""
    pairs = max(1, sm_count // 2)
    tiles = -(-M // 256) * -(-n_local // 512)
    fill = lambda units: units / (-(-units // pairs) * pairs)  # noqa: E731
    if tiles >= 2 * pairs and K >= 2 * 65536 and fill(2 * tiles) >= fill(tiles) + 0.05:
        return 2
    return 1


def bench_cublas_dense(ctx: Ctx, args, res: dict):
    """Same-box yardstick, opt-in (`--ops dense,cublas`): the library GEMM (cuBLAS through torch.matmul, fp16 in,
    fp16 out) on the dense workload's shape and inputs. Not the product path. Its timed region gets its own clock
    and power record, so a gap to the dense line splits into work per SM clock and clock (power) effects."""
    cfg = dense_cfg(args)
    A, Bt = wl.dense_inputs(cfg, ctx.dev)
    n0, n1 = sharding.dense_nshard(cfg.N, ctx.world, ctx.rank)
    Bt_r = Bt[n0:n1]
    C = torch.empty(cfg.M, n1 - n0, dtype=torch.float16, device=ctx.dev)

    def step():
        torch.matmul(A, Bt_r.t(), out=C)
    ms = time_region(ctx, step, args.steps, args.warmup, "cublas_dense")
    res["cublas_dense"] = {"ms": ms, "tflops": cfg.flops / (ms * 1e-3) / 1e12,
                           "what": "torch.matmul fp16 x fp16 -> fp16 (cuBLAS), same shape and inputs, same steps"}
    del A, Bt, Bt_r, C
    torch.cuda.empty_cache()


def dense_cfg(args) -> wl.DenseCfg:
    if args.shape:
        M, N, K = (int(x) for x in args.shape.split(","))
        return wl.DenseCfg(M, N, K, 1, "scaled_normal")
    return wl.DENSE_BIG


def bench_dense(ctx: Ctx, args, res: dict):
    cfg = dense_cfg(args)
    A, Bt = wl.dense_inputs(cfg, ctx.dev)
    k_splits = 1
    if args.dense_mode == "nshard":
        n0, n1 = sharding.dense_nshard(cfg.N, ctx.world, ctx.rank)
        Bt_r = Bt[n0:n1]
        C_r = torch.empty(cfg.M, n1 - n0, device=ctx.dev)
        k_splits = args.nshard_k_splits or nshard_k_splits(cfg.M, n1 - n0, cfg.K,
                                                           torch.cuda.get_device_properties(ctx.dev).multi_processor_count)
        if k_splits > 1:  # the shard's tiles leave the last wave of CTA pairs half empty: split K to fill it
            ws = torch.empty(_capi.gemm_splitk_workspace_bytes(cfg.M, n1 - n0, cfg.K, k_splits), dtype=torch.uint8,
                             device=ctx.dev)

            def step():
                _capi.gemm_f16f32_splitk(A, Bt_r, C_r, k_splits, workspace=ws, stream=ctx.stream)
            launches = 2  # GEMM over (tile, split) units + the split reduction
        else:
            def step():
                _capi.gemm_f16f32(A, Bt_r, C_r, stream=ctx.stream)
            launches = 1
        comm = None
    elif args.dense_mode == "splitk_nccl":
        k0, k1 = sharding.dense_ksplit(cfg.K, ctx.world, ctx.rank)
        Cp = torch.empty(cfg.M, cfg.N, device=ctx.dev)
        out = torch.empty(cfg.M // ctx.world, cfg.N, device=ctx.dev)

        def step():
            _capi.gemm_f16f32(A, Bt, Cp, k0, k1, stream=ctx.stream)
            if ctx.world > 1:
                dist.reduce_scatter_tensor(out, Cp)
        launches = 1
        comm = "reduce_scatter (NCCL)"
    else:
        from periodicdent42_b200.dist import SplitKReduceScatterGemm

        op = SplitKReduceScatterGemm(cfg.M, cfg.N) if ctx.world > 1 else None
        out = torch.empty(cfg.M // ctx.world, cfg.N, device=ctx.dev)

        def step():
            if op is None:
                _capi.gemm_f16f32(A, Bt, out, stream=ctx.stream)
            else:
                op(A, Bt, out, stream=ctx.stream)
        launches = 2 if ctx.world > 1 else 1  # scatter GEMM + slot reduction
        comm = "fused into the GEMM epilogue (NVLink peer stores) + 1-element all-reduce barrier"
    ms = time_region(ctx, step, args.steps, args.warmup, "dense")
    if args.dense_mode == "splitk" and ctx.world > 1:
        op.close()
    total_flops = cfg.flops
    tflops = total_flops / (ms * 1e-3) / 1e12
    res["dense"] = {"ms": ms, "tflops": tflops, "flops": total_flops, "launches_per_step": launches,
                    "mode": args.dense_mode, "comm": comm, "per_rank_k_splits": k_splits,
                    "per_rank_flops": total_flops / ctx.world}
    torch.cuda.synchronize()
    if args.dense_mode == "nshard":  # this rank's output columns [n0, n1)
        rows = _pick(cfg.M, 64, 101).to(ctx.dev)
        cols = _pick(n1 - n0, 64, 102 + ctx.rank).to(ctx.dev)
        ref = A[rows].double() @ Bt_r[cols].double().t()
        err = _rel_err(C_r[rows][:, cols], ref)
    else:  # this rank's reduce-scattered rows
        mr = cfg.M // ctx.world
        rows = _pick(mr, 64, 103 + ctx.rank).to(ctx.dev)
        cols = _pick(cfg.N, 64, 104).to(ctx.dev)
        ref = A[rows + ctx.rank * mr].double() @ Bt[cols].double().t()
        err = _rel_err(out[rows][:, cols], ref)
    res["dense"]["check"] = _check_entry(ctx, err, 1e-3, "64 rows x 64 columns of each rank's output")
    # e2e through the public API: host (pinned) inputs -> device, GEMM, result -> host, every step
    if not args.no_e2e and args.dense_mode == "nshard":
        import periodicdent42_b200 as bsk

        A_h = torch.empty(A.shape, dtype=A.dtype, pin_memory=True)
        A_h.copy_(A)
        Bt_h = torch.empty(Bt_r.shape, dtype=Bt.dtype, pin_memory=True)
        Bt_h.copy_(Bt_r)
        C_h = torch.empty(cfg.M, Bt_r.shape[0], dtype=torch.float32, pin_memory=True)
        del A, Bt, Bt_r
        torch.cuda.empty_cache()

        if ctx.world == 1:
            api = "periodicdent42_b200.gemm_from_host"

            def e2e_step():  # K streamed in chunks: PCIe copies of chunk i+1 overlap the GEMM of chunk i
                bsk.gemm_from_host(A_h, Bt_h.t(), out=C_h, k_chunk=args.e2e_k_chunk, sync=False)
        else:  # each rank copies 1/world of A's rows per chunk; NCCL all-gathers the chunk over NVLink
            from periodicdent42_b200.dist import HostShardedGemm
            api = "periodicdent42_b200.dist.HostShardedGemm"
            hsg = HostShardedGemm(cfg.M, Bt_h.shape[0], cfg.K, args.e2e_k_chunk)

            def e2e_step():
                hsg(A_h, Bt_h, C_h)
        ms_e2e = time_region(ctx, e2e_step, args.e2e_steps, 1, "dense_e2e")
        h2d = A_h.numel() * 2 if ctx.world == 1 else (hsg.r1 - hsg.r0) * cfg.K * 2
        res["dense"]["e2e"] = {"value": total_flops / (ms_e2e * 1e-3) / 1e12, "unit": UNIT,
                               "h2d_bytes_per_step": h2d + Bt_h.numel() * 2,
                               "d2h_bytes_per_step": C_h.numel() * 4, "ms_per_step": ms_e2e,
                               "steps": args.e2e_steps, "api": api, "k_chunk": args.e2e_k_chunk or "auto",
                               "bytes_scope": "per rank"}
        if ctx.world > 1:
            res["dense"]["e2e"]["nvlink_gather_bytes_per_step"] = (ctx.world - 1) * hsg.mr * cfg.K * 2
            del hsg
        del A_h, Bt_h, C_h
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- FP8 GEMM
def bench_fp8(ctx: Ctx, args, res: dict):
    cfg = wl.FP8
    Aq, Bqt, sa, sb = wl.fp8_inputs(cfg, ctx.dev)
    n0, n1 = sharding.dense_nshard(cfg.N, ctx.world, ctx.rank)
    Bq_r = Bqt[n0:n1]
    D = torch.empty(cfg.M, n1 - n0, dtype=torch.bfloat16, device=ctx.dev)

    def step():
        _capi.gemm_e4m3_bf16(Aq, Bq_r, sa, sb, D, stream=ctx.stream)
    # 0.5 GB inputs: flush L2 between steps by rotating through 4 input copies is not needed at
    # 268 MB per operand (> 126 MB L2); each step re-reads both operands from HBM.
    ms = time_region(ctx, step, args.op_steps, args.warmup, "fp8")
    torch.cuda.synchronize()
    rows = _pick(cfg.M, 64, 201).to(ctx.dev)
    cols = _pick(n1 - n0, 64, 202 + ctx.rank).to(ctx.dev)
    a_s = Aq.view(torch.uint8)[rows].view(Aq.dtype).double()  # row gathers on the byte view
    b_s = Bq_r.view(torch.uint8)[cols].view(Bq_r.dtype).double()
    ref = (a_s @ b_s.t()) * (sa.double() * sb.double())
    fp8_check = _check_entry(ctx, _rel_err(D[rows][:, cols], ref), 3e-2,
                             "64 rows x 64 columns of each rank's output")
    res["fp8"] = {"ms": ms, "tflops": cfg.flops / (ms * 1e-3) / 1e12, "flops": cfg.flops, "launches_per_step": 1,
                  "check": fp8_check,
                  # per rank: e4m3 A and this rank's B^T rows once, bf16 D columns once
                  "algorithmic_bytes": (cfg.M + (n1 - n0)) * cfg.K + cfg.M * (n1 - n0) * 2}
    del Aq, Bqt, D
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- BSR SpMM
def bench_bsr(ctx: Ctx, args, res: dict):
    cfg = wl.BSR
    crow, col, vals, B = wl.bsr_inputs(cfg, ctx.dev)
    Mb = cfg.M // cfg.block
    r0, r1 = sharding.bsr_block_rows(crow.cpu(), ctx.world, ctx.rank)
    rp32 = crow.to(torch.int32)
    ci32 = col.to(torch.int32)
    C = torch.empty(cfg.M, cfg.N, device=ctx.dev)

    def step():
        _capi.spmm_bsr_f16f32(rp32, ci32, vals, B, C, cfg.M, r0, r1, stream=ctx.stream)
    ms = time_region(ctx, step, args.op_steps, args.warmup, "bsr")
    blocks_r = int(crow[r1].item() - crow[r0].item())
    torch.cuda.synchronize()
    brs = (_pick(r1 - r0, 2, 301 + ctx.rank) + r0).tolist() if r1 > r0 else []
    cols = _pick(cfg.N, 64, 302).to(ctx.dev)
    crow_h, col_h = crow.cpu().tolist(), col.cpu().tolist()
    errs = []
    for br in brs:
        ref = torch.zeros(cfg.block, cols.numel(), dtype=torch.float64, device=ctx.dev)
        for j in range(crow_h[br], crow_h[br + 1]):
            kb = col_h[j]
            ref += vals[j].double() @ B[kb * cfg.block:(kb + 1) * cfg.block][:, cols].double()
        errs.append(_rel_err(C[br * cfg.block:(br + 1) * cfg.block][:, cols], ref))
    bsr_check = _check_entry(ctx, max(errs) if errs else 0.0, 1e-3,
                             "2 block-rows x 64 columns of each rank's block-row range")
    res["bsr"] = {"ms": ms, "tflops": cfg.flops / (ms * 1e-3) / 1e12, "flops": cfg.flops, "launches_per_step": 1,
                  "check": bsr_check,
                  # per rank: its stored blocks, the dense B, its C rows
                  "algorithmic_bytes": blocks_r * cfg.block * cfg.block * 2 + cfg.K * cfg.N * 2
                  + (r1 - r0) * cfg.block * cfg.N * 4,
                  "nnzb": int(crow[-1].item()), "block_rows": [r0, r1], "Mb": Mb}
    del crow, col, vals, B, C
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- attention backward
def _attn_bwd_fp64(q, k, v, dO, rp, ci, bh: int, qb: int, kb: int, scale: float, cfg):
    """fp64 autograd gradients of pair bh: dQ of query block-row qb, dK and dV of key block-row kb. Query rows are
    independent, so the loss sum(O_i * dO_i) over qb and every query block-row whose mask holds kb gives those
    blocks exactly."""
    nqb, blk = cfg.S // cfg.block, cfg.block
    rpl, cil = rp.tolist(), ci.tolist()
    rows = sorted({qb} | {i for i in range(nqb) if kb in cil[rpl[bh * nqb + i]:rpl[bh * nqb + i + 1]]})
    qd, kd, vd = (t.view(-1, cfg.S, cfg.D)[bh].double().requires_grad_() for t in (q, k, v))
    dOd = dO.view(-1, cfg.S, cfg.D)[bh].double()
    loss = 0.0
    for i in rows:
        o = _attn_block_fp64(qd.unsqueeze(0), kd.unsqueeze(0), vd.unsqueeze(0), rp[bh * nqb:], ci, 0, i, scale,
                             cfg, row_base=0)
        loss = loss + (o * dOd[i * blk:(i + 1) * blk]).sum()
    gq, gk, gv = torch.autograd.grad(loss, (qd, kd, vd))
    return gq[qb * blk:(qb + 1) * blk], gk[kb * blk:(kb + 1) * blk], gv[kb * blk:(kb + 1) * blk]


def bench_attn_bwd(ctx: Ctx, args, res: dict):
    """Backward of the attention workload (the forward's shapes and mask): delta + dK/dV pass + dQ pass, through
    the C ABI, LSE and column lists prepared outside the timed region. Useful FLOPs: the standard count of 5
    block GEMMs per nonzero block (2.5 x the forward's 2); the two-pass deterministic scheme executes 7."""
    cfg = wl.ATTN
    q, k, v = wl.attn_inputs(cfg, ctx.dev)
    rp, ci = wl.attn_mask_bsr(cfg)
    pairs, nqb = cfg.B * cfg.H, cfg.S // 128
    b0, b1 = sharding.attn_pairs(rp, nqb, pairs, ctx.world, ctx.rank)
    rp32, ci32 = rp.to(torch.int32).to(ctx.dev), ci.to(torch.int32).to(ctx.dev)
    scale = 1.0 / math.sqrt(cfg.D)
    O = torch.empty_like(q)
    lse = torch.empty(pairs * cfg.S, dtype=torch.float32, device=ctx.dev)
    _capi.bsattn_fwd_ex(q, k, v, O, lse, rp32, ci32, scale, True, stream=ctx.stream)
    col_ptr, row_idx = _capi.bsattn_mask_transpose(rp32, ci32, pairs, nqb, stream=ctx.stream)
    g = torch.Generator(device=ctx.dev).manual_seed(7)
    dO = torch.randn(q.shape, generator=g, device=ctx.dev).to(q.dtype)
    dQ, dK, dV = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(2 * pairs * cfg.S, dtype=torch.float32, device=ctx.dev)
    # the (b,h) pairs of this rank: views starting at pair b0 (row lists rebased to that pair)
    sl = slice(b0, b1)
    Bv = lambda t: t.view(pairs, cfg.S, cfg.D)[sl].view(1, b1 - b0, cfg.S, cfg.D)  # noqa: E731
    base = int(rp[b0 * nqb])
    rp_r = (rp[b0 * nqb:b1 * nqb + 1] - base).to(torch.int32).to(ctx.dev)
    ci_r = ci[base:int(rp[b1 * nqb])].to(torch.int32).to(ctx.dev)
    cp_r = (col_ptr[b0 * nqb:b1 * nqb + 1] - base).contiguous()
    ri_r = row_idx[base:int(rp[b1 * nqb])].contiguous()
    lse_r = lse.view(pairs, cfg.S)[sl].reshape(-1)
    dl_r = delta[:2 * (b1 - b0) * cfg.S]  # this rank's scratch: Delta and -LSE log2(e) of its pairs

    def step():
        _capi.bsattn_bwd(Bv(dO), Bv(q), Bv(k), Bv(v), Bv(O), lse_r, Bv(dQ), Bv(dK), Bv(dV), rp_r, ci_r, cp_r, ri_r,
                         scale, True, delta=dl_r, stream=ctx.stream)
    ms = time_region(ctx, step, args.op_steps, args.warmup, "attn_bwd")
    torch.cuda.synchronize()
    errs = []
    for bh in (_pick(b1 - b0, 2, 501 + ctx.rank) + b0).tolist():
        qb, kb = _pick(nqb, 2, 502 + bh).tolist()
        gq, gk, gv = _attn_bwd_fp64(q, k, v, dO, rp, ci, bh, qb, kb, scale, cfg)
        blk = lambda t, b: t.view(-1, cfg.S, cfg.D)[bh, b * 128:(b + 1) * 128]  # noqa: E731
        errs += [_rel_err(blk(dQ, qb), gq), _rel_err(blk(dK, kb), gk), _rel_err(blk(dV, kb), gv)]
    bwd_check = _check_entry(ctx, max(errs), 2e-2, "dQ of 1 query block-row, dK and dV of 1 key block-row, "
                                                  "of 2 (b,h) pairs per rank")
    nnz = int(rp[-1])
    flops = 2.5 * 4 * 128 ** 2 * cfg.D * nnz
    res["attn_bwd"] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "flops": flops, "launches_per_step": 3,
                       # per rank: read Q, K, V, O, dO and the LSE, write dQ, dK, dV (its pairs)
                       "algorithmic_bytes": (b1 - b0) * cfg.S * (8 * cfg.D * 2 + 4),
                       "nnz_blocks": nnz, "executed_gemm_ratio": 7 / 5, "check": bwd_check}
    del q, k, v, O, dO, dQ, dK, dV
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- autotune
TUNE_SHAPES = [(8192, 1024, 237568), (8192, 2048, 237568), (8192, 4096, 237568), (8192, 8192, 8192),
               (4096, 4096, 4096), (2048, 8192, 16384)]


def bench_autotune(ctx: Ctx, args, res: dict):
    """Dense GEMM launch-configuration tuning: per shape, after ~100 ms of settling, every (tile, group) variant
    timed round-robin twice (3 warm-ups, 10 runs, CUDA events, best of the two), default policy vs the fastest. The first three shapes are the per-rank shards of the headline
    GEMM at N = 8, 4, 2. Rank 0 only (the others idle); no data-path collective."""
    from periodicdent42_b200 import autotune as at

    out = []
    if ctx.rank == 0:
        cache = at.AutotuneCache(args.tune_cache_out) if args.tune_cache_out else None
        for (M, N, K) in TUNE_SHAPES:
            e = at.tune_gemm(M, N, K, warmup=3, runs=10, rounds=2, cache=cache, save=cache is not None)
            fl = 2.0 * M * N * K
            out.append({"shape": [M, N, K], "default_tflops": fl / (e["default_ms"] * 1e-3) / 1e12,
                        "tuned_tflops": fl / (e["ms"] * 1e-3) / 1e12, "speedup": e["default_ms"] / e["ms"],
                        "tile": e["tile_name"], "group_m": e["group_m"], "variants": e["variants"]})
            torch.cuda.empty_cache()
        at.clear()
    ctx.barrier()
    res["autotune"] = out


# ----------------------------------------------------------------------------------------- BSR x BSR
def bench_bsr_bsr(ctx: Ctx, args, res: dict):
    """A = the BSR workload's matrix (8192 x 8192, 16 of 64 128x128 blocks per block-row); B = a second 8192 x 8192
    BSR matrix with the same density (seed 5). Useful FLOPs = 2 * 128^3 per (A block, B block) pair that meet.
    Block-rows sharded like the BSR SpMM at N > 1."""
    cfg = wl.BSR
    crow, col, vals, _ = wl.bsr_inputs(cfg, ctx.dev)
    Kb, Nb = cfg.K // cfg.block, cfg.N // cfg.block
    bcrow, bcol = wl.bsr_pattern(Kb, Nb, cfg.nnz_per_row, torch.Generator().manual_seed(5))
    g = torch.Generator(device=ctx.dev).manual_seed(5)
    bvals = torch.randn(int(bcrow[-1]), 128, 128, generator=g, device=ctx.dev).half()
    b_per_row = (bcrow[1:] - bcrow[:-1])
    pairs = int(b_per_row[col.cpu().long()].sum())  # sum over A blocks (i, k) of B's blocks in row k
    flops = 2 * 128 ** 3 * pairs
    r0, r1 = sharding.bsr_block_rows(crow.cpu(), ctx.world, ctx.rank)
    rp, ci = crow.to(torch.int32), col.to(torch.int32)
    brp, bci = bcrow.to(torch.int32).to(ctx.dev), bcol.to(torch.int32).to(ctx.dev)
    C = torch.empty(cfg.M, cfg.N, device=ctx.dev)

    def step():
        _capi.spmm_bsr_bsr_f16f32(rp, ci, vals, brp, bci, bvals, C, cfg.M, cfg.N, cfg.K, r0, r1, stream=ctx.stream)
    ms = time_region(ctx, step, args.op_steps, args.warmup, "bsr_bsr")
    torch.cuda.synchronize()
    crow_h, col_h, bcrow_h, bcol_h = crow.cpu().tolist(), col.cpu().tolist(), bcrow.tolist(), bcol.tolist()
    errs = []
    for br in ((_pick(r1 - r0, 2, 601 + ctx.rank) + r0).tolist() if r1 > r0 else []):
        ref = torch.zeros(128, cfg.N, dtype=torch.float64, device=ctx.dev)
        for j in range(crow_h[br], crow_h[br + 1]):
            kb = col_h[j]
            for t in range(bcrow_h[kb], bcrow_h[kb + 1]):
                nb = bcol_h[t]
                ref[:, nb * 128:(nb + 1) * 128] += vals[j].double() @ bvals[t].double()
        errs.append(_rel_err(C[br * 128:(br + 1) * 128], ref))
    bb_check = _check_entry(ctx, max(errs) if errs else 0.0, 1e-3, "2 whole block-rows of each rank's range")
    res["bsr_bsr"] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "flops": flops, "launches_per_step": 1,
                      "check": bb_check,
                      "algorithmic_bytes": int(crow[r1] - crow[r0]) * 128 * 128 * 2 + int(bcrow[-1]) * 128 * 128 * 2
                      + (r1 - r0) * 128 * cfg.N * 4,
                      "block_pairs": pairs, "nnzb": int(crow[-1].item()), "b_nnzb": int(bcrow[-1])}
    del crow, col, vals, bvals, C
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- BSR conversion
def bench_convert(ctx: Ctx, args, res: dict):
    """Dense -> BSR and CSR -> BSR on the device for the BSR workload's matrix (8192 x 8192 fp16, 1024 of 4096
    128x128 blocks stored), through the C ABI with preallocated outputs. Headline step: the single-call form
    (no host round trip) with room for every block (capacity M/bs x K/bs, so nothing about the pattern is known
    in advance); the two-phase form (pattern call returns nnzb to the host, then fill) is timed beside it.
    Replicas at N > 1 (every rank converts the whole matrix)."""
    import ctypes

    cfg = wl.BSR
    crow, col, vals, _ = wl.bsr_inputs(cfg, ctx.dev)
    M, K, bs = cfg.M, cfg.K, cfg.block
    A = torch.sparse_bsr_tensor(crow, col, vals, size=(M, K)).to_dense()
    nnzb = int(crow[-1].item())
    cap = (M // bs) * (K // bs)
    lib = _capi.lib()
    ws = torch.empty(_capi.bsr_convert_workspace_bytes(M, K, bs), dtype=torch.uint8, device=ctx.dev)
    rp = torch.empty(M // bs + 1, dtype=torch.int32, device=ctx.dev)
    ci = torch.empty(cap, dtype=torch.int32, device=ctx.dev)
    vo = torch.empty(cap, bs, bs, dtype=torch.float16, device=ctx.dev)
    n_b, n_e = ctypes.c_int64(0), ctypes.c_int64(0)
    st = ctx.stream.cuda_stream

    def step_dense():
        _capi.check(lib.bsk_dense_to_bsr_bounded(A.data_ptr(), K, 2, M, K, bs, rp.data_ptr(), ci.data_ptr(), 4,
                                                 vo.data_ptr(), cap, ws.data_ptr(), ws.numel(), st), "dense")

    def step_dense_2phase():
        _capi.check(lib.bsk_dense_to_bsr_pattern(A.data_ptr(), K, 2, M, K, bs, rp.data_ptr(), 4, ws.data_ptr(),
                                                 ws.numel(), ctypes.byref(n_b), ctypes.byref(n_e), st), "pattern")
        _capi.check(lib.bsk_dense_to_bsr_fill(A.data_ptr(), K, 2, M, K, bs, rp.data_ptr(), ci.data_ptr(), 4,
                                              vo.data_ptr(), n_b.value, ws.data_ptr(), ws.numel(), st), "fill")
    ms_d = time_region(ctx, step_dense, args.op_steps, args.warmup, "convert_dense")
    assert int(rp[-1].item()) == nnzb and torch.equal(ci[:nnzb].long(), col) and torch.equal(vo[:nnzb], vals), \
        "dense->BSR mismatch"
    ms_d2 = time_region(ctx, step_dense_2phase, args.op_steps, args.warmup, "convert_dense_2phase")
    csr = A.to_sparse_csr()
    c_rp, c_ci, c_v = csr.crow_indices().to(torch.int32), csr.col_indices().to(torch.int32), csr.values()
    nnz = c_v.numel()
    del A, csr

    def step_csr():
        _capi.check(lib.bsk_csr_to_bsr_bounded(c_rp.data_ptr(), c_ci.data_ptr(), 4, c_v.data_ptr(), 2, nnz, M, K, bs,
                                               rp.data_ptr(), ci.data_ptr(), 4, vo.data_ptr(), cap, ws.data_ptr(),
                                               ws.numel(), st), "csr")

    def step_csr_2phase():
        _capi.check(lib.bsk_csr_to_bsr_pattern(c_rp.data_ptr(), c_ci.data_ptr(), 4, c_v.data_ptr(), 2, nnz, M, K, bs,
                                               rp.data_ptr(), 4, ws.data_ptr(), ws.numel(), ctypes.byref(n_b),
                                               ctypes.byref(n_e), st), "pattern")
        _capi.check(lib.bsk_csr_to_bsr_fill(c_rp.data_ptr(), c_ci.data_ptr(), 4, c_v.data_ptr(), 2, nnz, M, K, bs,
                                            rp.data_ptr(), ci.data_ptr(), 4, vo.data_ptr(), n_b.value, ws.data_ptr(),
                                            ws.numel(), st), "fill")
    vo.fill_(1.0)
    ms_c = time_region(ctx, step_csr, args.op_steps, args.warmup, "convert_csr")
    assert int(rp[-1].item()) == nnzb and torch.equal(vo[:nnzb], vals), "CSR->BSR mismatch"
    ms_c2 = time_region(ctx, step_csr_2phase, args.op_steps, args.warmup, "convert_csr_2phase")
    blk_bytes = nnzb * bs * bs * 2
    # algorithmic bytes: dense: read the matrix, read the stored blocks again, write them (+ indices);
    # CSR: read crow, col, values twice (pattern and scatter), zero and write the values
    dense_bytes = M * K * 2 + 2 * blk_bytes + (M // bs + 1 + nnzb) * 4
    csr_bytes = (M + 1) * 4 * 2 + 2 * nnz * (4 + 2) + 2 * blk_bytes + (M // bs + 1 + nnzb) * 4
    res["convert"] = {"ms_dense": ms_d, "gbs_dense": dense_bytes / (ms_d * 1e-3) / 1e9, "bytes_dense": dense_bytes,
                      "ms_csr": ms_c, "gbs_csr": csr_bytes / (ms_c * 1e-3) / 1e9, "bytes_csr": csr_bytes,
                      "ms_dense_two_phase": ms_d2, "ms_csr_two_phase": ms_c2,
                      "nnzb": nnzb, "scaling": "replicas"}
    del c_rp, c_ci, c_v, crow, col, vals, ws, rp, ci, vo
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- attention
def _attn_block_fp64(q, k, v, rp, ci, bh: int, qb: int, scale: float, cfg, row_base: int | None = None
                     ) -> torch.Tensor:
    """fp64 block-sparse attention of query block-row qb of pair bh (the key blocks of its mask row, the diagonal
    block causal), on the device. The row's entry in rp is row_base + qb (default bh * S/block + qb)."""
    nqb, blk = cfg.S // cfg.block, cfg.block
    p = (bh * nqb if row_base is None else row_base) + qb
    cols = ci[int(rp[p]):int(rp[p + 1])].tolist()
    if not cols:
        return torch.zeros(blk, cfg.D, dtype=torch.float64, device=q.device)
    qv, kv, vv = (t.view(-1, cfg.S, cfg.D)[bh] for t in (q, k, v))
    Qb = qv[qb * blk:(qb + 1) * blk].double()
    Kc = torch.cat([kv[c * blk:(c + 1) * blk] for c in cols]).double()
    Vc = torch.cat([vv[c * blk:(c + 1) * blk] for c in cols]).double()
    s = (Qb @ Kc.t()) * scale
    kpos = torch.cat([torch.arange(c * blk, (c + 1) * blk, device=q.device) for c in cols])
    diag = torch.cat([torch.full((blk,), c == qb, device=q.device) for c in cols])
    qpos = torch.arange(qb * blk, (qb + 1) * blk, device=q.device)
    s = s.masked_fill(diag[None, :] & (kpos[None, :] > qpos[:, None]), float("-inf"))
    return torch.softmax(s, dim=1) @ Vc


def bench_attn(ctx: Ctx, args, res: dict):
    cfg = wl.ATTN
    q, k, v = wl.attn_inputs(cfg, ctx.dev)
    rp, ci = wl.attn_mask_bsr(cfg)
    nqb = cfg.S // cfg.block
    P = cfg.B * cfg.H
    b0, b1 = sharding.attn_pairs(rp, nqb, P, ctx.world, ctx.rank)
    rp32 = rp.to(torch.int32).to(ctx.dev)
    ci32 = ci.to(torch.int32).to(ctx.dev)
    O = torch.empty_like(q)
    scale = 1.0 / math.sqrt(cfg.D)

    def step():
        _capi.bsattn_fwd_bf16(q, k, v, O, rp32, ci32, scale, True, b0, b1, stream=ctx.stream)
    ms = time_region(ctx, step, args.op_steps, args.warmup, "attn")
    flops = wl.attn_flops(rp, cfg.block, cfg.D)
    torch.cuda.synchronize()
    attn_errs, attn_tols = [], []
    for bh in (_pick(b1 - b0, 2, 401 + ctx.rank) + b0).tolist():
        for qb in _pick(nqb, 2, 402 + bh).tolist():
            ref = _attn_block_fp64(q, k, v, rp, ci, bh, qb, scale, cfg)
            got = O.view(-1, cfg.S, cfg.D)[bh, qb * cfg.block:(qb + 1) * cfg.block]
            attn_errs.append(_rel_err(got, ref))
            attn_tols.append(_rel_err(ref.to(O.dtype), ref) + 1e-3)  # bf16 storage floor + 1e-3
    worst = max((e - t for e, t in zip(attn_errs, attn_tols)), default=-1.0)
    attn_check = _check_entry(ctx, worst, 0.0, "2 query block-rows of 2 (b,h) pairs per rank; err = error - "
                                              "(bf16 storage floor + 1e-3), ok when <= 0")
    res["attn"] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "flops": flops, "launches_per_step": 1,
                   "check": attn_check,
                   # per rank: read Q, K, V and write O of its (b,h) pairs
                   "algorithmic_bytes": (b1 - b0) * cfg.S * cfg.D * 2 * 4,
                   "nnz_blocks": int(rp[-1].item()), "pairs": [b0, b1]}
    del q, k, v, O
    torch.cuda.empty_cache()


# ----------------------------------------------------------------------------------------- CPU baseline
def cpu_dense_sample(cfg: wl.DenseCfg, k_slice: int, seconds: float, threads: int | None = None):
    """The reference's CPU torch path (oracle: torch.matmul on fp32-upcast operands) on a K slice of the
    headline shape; repeats until `seconds` of CPU work. Returns (TFLOPS, reps, cores)."""
    from oracle import reference_path as ref

    torch.set_num_threads(threads or os.cpu_count() or 1)
    A, Bt = wl.dense_inputs(wl.DenseCfg(cfg.M, cfg.N, cfg.K, cfg.seed, cfg.dist), "cpu", k_slice=k_slice)
    flops = 2.0 * cfg.M * cfg.N * k_slice
    ref.dense_ref(A[:256], Bt[:256])  # warm the BLAS threads
    t0 = time.perf_counter()
    reps = 0
    while True:
        ref.dense_ref(A, Bt)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 50:
            break
    return flops * reps / el / 1e12, reps, torch.get_num_threads()


def _cpu_loop(fn, seconds: float, max_reps: int = 1000):
    """Runs fn until `seconds` of wall time (at least once); returns (elapsed s, reps)."""
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= max_reps:
            return el, reps


def cpu_op_samples(seconds: float) -> dict:
    """The reference's CPU torch path of the FP8, BSR and attention operators on bounded samples of their benchmark
    workloads, all host threads, each reported per FLOP of the same kind the GPU line counts (TFLOPS):
      fp8   torch._scaled_mm (e4m3 x e4m3, per-tensor scales, bf16 out) on a 256 x 256 output tile of the workload
            with a K = 2048 slice (the CPU kernel runs at well under 1 GFLOP/s, so the sample is small)
      bsr   torch.sparse.mm on the fp32-upcast BSR matrix (fp16 BSR is not implemented on the CPU) for the first
            block-rows of the workload against the whole dense B; nonzero-block FLOPs
      attn  the block-sparse attention of the workload's first (b,h) pairs, fp32 (masked-SDPA semantics over the
            nonzero key blocks), nonzero-block FLOPs"""
    from oracle import reference_path as ref

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    out = {}
    # FP8
    g = torch.Generator().manual_seed(wl.FP8.seed)
    ks = 2048
    Aq, sa = wl.quantize_e4m3(torch.randn(256, ks, generator=g))
    Bq, sb = wl.quantize_e4m3(torch.randn(256, ks, generator=g))
    el, reps = _cpu_loop(lambda: ref.fp8_ref(Aq, Bq, sa, sb), seconds / 3)
    out["fp8"] = {"value": 2.0 * 256 * 256 * ks * reps / el / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
                  "sample": f"{reps} x torch._scaled_mm 256x256x{ks} (e4m3, per-tensor scales, bf16 out)"}
    # BSR
    cfg = wl.BSR
    crow, col, vals, B = wl.bsr_inputs(cfg, "cpu")
    rows = 4
    nz = int(crow[rows])
    Bf = B.float()
    Ab = torch.sparse_bsr_tensor(crow[:rows + 1], col[:nz], vals[:nz].float(), size=(rows * cfg.block, cfg.K))
    el, reps = _cpu_loop(lambda: torch.sparse.mm(Ab, Bf), seconds / 3)
    out["bsr"] = {"value": 2.0 * nz * cfg.block * cfg.block * cfg.N * reps / el / 1e12, "unit": UNIT,
                  "cores": cores, "kind": "port",
                  "sample": f"{reps} x torch.sparse.mm(fp32 BSR, fp32 B) on {rows} of {cfg.M // cfg.block} block-rows "
                            f"({nz} blocks) x the full 8192x8192 B"}
    del B, Bf, vals
    # attention
    acfg = wl.ATTN
    nqb = acfg.S // acfg.block
    g = torch.Generator().manual_seed(acfg.seed)
    rp, ci = wl.attn_mask_bsr(acfg, n_pairs=2)
    q, k, v = (torch.randn(acfg.S, acfg.D, generator=g).to(torch.bfloat16) for _ in range(3))
    scale = 1.0 / math.sqrt(acfg.D)
    state = {"pairs": 0, "blocks": 0}

    def one_pair():
        p = state["pairs"] % 2
        r0, r1 = p * nqb, (p + 1) * nqb
        ref.attn_blocksparse(q, k, v, rp[r0:r1 + 1], ci[int(rp[r0]):int(rp[r1])], scale, True)
        state["pairs"] += 1
        state["blocks"] += int(rp[r1] - rp[r0])
    el, reps = _cpu_loop(one_pair, seconds / 3)
    out["attn"] = {"value": 4.0 * acfg.block * acfg.block * acfg.D * state["blocks"] / el / 1e12, "unit": UNIT,
                   "cores": cores, "kind": "port",
                   "sample": f"{reps} (b,h) pairs of S={acfg.S}, D={acfg.D}, {state['blocks']} nonzero blocks, "
                             "fp32 block-sparse restatement of masked SDPA"}
    return out


def run_reference(args):
    """--impl reference: the reference's CPU torch path, rank 0 only, bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import reference_path as ref

    cfg = dense_cfg(args)
    k_slice = min(4096, cfg.K)
    torch.set_num_threads(os.cpu_count() or 1)
    A, Bt = wl.dense_inputs(cfg, "cpu", k_slice=k_slice)
    flops = 2.0 * cfg.M * cfg.N * k_slice
    for _ in range(args.warmup):
        ref.dense_ref(A, Bt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.dense_ref(A, Bt)
    el = (time.perf_counter() - t0) / args.steps
    tf = flops / el / 1e12
    sample = f"{cfg.M}x{cfg.N}x{k_slice} K-slice of the {cfg.M}x{cfg.N}x{cfg.K} GEMM, torch.matmul on fp32-upcast operands"
    line = {"metric": METRIC, "value": tf, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"dense fp16->fp32 GEMM M={cfg.M} N={cfg.N} K={cfg.K} (CPU sample K={k_slice})",
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": tf, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": tf, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------------- roofline
def per_clock(tflops_per_gpu: float, region: dict, sm_count: int, mult: int) -> dict:
    """Work per SM clock of a timed region (median SM clock of its samples): FLOP / clk / SM and its fraction of
    the dense tensor peak per clock (8192 for fp16/bf16, 16384 for e4m3)."""
    fpc = tflops_per_gpu * 1e12 / (region["sm_mhz"] * 1e6 * sm_count)
    return {"sm_mhz": region["sm_mhz"], "samples": region["samples"], "reasons": region["reasons"],
            "flop_per_clk_per_sm": fpc, "frac_of_clock_peak": fpc / (8192 * mult)}


def op_roofline(name: str, r: dict, region, peaks: dict, peak_src: str, world: int, sm_count: int, traffic) -> dict:
    """Tensor-core roofline of one operator's timed region. The denominator follows the region's own clock record:
    the measured cuBLAS burst peak when the region ran without the power cap, the sustained (power-capped) one when
    `sw_power_cap` was active in it; FP8 counts twice the bf16 figure."""
    mult = 2 if name == "fp8" else 1
    per_gpu = r["tflops"] / world
    capped = bool(region) and "sw_power_cap" in region["reasons"]
    base = peaks["bf16_tflops_sustained"] if capped else peaks["bf16_tflops"]
    peak = base * mult
    out = {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu / peak,
           "peak_kind": ("2 x " if mult == 2 else "") + f"{peak_src} bf16 "
                        + ("sustained (sw_power_cap active in this region)" if capped
                           else "burst (no power cap in this region)"),
           "algorithmic_bytes": r.get("algorithmic_bytes"),
           "traffic": traffic["bytes_per_launch"] if traffic and world == 1 else None,
           "traffic_source": traffic["source"] if traffic and world == 1 else None}
    if region:
        out.update(per_clock(per_gpu, region, sm_count, mult))
    return out


# ----------------------------------------------------------------------------------------- main
def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        return 1
    ctx = Ctx()
    ctx.init_gpu()
    _capi.lib()
    peaks, peak_src = load_peaks()
    ops = [o.strip() for o in args.ops.split(",") if o.strip()]
    res = {}
    global CLOCKS
    clocks = Clocks(range(ctx.world)) if ctx.rank == 0 else None
    CLOCKS = clocks
    if clocks:
        clocks.start()
    try:
        for op in ops:
            {"dense": bench_dense, "fp8": bench_fp8, "bsr": bench_bsr, "attn": bench_attn,
             "convert": bench_convert, "bsr_bsr": bench_bsr_bsr, "autotune": bench_autotune,
             "attn_bwd": bench_attn_bwd, "cublas": bench_cublas_dense}[op](ctx, args, res)
    finally:
        clk = clocks.stop() if clocks else None
    err_word = _capi.device_error()
    cpu = None
    cpu_ops = {}
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        if "dense" in res:
            tf, reps, cores = cpu_dense_sample(dense_cfg(args), min(4096, dense_cfg(args).K), args.cpu_seconds)
            cpu = {"value": tf, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"{reps} x torch.matmul(fp32) on the 8192x8192x4096 K-slice of the headline shape"}
        if any(o in res for o in ("fp8", "bsr", "attn")):
            cpu_ops = cpu_op_samples(args.cpu_seconds)
    if ctx.rank == 0:
        d = res.get("dense")
        traffic = load_traffic()
        peak_t = peaks["bf16_tflops_sustained"]
        line = {"metric": METRIC, "value": d["tflops"] if d else None, "unit": UNIT, "n_gpus": ctx.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": d["ms"] if d else None,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded device RNG, the benchmark configurations' shapes and distributions)",
                "config": {"workload": "dense fp16->fp32 GEMM M=8192 N=8192 K=237568 (A row-major, B col-major)"
                           if not args.shape else f"dense fp16->fp32 GEMM {args.shape} (profiling case)",
                           "parallelism": f"{args.dense_mode} x{ctx.world}",
                           "l2": "inputs larger than L2 (7.8 GB per step)"}}
        if d:
            kern = traffic.get("gemm_f16f32")
            per_launch_flops = d["per_rank_flops"]
            line["roofline"] = {"bound": "tensor", "achieved": per_launch_flops / (d["ms"] * 1e-3) / 1e12,
                                "peak": peak_t, "unit": "TFLOP/s",
                                "frac": per_launch_flops / (d["ms"] * 1e-3) / 1e12 / peak_t,
                                "peak_kind": f"{peak_src} bf16 sustained (cuBLAS, power-capped loop)",
                                "peak_burst": peaks["bf16_tflops"],
                                "traffic": (kern["read_bytes_per_unit_k"] * dense_cfg(args).K + kern["write_bytes_per_launch"]
                                            if kern and ctx.world == 1 else None),
                                "traffic_source": kern["source"] if kern and ctx.world == 1 else None,
                                "algorithmic_bytes": (dense_cfg(args).M + dense_cfg(args).N // ctx.world)
                                * dense_cfg(args).K * 2 + dense_cfg(args).M * dense_cfg(args).N // ctx.world * 4}
            line["e2e"] = d.get("e2e")
            line["check"] = d.get("check")
            line["gpu_launches"] = args.steps * d["launches_per_step"]
        line["cpu_baseline"] = cpu
        line["clocks"] = clk
        opsum = {}
        regions = (clk or {}).get("per_region", {})
        sm_count = torch.cuda.get_device_properties(ctx.dev).multi_processor_count
        if d and regions.get("dense"):
            line["per_clock"] = per_clock(d["tflops"] / ctx.world, regions["dense"], sm_count, 1)
        for name in ("fp8", "bsr", "attn", "attn_bwd", "bsr_bsr"):
            if name in res:
                r = res[name]
                opsum[name] = {"tflops": r["tflops"], "ms": r["ms"],
                               "roofline": op_roofline(name, r, regions.get(name), peaks, peak_src, ctx.world,
                                                       sm_count, traffic.get(name)),
                               "cpu_baseline": cpu_ops.get(name)}
                for kk in ("nnzb", "nnz_blocks", "block_pairs", "b_nnzb", "algorithmic_bytes", "check"):
                    if kk in r:
                        opsum[name][kk] = r[kk]
        if "convert" in res:
            r = res["convert"]
            opsum["bsr_convert"] = {"dense_gbs": r["gbs_dense"], "dense_ms": r["ms_dense"],
                                    "csr_gbs": r["gbs_csr"], "csr_ms": r["ms_csr"], "peak_gbs": peaks["hbm_gbs"],
                                    "dense_ms_two_phase": r["ms_dense_two_phase"],
                                    "csr_ms_two_phase": r["ms_csr_two_phase"],
                                    "dense_frac_of_peak": r["gbs_dense"] / peaks["hbm_gbs"],
                                    "csr_frac_of_peak": r["gbs_csr"] / peaks["hbm_gbs"],
                                    "peak_basis": f"{peak_src} HBM copy", "nnzb": r["nnzb"],
                                    "scaling": r["scaling"]}
        if res.get("autotune"):
            opsum["autotune_dense"] = res["autotune"]
        if "cublas_dense" in res:  # work per SM clock of both timed regions (median SM clock of each region)
            r = dict(res["cublas_dense"])
            regions = (clk or {}).get("per_region", {})
            sm_count = torch.cuda.get_device_properties(ctx.dev).multi_processor_count
            for name, tf in (("cublas_dense", r["tflops"]), ("dense", d["tflops"] if d else None)):
                reg = regions.get(name)
                if reg and tf:
                    r[f"{name}_sm_mhz"] = reg["sm_mhz"]
                    r[f"{name}_power_w_median"] = reg["power_w_median"]
                    r[f"{name}_flop_per_clk_per_sm"] = tf / ctx.world * 1e12 / (reg["sm_mhz"] * 1e6 * sm_count)
            opsum["cublas_dense"] = r
        line["ops"] = opsum
        checks = {name: {kk: r["check"][kk] for kk in ("err", "tol", "ok")}
                  for name, r in res.items() if isinstance(r, dict) and "check" in r}
        line["checks"] = {"all_ok": all(c["ok"] for c in checks.values()), "ranks": ctx.world, **checks}
        line["device_error_word"] = err_word
        print(json.dumps(line), flush=True)
    ctx.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
