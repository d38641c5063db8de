"""Per-shape launch-configuration autotuner with a persistent JSON cache.

Follows the reference's sparse auto-tuner (optim_local/src/sparse/autotune_sparse.h: time every kernel variant
with CUDA events after warm-up runs, keep the fastest, cache the winner per problem key in a file) and replaces
its size-bucketed tile table ``_autotune_config`` (BlackwellSparseK/python/ops.py:209-217). The variants here are
the launch configurations the sm_100 kernels accept -- tile kind (single CTA 128x256, CTA pair 256x256, CTA pair
256x512; dense GEMMs only) and tile-rasterisation group -- and the winner is registered in the library's
per-shape table (``bsk_config_set``), which every later launch of that operator and shape consults.

Cache file: JSON ``{device_key: {"op:MxNxK": {"tile": t, "group_m": g, "ms": ..., "default_ms": ...}}}`` where
device_key names the GPU model, SM count and library version, so a cache copied to other hardware is ignored.
Location: ``$BSK_AUTOTUNE_CACHE`` or ``~/.cache/periodicdent42_b200/autotune.json``.
"""
from __future__ import annotations

import json
import os
import tempfile
from typing import Callable, Iterable, Optional

import torch

from . import _capi

OPS = {"gemm_f16f32": 1, "gemm_e4m3_bf16": 2, "spmm_bsr": 3, "spmm_bsr_bsr": 4}
TILES = {-1: "policy", 0: "single_128x256", 1: "pair_256x256", 2: "pair_256x512"}
SPMM_TILES = {-1: "policy", 0: "single_128x256", 1: "pair_128x512_transposed"}  # BSR x dense SpMM
GROUPS = (0, 1, 2, 4, 8, 16, 32, 64)


def default_cache_path() -> str:
    return os.environ.get("BSK_AUTOTUNE_CACHE") or os.path.join(os.path.expanduser("~"), ".cache",
                                                                 "periodicdent42_b200", "autotune.json")


def device_key(device=None) -> str:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    props = torch.cuda.get_device_properties(dev)
    return f"{props.name}|sm{props.major}{props.minor}|{props.multi_processor_count}SM|lib{_capi.lib().bsk_version()}"


def shape_key(op: str, M: int, N: int, K: int) -> str:
    if op not in OPS:
        raise ValueError(f"unknown operator {op!r}; one of {sorted(OPS)}")
    return f"{op}:{M}x{N}x{K}"


def parse_shape_key(key: str) -> tuple[str, int, int, int]:
    op, dims = key.split(":")
    M, N, K = (int(x) for x in dims.split("x"))
    return op, M, N, K


def candidates(op: str, M: int, N: int, K: int) -> list[tuple[int, int]]:
    """(tile, group_m) variants to time: every tile kind (the policy's own choice first) times the rasterisation
    groups that differ for this many M tiles. Dense GEMMs: single 128x256, pair 256x256, pair 256x512; BSR x dense
    SpMM: single 128x256, CTA-pair 128x512 (at least 512 output columns); BSR x BSR: the group only."""
    if op in ("gemm_f16f32", "gemm_e4m3_bf16"):
        tiles = [-1, 0, 1, 2]
    elif op == "spmm_bsr":
        # BSK_SPMM_TILE forces one tile kind over any registered configuration, so tile variants would all time
        # the same kernel and the cache would record an arbitrary winner: tune the group only
        tiles = [-1, 0, 1] if N >= 512 and not os.environ.get("BSK_SPMM_TILE") else [-1]
    else:
        tiles = [-1]
    out = []
    for t in tiles:
        rows = 128 if t == 0 or (t == -1 and M <= 128) or op.startswith("spmm") else 256
        m_tiles = max(1, -(-M // rows))
        seen = set()
        for g in GROUPS:
            eff = g if g == 0 else min(g, m_tiles)
            if eff in seen:
                continue
            seen.add(eff)
            out.append((t, g))
    return out


class AutotuneCache:
    """The JSON cache file, per device key."""

    def __init__(self, path: Optional[str] = None):
        self.path = path or default_cache_path()
        self.data: dict = {}
        if os.path.exists(self.path):
            with open(self.path) as f:
                self.data = json.load(f)

    def entries(self, dkey: str) -> dict:
        return self.data.setdefault(dkey, {})

    def get(self, dkey: str, key: str) -> Optional[dict]:
        return self.data.get(dkey, {}).get(key)

    def put(self, dkey: str, key: str, entry: dict) -> None:
        self.entries(dkey)[key] = entry

    def save(self) -> None:
        d = os.path.dirname(self.path)
        if d:
            os.makedirs(d, exist_ok=True)
        fd, tmp = tempfile.mkstemp(dir=d or ".", prefix=".autotune", suffix=".json")
        with os.fdopen(fd, "w") as f:
            json.dump(self.data, f, indent=1, sort_keys=True)
        os.replace(tmp, self.path)


def register(op: str, M: int, N: int, K: int, tile: int, group_m: int) -> None:
    _capi.check(_capi.lib().bsk_config_set(OPS[op], M, N, K, tile, group_m), "bsk_config_set")


def registered(op: str, M: int, N: int, K: int) -> Optional[tuple[int, int]]:
    import ctypes

    t, g = ctypes.c_int(-1), ctypes.c_int(0)
    found = _capi.lib().bsk_config_get(OPS[op], M, N, K, ctypes.byref(t), ctypes.byref(g))
    if found < 0:
        _capi.check(found, "bsk_config_get")
    return (t.value, g.value) if found == 1 else None


def clear() -> None:
    _capi.check(_capi.lib().bsk_config_clear(), "bsk_config_clear")


def load_cache(path: Optional[str] = None, device=None) -> int:
    """Registers every cached configuration of this device; returns how many."""
    cache = AutotuneCache(path)
    n = 0
    for key, e in cache.data.get(device_key(device), {}).items():
        op, M, N, K = parse_shape_key(key)
        register(op, M, N, K, int(e["tile"]), int(e["group_m"]))
        n += 1
    return n


def time_ms(fn: Callable[[], None], warmup: int = 5, runs: int = 20) -> float:
    """Mean CUDA-event time of fn on the current stream after `warmup` untimed calls (the reference tuner's
    protocol: 5 warm-ups, 20 timed runs)."""
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(runs):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / runs


def tune(op: str, M: int, N: int, K: int, run: Callable[[], None], variants: Optional[Iterable] = None,
         warmup: int = 5, runs: int = 20, rounds: int = 2, settle_ms: float = 100.0,
         cache: Optional[AutotuneCache] = None, save: bool = True) -> dict:
    """Times `run` (one launch of `op` at this shape) under every variant, registers the fastest and records
    it in the cache. Returns the cache entry. The GPU first runs the op for about `settle_ms` (clocks and power
    reach their working state), then the variants are timed round-robin `rounds` times and each keeps its best
    time, so no variant is favoured by when it ran."""
    key = shape_key(op, M, N, K)
    prior = registered(op, M, N, K)
    variants = list(variants or candidates(op, M, N, K))
    best = {}
    try:
        register(op, M, N, K, -1, 0)
        one = time_ms(run, 1, 1)
        time_ms(run, 0, max(1, int(settle_ms / max(one, 1e-3))))
        for _ in range(max(1, rounds)):
            for tile, group in variants:
                register(op, M, N, K, tile, group)
                ms = time_ms(run, warmup, runs)
                best[(tile, group)] = min(ms, best.get((tile, group), float("inf")))
    finally:
        if prior is not None:
            register(op, M, N, K, *prior)
    results = [(ms, t, g) for (t, g), ms in best.items()]
    default_ms = best.get((-1, 0))
    best_ms, tile, group = min(results)
    register(op, M, N, K, tile, group)
    entry = {"tile": tile, "tile_name": (SPMM_TILES if op == "spmm_bsr" else TILES)[tile], "group_m": group, "ms": best_ms, "default_ms": default_ms,
             "variants": len(results), "warmup": warmup, "runs": runs, "rounds": rounds}
    if cache is None and save:
        cache = AutotuneCache()
    if cache is not None:
        cache.put(device_key(), key, entry)
        if save:
            cache.save()
    return entry


def tune_gemm(M: int, N: int, K: int, device=None, **kw) -> dict:
    """Tunes the dense fp16 GEMM at (M, N, K) on random operands."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(M, K, generator=g, device=dev).half()
    Bt = torch.randn(N, K, generator=g, device=dev).half()
    C = torch.empty(M, N, device=dev)
    return tune("gemm_f16f32", M, N, K, lambda: _capi.gemm_f16f32(A, Bt, C), **kw)


def tune_spmm_bsr(row_ptr, col_idx, vals, B, M: int, **kw) -> dict:
    """Tunes the BSR SpMM (tile kind and rasterisation group) on the caller's operands (int32 indices, fp16 values)."""
    K, N = B.shape
    C = torch.empty(M, N, device=B.device)
    return tune("spmm_bsr", M, N, K, lambda: _capi.spmm_bsr_f16f32(row_ptr, col_idx, vals, B, C, M), **kw)
