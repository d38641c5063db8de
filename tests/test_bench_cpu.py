"""bench.py's output contract on CPU: the reference arm (`--impl reference`, the reference's CPU torch path) prints
one JSON line with the keys the benchmark driver reads, and the GPU arm refuses to run without a device."""
import json
import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, env=None):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args], cwd=REPO, capture_output=True,
                       text=True, timeout=600, env=env)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    return r.returncode, (json.loads(lines[-1]) if lines else None), r


def test_reference_arm_line():
    rc, line, r = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--shape", "512,512,2048")
    assert rc == 0, r.stderr[-2000:]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 2 and line["warmup"] == 1
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1")
    rc, line, r = _run("--impl", "reference", "--steps", "1", "--warmup", "1", "--shape", "256,256,1024", env=env)
    assert rc == 0 and line is None, r.stdout[-500:]


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_gpu_arm_without_a_device_fails_loudly():
    rc, line, _ = _run("--steps", "1", "--warmup", "1")
    assert rc != 0 and line is not None and "error" in line


def _bench_module():
    sys.path.insert(0, REPO)
    import bench

    return bench


def test_self_check_attention_references_match_the_oracle():
    """The sampled fp64 references that bench.py checks each rank's attention output and gradients against agree
    with the oracle (forward) and with fp64 autograd through the oracle over the whole pair (backward)."""
    from oracle import reference_path as ref
    from periodicdent42_b200 import workloads as wl

    bench = _bench_module()
    cfg = wl.AttnCfg(1, 2, 1024, 32, 128, 2, 2, 9)
    q, k, v = (t.double() for t in wl.attn_inputs(cfg, "cpu"))
    rp, ci = wl.attn_mask_bsr(cfg)
    nqb, scale = cfg.S // cfg.block, 0.3
    dO = torch.randn(q.shape, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    for bh in range(cfg.B * cfg.H):
        qp, kp, vp = (t.view(-1, cfg.S, cfg.D)[bh].clone().requires_grad_() for t in (q, k, v))
        rpp = rp[bh * nqb:(bh + 1) * nqb + 1]
        want = ref.attn_blocksparse_fp64(qp, kp, vp, rpp, ci[int(rpp[0]):int(rpp[-1])], scale, True, cfg.block)
        for qb in range(nqb):
            got = bench._attn_block_fp64(q, k, v, rp, ci, bh, qb, scale, cfg)
            assert torch.allclose(got, want[qb * 128:(qb + 1) * 128], atol=1e-12, rtol=0)
        gq, gk, gv = torch.autograd.grad((want * dO.view(-1, cfg.S, cfg.D)[bh]).sum(), (qp, kp, vp))
        for qb, kb in ((0, 3), (5, 5), (7, 1)):
            sq, sk, sv = bench._attn_bwd_fp64(q, k, v, dO, rp, ci, bh, qb, kb, scale, cfg)
            assert torch.allclose(sq, gq[qb * 128:(qb + 1) * 128], atol=1e-10, rtol=0)
            assert torch.allclose(sk, gk[kb * 128:(kb + 1) * 128], atol=1e-10, rtol=0)
            assert torch.allclose(sv, gv[kb * 128:(kb + 1) * 128], atol=1e-10, rtol=0)


def test_self_check_helpers():
    bench = _bench_module()
    a = torch.ones(4, 4, dtype=torch.float64)
    assert bench._rel_err(a, a) == 0.0
    assert abs(bench._rel_err(a * 1.01, a) - 0.01) < 1e-12
    p = bench._pick(100, 10, 1)
    assert p.numel() == 10 and torch.equal(p, torch.sort(p).values) and torch.equal(p, bench._pick(100, 10, 1))
    assert bench._pick(5, 10, 1).numel() == 5


def test_nshard_k_splits_policy():
    """The benchmark's per-rank split of K: only the 2-rank shard of the headline (half-empty last wave of CTA pairs,
    long K) is split."""
    bench = _bench_module()
    assert [bench.nshard_k_splits(8192, n, 237568, 148) for n in (8192, 4096, 2048, 1024)] == [1, 2, 1, 1]
    assert bench.nshard_k_splits(8192, 4096, 16384, 148) == 1  # short K: no split
