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
