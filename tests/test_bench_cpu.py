"""bench.py on the CPU: the reference arm's JSON contract (it runs the
oracle's host loops, no GPU) and the host-side helpers of the GPU arm."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


def _run_bench(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("workload", ["batched", "sgemv"])
def test_reference_arm_json_line(workload):
    p = _run_bench(["--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] == 3 and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]


def test_reference_arm_other_ranks_exit_quietly():
    p = _run_bench(["--impl", "reference", "--workload", "batched", "--steps", "1", "--warmup", "3"],
                   {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_sgemm_kernels_per_call(monkeypatch):
    # The TMA-fed SGEMM path is two launches (transpose of A, GEMM); the
    # others are one.  Mirrors sgemm_tma_eligible.
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.delenv("B2B_SGEMM_VARIANT", raising=False)
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 2
    assert bench.sgemm_kernels_per_call(4096, 1024, 4096) == 2
    assert bench.sgemm_kernels_per_call(512, 512, 512) == 1        # N < 1024
    assert bench.sgemm_kernels_per_call(100, 2048, 64) == 1        # M < 128
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192, tf32x3=True) == 1
    monkeypatch.setenv("B2B_SGEMM_VARIANT", "11")
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 1
    monkeypatch.setenv("B2B_SGEMM_VARIANT", "21")
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 2
