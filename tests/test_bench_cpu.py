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
    # The TMA-fed SGEMM path is the persistent kernel on row-major A (one
    # launch), or for the forced transposed-A forms the transpose of A and
    # the GEMM; split-K adds the reduce.  The others are one.  Mirrors
    # sgemm_tma_eligible.
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.delenv("B2B_SGEMM_VARIANT", raising=False)
    monkeypatch.delenv("B2B_SGEMM_KSPLIT", raising=False)
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 1
    assert bench.sgemm_kernels_per_call(8192, 4096, 4096) == 1      # 6.9 waves: unsplit
    assert bench.sgemm_kernels_per_call(4096, 1024, 4096) == 2      # S = 8: GEMM + reduce
    assert bench.sgemm_kernels_per_call(8192, 8192, 8190) == 2      # K % 4 != 0: transpose + GEMM
    assert bench.sgemm_kernel_name(8192, 8192, 8192).startswith("sgemm_tma_rowa_ws_kernel")
    # split-K adds the reduce: grids under one wave, or just past a whole one
    assert bench.sgemm_ksplit(148, 1024, 1024, 1024) == 4
    assert bench.sgemm_ksplit(148, 4096, 4096, 4096) == 2
    assert bench.sgemm_ksplit(148, 8192, 8192, 8192) == 1
    assert bench.sgemm_kernels_per_call(1024, 1024, 1024) == 2   # persistent GEMM + reduce
    assert bench.sgemm_kernels_per_call(2048, 1024, 4096) == 2
    assert bench.sgemm_kernels_per_call(1024, 1024, 1022) == 3   # K % 4 != 0: transpose + GEMM + reduce
    assert bench.sgemm_kernels_per_call(512, 4096, 4096, splits=2) == 2
    monkeypatch.setenv("B2B_SGEMM_KSPLIT", "1")
    assert bench.sgemm_kernels_per_call(1024, 1024, 1024) == 1
    monkeypatch.delenv("B2B_SGEMM_KSPLIT")
    assert bench.sgemm_kernels_per_call(512, 512, 512) == 2        # any size on the persistent kernel; S = 2
    assert bench.sgemm_kernels_per_call(100, 2048, 64) == 1        # M < 128, unsplit
    assert bench.sgemm_kernels_per_call(129, 257, 65) == 1         # N % 4 != 0: the cp.async kernel
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192, tf32x3=True) == 1
    monkeypatch.setenv("B2B_SGEMM_VARIANT", "11")
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 1
    monkeypatch.setenv("B2B_SGEMM_VARIANT", "21")
    assert bench.sgemm_kernels_per_call(8192, 8192, 8192) == 2


def test_dgemm_kernels_per_call(monkeypatch):
    # The persistent DMMA DGEMM is one launch, plus the reduce when its
    # split-K model picks a split (grids that fill the GPU badly).  Mirrors
    # dgemm_ksplit in dgemm_dmma.cu.
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.delenv("B2B_DGEMM_VARIANT", raising=False)
    monkeypatch.delenv("B2B_DGEMM_KSPLIT", raising=False)
    assert bench.dgemm_ksplit(148, 4096, 4096, 4096) == 1
    assert bench.dgemm_ksplit(148, 1024, 1024, 1024) == 2
    assert bench.dgemm_ksplit(148, 2048, 2048, 2048) == 4        # 1.73 waves
    assert bench.dgemm_ksplit(148, 4096, 512, 4096) == 8         # a DGEMM 4096^3 column panel on 8 GPUs
    assert bench.dgemm_kernels_per_call(4096, 4096, 4096) == 1
    assert bench.dgemm_kernels_per_call(1024, 1024, 1024) == 2
    assert bench.dgemm_kernels_per_call(1024, 1024, 1023) == 1   # K odd: the DFMA kernel
    monkeypatch.setenv("B2B_DGEMM_KSPLIT", "4")
    assert bench.dgemm_kernels_per_call(4096, 4096, 4096) == 2
    monkeypatch.setenv("B2B_DGEMM_VARIANT", "8")
    assert bench.dgemm_kernels_per_call(1024, 1024, 1024) == 1


def _bench_args(argv):
    sys.path.insert(0, ROOT)
    import argparse

    import bench

    # the parser bench.main() builds, without running it
    ns = argparse.Namespace(workload="hgemm", op="dot", trans=False, gather=False, gather_multicast=False,
                            gather_nccl=False, no_gather=False, weak=False, no_secondary=False, tf32x3=False,
                            fused=False, mlp_streams=2, m=None, n=None, k=None)
    for a in argv:
        k, _, v = a.partition("=")
        setattr(ns, k, v if v else True)
    return bench, ns


@pytest.mark.parametrize("world", [1, 2])
def test_reference_arm_prints_the_library_config(world):
    # The reference arm's config record is the one the library arm prints at
    # the same world size (both come from workload_config).
    bench, ns = _bench_args(["workload=batched"])
    p = _run_bench(["--impl", "reference", "--workload", "batched", "--steps", "1", "--warmup", "3"],
                   {"RANK": "0", "WORLD_SIZE": str(world), "LOCAL_RANK": "0"})
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads(p.stdout.strip().splitlines()[-1])
    assert d["config"] == bench.workload_config("batched", ns, world)
    assert d["scaling"] == d["config"]["scaling"] == ("strong" if world > 1 else "weak")
    assert d["data"] == bench.DATA


def test_hgemm_config_at_n_gpus():
    # One GPU: the 8192^3 problem, no gather.  N GPUs: the same fixed problem,
    # 8192/N columns per GPU, C gathered by the fused kernel; --weak and
    # --no-gather give the panel-only forms.
    bench, ns = _bench_args([])
    c1 = bench.workload_config("hgemm", ns, 1)
    assert (c1["m"], c1["n"], c1["k"], c1["gather"], c1["scaling"]) == (8192, 8192, 8192, False, "weak")
    c8 = bench.workload_config("hgemm", ns, 8)
    assert (c8["n"], c8["n_per_gpu"], c8["gather"], c8["scaling"]) == (8192, 1024, "fused", "strong")
    _, ns_w = _bench_args(["weak"])
    cw = bench.workload_config("hgemm", ns_w, 8)
    assert (cw["n"], cw["n_per_gpu"], cw["gather"], cw["scaling"]) == (65536, 8192, False, "weak")
    _, ns_n = _bench_args(["no_gather"])
    assert bench.workload_config("hgemm", ns_n, 4)["gather"] is False
    _, ns_c = _bench_args(["gather_nccl"])
    assert bench.workload_config("hgemm", ns_c, 2)["gather"] == "nccl"
    # SGEMM / DGEMM gather only when asked
    assert bench.workload_config("sgemm", ns, 8)["gather"] is False


def test_secondary_configurations():
    bench, ns = _bench_args([])
    assert bench.secondary_names(ns, 1) == ["sgemm", "sgemv", "batched", "dgemm"]
    assert bench.secondary_names(ns, 8) == ["batched", "hgemm-weak", "sgemm", "sgemm-gather", "dgemm"]
    _, ns2 = _bench_args(["no_secondary"])
    assert bench.secondary_names(ns2, 1) == []
    _, ns3 = _bench_args(["workload=sgemm"])
    assert bench.secondary_names(ns3, 1) == []


def test_seeded_inputs_are_shared_and_chunked():
    import torch

    bench, _ = _bench_args([])
    a = bench.host_tensor((64, 32), bench.TID["A"], torch.float16, "normal")
    b = bench.host_tensor((64, 32), bench.TID["A"], torch.float16, "normal")
    assert torch.equal(a, b) and a.dtype == torch.float16
    assert float(a.float().std()) == pytest.approx(0.1, rel=0.2)
    u = bench.host_tensor((1 << 16,), bench.TID["B"], torch.float32)
    assert float(u.min()) >= -1.0 and float(u.max()) < 1.0
    assert not torch.equal(u[:2048].reshape(64, 32).half(), a)  # different tensor ids, different numbers
    # a rank's batch range is the same numbers as that range of the whole
    whole = bench.batched_inputs(bench.TID["A"], 0, 1024, 8)
    part = bench.batched_inputs(bench.TID["A"], 300, 700, 8)
    assert torch.equal(part, whole[300:700])
