#!/usr/bin/env python
"""bench.py -- throughput of the b2blas GEMM/GEMV hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W] [--impl b2blas|reference]

One JSON line on rank 0.  The default workload is the HGEMM configuration:
8192 x 8192 x 8192, f16 in / f32 accumulate / f16 out, alpha 1, beta 0,
inputs i.i.d. normal(0, 0.1) rounded to f16 (seeded, synthetic).  On N > 1
GPUs (one process per GPU, torchrun) the same fixed 8192^3 problem is
column-sharded with A replicated (8192/N columns of B and C per GPU) and
the all-gather is fused into the GEMM: every rank's epilogue stores its
panel into every rank's full row-major C over NVLink peer pointers, so each
rank ends every step with the whole C ("strong" scaling; --no-gather keeps
the panels, --gather-nccl gathers through NCCL + a re-layout kernel,
--weak gives every rank its own 8192-column panel of an 8192 x 8192N x 8192
product instead).

A "step" is one GEMM call over one batch of resident device inputs, timed
with CUDA events on the stream the kernels run on (K steps between a barrier
+ synchronize on both sides, max over ranks).  `e2e` is the same metric
through the host-slice API (b2b_hgemm_simple): every step copies A and B from
page-locked host memory and C back.

`secondary` carries the metric's other configurations, each device-timed
the same way in its own region with its own clock record and roofline: on
one GPU SGEMM 8192^3 (alpha 1.5, beta 0.5), SGEMV 16384^2 N, strided-batched
SGEMM 4096 x 256^3 and DGEMM 4096^3; on N GPUs the batch-sharded
strided-batched SGEMM (strong), the weak-scaled HGEMM without a gather, and
SGEMM 8192^3 (without and with the gathered C) and DGEMM 4096^3 with the
columns of B and C sharded and A replicated (--no-secondary skips them).

Other workloads (--workload): sgemm (8192^3, alpha 1.5, beta 0.5), dgemm
(4096^3), batched (4096 x 256^3 strided, batch-sharded), sgemv / dgemv /
hgemv (16384^2, N, or T with --trans), reduce (sdot by default, --op
nrm2|asum|iamax; 2^28-element f32 vectors), mlp (4 layers
1024-4096-4096-4096-1024, batch 4096, sgemm + saxpy bias).

Inputs: both arms draw every tensor from torch's CPU generator with a fixed
seed per tensor (host_tensor), so the library and the reference arm see the
same numbers; the library arm copies them to the device before timing.

On one GPU the line also carries `reference_kernels`: the reference's own GPU
kernels for the same operation (naive / tiled / vectorized / double_buf
GEMMs, hgemm_half, the strided-batched and GEMV kernels, the 32-thread
reductions, the mlp example's sgemm_tiled + saxpy), restated in CUDA C
because the reference's Rust / cuda-oxide build cannot run here, timed on the
same resident buffers (--no-ref-kernels skips them).

--impl reference times the CPU restatement of the reference's algorithm
(the oracle's host triple loop) on this machine's cores, rank 0 only, with a
bounded sample of the same workload per step, and prints the same config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cublas-rs_b200"))
sys.path.insert(0, ROOT)

METRIC = "GEMM TFLOP/s & % of roofline at 1/2/4/8 B200 (8192³ HGEMM/SGEMM); SGEMV GB/s"

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["_source"] = "measured (MEASURED_PEAKS.json)"
        return d
    d = dict(FALLBACK_PEAKS)
    d["_source"] = "fallback (no MEASURED_PEAKS.json)"
    return d


def load_traffic():
    """Per-launch DRAM bytes of each workload's dominant kernel, from the
    committed ncu summary (profiles/dram_traffic.json), or {}."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# --------------------------------------------------------------- clocks

_REASONS = [
    (0x1, "gpu_idle"), (0x2, "applications_clocks_setting"), (0x4, "sw_power_cap"), (0x8, "hw_slowdown"),
    (0x10, "sync_boost"), (0x20, "sw_thermal_slowdown"), (0x40, "hw_thermal_slowdown"),
    (0x80, "hw_power_brake_slowdown"), (0x100, "display_clock_setting"),
]


class ClockSampler:
    """Polls NVML (SM clock, event reasons) every few ms while running."""

    def __init__(self, cuda_index: int, period_s: float = 0.002):
        self.samples = []
        self.max_mhz = None
        self.ok = False
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nv = pynvml
            h = None
            try:
                uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hi = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hi)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        h = hi
                        break
            except Exception:
                h = None
            if h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[cuda_index]) if vis and vis.split(",")[0].isdigit() else cuda_index
                h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                clk = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                try:
                    pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
                except Exception:
                    pw = None
                self.samples.append((clk, rs, pw))
            except Exception:
                pass
            self._stop.wait(self._period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml" if self.ok else "unavailable"}
        clks = [c for c, _, _ in self.samples]
        mask = 0
        for _, r, _ in self.samples:
            mask |= int(r)
        reasons = [name for bit, name in _REASONS if mask & bit and name != "gpu_idle"]
        pws = [p for _, _, p in self.samples if p is not None]
        return {"sm_mhz": statistics.median(clks), "sm_min_mhz": min(clks), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_median": statistics.median(pws) if pws else None,
                "power_w_max": max(pws) if pws else None, "source": "nvml"}


# ------------------------------------------------------------ workloads

# Which page-locked allocator the end-to-end pass uses: the library's
# (b2b_host_alloc = cudaHostAlloc) or torch's pin_memory.
E2E_HOST = {"handle": None}


def sgemm_ksplit(sm_count, m, n, k):
    """The library's split-K choice for the TMA-fed SGEMM (sgemm_ksplit in
    sgemm_tma.cu), restated to count launches: S in {1, 2, 3, 4, 6, 8} with
    the least estimated time, taken when it saves 5% or more."""
    import math

    tiles = ((m + 127) // 128) * ((n + 255) // 256)
    kt = (k + 31) // 32

    def est(S):
        t = math.ceil(tiles * S / sm_count) * ((kt + S - 1) // S) * 5.2
        if S > 1:
            t += 4.0 * (S + 1) * m * n / 6e12 * 1e6 + 4.0
        return t

    t1 = est(1)
    best, tb = 1, t1
    for S in (2, 3, 4, 6, 8):
        if (kt + S - 1) // S < 8:
            break
        t = est(S)
        if t < tb:
            best, tb = S, t
    return best if tb <= 0.95 * t1 else 1


def dgemm_ksplit(sm_count, m, n, k):
    """The library's split-K choice for the persistent DMMA DGEMM (dgemm_ksplit
    in dgemm_dmma.cu), restated to count launches: 128 x 128 tiles, k-tiles of
    32 at ~4.7 us, a reduce of 8 (S + 1) M N bytes, taken when it saves 5%."""
    import math

    tiles = ((m + 127) // 128) * ((n + 127) // 128)
    kt = (k + 31) // 32

    def est(S):
        t = math.ceil(tiles * S / sm_count) * ((kt + S - 1) // S) * 4.7
        if S > 1:
            t += 8.0 * (S + 1) * m * n / 6e12 * 1e6 + 4.0
        return t

    t1 = est(1)
    best, tb = 1, t1
    for S in (2, 3, 4, 6, 8):
        if (kt + S - 1) // S < 8:
            break
        t = est(S)
        if t < tb:
            best, tb = S, t
    return best if tb <= 0.95 * t1 else 1


def dgemm_kernels_per_call(m, n, k, sm_count=148):
    """Kernels one DGEMM call launches on the DMMA path (K and N even, 16-byte
    aligned operands): the persistent kernel, plus the reduce when split-K
    applies."""
    variant = int(os.environ.get("B2B_DGEMM_VARIANT", "0") or 0)
    if variant != 0 or k % 2 or n % 2:
        return 1
    forced = int(os.environ.get("B2B_DGEMM_KSPLIT", "0") or 0)
    S = forced if forced > 0 else dgemm_ksplit(sm_count, m, n, k)
    return 2 if min(S, (k + 31) // 32) > 1 else 1


def sgemm_kernels_per_call(m, n, k, tf32x3=False, sm_count=148, splits=None):
    """Kernels one single SGEMM call launches on the TMA-fed FFMA path: the
    GEMM (the persistent row-major-A kernel, which transposes A in shared
    memory; variant 0 with K % 4 == 0), else the transpose of A and the
    GEMM, plus the reduce when split-K applies; 1 off that path.  `splits`
    forces the split (a host-slice call's tiles take the whole GEMM's).
    Mirrors the library's dispatch (run_sgemm in gemm_simt.cu,
    sgemm_tma_eligible, sgemm_ksplit and launch_sgemm_tma in sgemm_tma.cu)
    for 16-byte aligned operands."""
    variant = int(os.environ.get("B2B_SGEMM_VARIANT", "0") or 0)
    if tf32x3 or variant not in (0, 20, 21, 22):
        return 1
    rowa = variant == 0 and k % 4 == 0 and n % 4 == 0  # the persistent kernel: any size (sgemm_tma_path)
    transposed = m % 4 == 0 and n % 4 == 0 and (splits is not None or (m >= 128 and n >= 1024)) and \
        32 <= k <= 65535 * 32
    if not (rowa or transposed):
        return 1
    forced = int(os.environ.get("B2B_SGEMM_KSPLIT", "0") or 0)
    S = splits if splits is not None else forced if forced > 0 else sgemm_ksplit(sm_count, m, n, k)
    S = min(S, (k + 31) // 32)
    return (1 if rowa else 2) + (1 if S > 1 else 0)


def sgemm_kernel_name(m, n, k):
    """The dominant kernel of one single SGEMM call (FFMA path)."""
    if int(os.environ.get("B2B_SGEMM_VARIANT", "0") or 0) == 0 and k % 4 == 0 and n % 4 == 0:
        split = sgemm_kernels_per_call(m, n, k) > 1
        return "sgemm_tma_rowa_ws_kernel<true> (persistent; A transposed in shared memory)" + \
            (" + split-K reduce" if split else "")
    return "sgemm_tma_kernel"


def _cur_stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def _pinned_numpy(t):
    """Page-locked host copy of a device tensor, as a numpy array."""
    import numpy as np
    import torch

    h = E2E_HOST["handle"]
    if h is not None:
        np_dt = {torch.float16: np.float16, torch.float32: np.float32, torch.float64: np.float64}[t.dtype]
        arr = h.host_empty(t.numel(), np_dt).reshape(tuple(t.shape))
        arr[...] = t.cpu().numpy()
        return arr, arr
    ht = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=True)
    ht.copy_(t)
    return ht, ht.numpy()


# ------------------------------------------------------ seeded inputs

DATA = ("synthetic: torch CPU generator, one fixed seed per tensor; normal(0,0.1)->f16 for HGEMM, "
        "uniform[-1,1) otherwise")

# Tensor ids of the seeded inputs: seed = INPUT_SEED + 1000 * chunk + id.
INPUT_SEED = 4200
TID = {"A": 1, "B": 2, "C": 3, "x": 4, "bias": 5, "y": 6, "W": 10}
BATCH_CHUNK = 512  # strided-batched inputs are drawn 512 batches at a time


def host_tensor(shape, tid, dtype, dist="uniform", std=0.1, chunk=0):
    """A seeded synthetic input on the host (torch CPU generator): uniform
    [-1, 1) or normal(0, std), then cast to `dtype` (f16 inputs are rounded
    from f32).  Both bench arms call this, so they see the same numbers."""
    import torch

    g = torch.Generator().manual_seed(INPUT_SEED + 1000 * chunk + tid)
    if dist == "normal":
        t = torch.randn(shape, generator=g, dtype=torch.float64 if dtype == torch.float64 else torch.float32) * std
    else:
        t = torch.rand(shape, generator=g, dtype=torch.float64 if dtype == torch.float64 else torch.float32) * 2 - 1
    return t.to(dtype)


def batched_inputs(tid, b0, b1, m):
    """Batches [b0, b1) of a strided-batched operand (m x m per batch), drawn
    in chunks of BATCH_CHUNK batches so that each rank of a batch-sharded run
    only generates its own range."""
    import torch

    parts = []
    c = b0 // BATCH_CHUNK
    while c * BATCH_CHUNK < b1:
        lo, hi = c * BATCH_CHUNK, (c + 1) * BATCH_CHUNK
        t = host_tensor((BATCH_CHUNK, m, m), tid, torch.float32, chunk=c)
        parts.append(t[max(b0, lo) - lo:min(b1, hi) - lo])
        c += 1
    return torch.cat(parts) if len(parts) > 1 else parts[0].contiguous()


def split_range(total, parts, index, align=1):
    """[begin, end) of part `index` of `total` items in `parts` contiguous
    pieces (boundaries multiples of `align`); the same rule as
    b2blas.shard.split_range, restated so the reference arm needs no part of
    the library."""
    units = (total + align - 1) // align
    base, rem = divmod(units, parts)
    b = index * base + min(index, rem)
    e = b + base + (1 if index < rem else 0)
    return min(b * align, total), min(e * align, total)


GEMM_KINDS = ("hgemm", "sgemm", "dgemm")
GEMM_ALPHA_BETA = {"hgemm": (1.0, 0.0), "sgemm": (1.5, 0.5), "dgemm": (1.5, 0.5)}


def gemm_dims(name, args):
    d = 4096 if name == "dgemm" else 8192
    return args.m or d, args.n or d, args.k or d


def gather_mode(name, args, world):
    """The gather a column-sharded GEMM asks for at `world` ranks: None,
    "fused" (peer stores from the GEMM epilogue), "fused-multicast" or
    "nccl".  HGEMM gathers by default on N > 1 GPUs (the fixed 8192^3
    problem, every rank ends with the whole C)."""
    if world <= 1 or name not in GEMM_KINDS:
        return None
    if args.gather_nccl:
        return "nccl"
    if args.gather_multicast:
        return "fused-multicast"
    if args.gather:
        return "fused"
    if args.no_gather or args.weak:
        return None
    return "fused" if name == "hgemm" else None


def workload_config(name, args, world):
    """The `config` record of a workload.  A function of the arguments and the
    world size only, so that both arms print the same dict."""
    if name in GEMM_KINDS:
        m, n, k = gemm_dims(name, args)
        alpha, beta = GEMM_ALPHA_BETA[name]
        weak = bool(args.weak) and name == "hgemm"
        n_glob = n * world if weak else n
        per = n if weak else split_range(n, world, 0, 8)[1]
        g = gather_mode(name, args, world)
        if world > 1:
            how = (f", column-sharded over {world} GPUs ({per} columns per GPU), A replicated"
                   + (", C gathered on every GPU" if g else ""))
        else:
            how = ""
        return {"workload": f"{name} {m}x{n_glob}x{k}" + how, "m": m, "n": n_glob, "k": k, "n_per_gpu": per,
                "alpha": alpha, "beta": beta, "gather": g or False, "parallelism": f"column-shard x{world}",
                "scaling": ("weak" if weak else "strong") if world > 1 else "weak",
                "l2": "inputs larger than L2 (126 MB): no flush needed"}
    if name == "batched":
        nb = getattr(args, "batch", None) or 4096
        b0, b1 = split_range(nb, world, 0)
        return {"workload": f"strided-batched sgemm {nb} x 256^3"
                            + (f", {b1 - b0} batches per GPU" if world > 1 else ""),
                "batch": nb, "batch_per_gpu": b1 - b0, "m": 256, "n": 256, "k": 256,
                "alpha": 1.0, "beta": 0.0, "parallelism": f"batch-shard x{world}",
                "scaling": "strong" if world > 1 else "weak",
                "l2": f"inputs larger than L2 ({3 * nb * 256 * 256 * 4 / 2 ** 30:g} GiB): no flush needed"}
    if name in ("sgemv", "dgemv", "hgemv"):
        esz = {"s": 4, "d": 8, "h": 2}[name[0]]
        gib = 16384 * 16384 * esz / 2 ** 30
        t = "T" if args.trans else "N"
        return {"workload": f"{name} 16384x16384 {t}" + (", one replica per GPU" if world > 1 else ""),
                "m": 16384, "n": 16384, "trans": t, "alpha": 1.0, "beta": 0.0,
                "parallelism": f"replicas x{world}", "scaling": "weak",
                "l2": f"A is {gib:g} GiB, larger than L2: no flush needed"}
    if name == "reduce":
        n = args.n or (1 << 28)
        vec = 2 if args.op == "dot" else 1
        return {"workload": f"s{args.op} n={n}" + (", one replica per GPU" if world > 1 else ""),
                "n": n, "parallelism": f"replicas x{world}", "scaling": "weak",
                "l2": f"{vec} x {n * 4 / 2 ** 30:g} GiB inputs, larger than L2: no flush needed"}
    if name == "mlp":
        how = ("fused sgemm+bias+ReLU epilogue" if args.fused else "sgemm + saxpy bias") + \
            (", 3xTF32" if args.tf32x3 else "")
        streams = 2 if getattr(args, "mlp_streams", 2) == 2 else 1
        return {"workload": f"mlp forward 1024-4096-4096-4096-1024, batch 4096, {how}"
                            + (", two half-batch streams" if streams == 2 else "")
                            + (", one replica per GPU" if world > 1 else ""),
                "layers": [1024, 4096, 4096, 4096, 1024], "batch": 4096, "streams": streams,
                "parallelism": f"replicas x{world}", "scaling": "weak",
                "l2": "weights + activations larger than L2: no flush needed"}
    raise SystemExit(f"unknown workload {name}")


class Workload:
    name = ""
    unit = "TFLOP/s"
    dtype = "f32"
    scaling = "weak"
    launches_per_step = 1
    kernel = ""
    bound = "tensor"
    world = 1
    args = None

    def units_per_step(self):  # flops (or bytes) this rank processes per step
        raise NotImplementedError

    def total_units_per_step(self):  # over all ranks (replicas: world x this rank's)
        return self.units_per_step() * self.world

    def scale(self, v):  # units/s -> unit
        return v / 1e12

    def config(self):
        return workload_config(self.name, self.args, self.world)


class GemmWorkload(Workload):
    """C = alpha*A*B + beta*C with A replicated and B/C column panels."""

    def __init__(self, h, rank, world, args, kind):
        import numpy as np
        import torch

        import b2blas
        from b2blas import shard

        m, n_total, k = gemm_dims(kind, args)
        alpha, beta = GEMM_ALPHA_BETA[kind]
        weak = bool(args.weak) and kind == "hgemm"
        self.name, self.args = kind, args
        self.h, self.kind = h, kind
        self.m, self.k, self.alpha, self.beta = m, k, alpha, beta
        self.world, self.rank = world, rank
        if weak:
            self.n = n_total
            self.widths = [n_total] * world
            self.global_n = n_total * world
            self.scaling = "weak"
        else:
            self.widths = shard.column_panels(n_total, world, 8)
            self.n = self.widths[rank]
            self.global_n = n_total
            self.scaling = "strong" if world > 1 else "weak"
        self.col_off = sum(self.widths[:rank])
        dev = torch.device("cuda", torch.cuda.current_device())
        tdt = {"hgemm": torch.float16, "sgemm": torch.float32, "dgemm": torch.float64}[kind]
        self.dtype = {"hgemm": "f16", "sgemm": "f32", "dgemm": "f64"}[kind]
        self.np_dt = {"hgemm": np.uint16, "sgemm": np.float32, "dgemm": np.float64}[kind]
        # The same seeded host inputs as the reference arm: A replicated; B
        # and C the rank's column panel of the whole problem's (weak: the
        # rank's own panel, drawn with the rank as chunk index).
        dist = "normal" if kind == "hgemm" else "uniform"
        self.A = host_tensor((m, k), TID["A"], tdt, dist).to(dev)
        if weak:
            self.B = host_tensor((k, self.n), TID["B"], tdt, dist, chunk=rank).to(dev)
        else:
            self.B = host_tensor((k, n_total), TID["B"], tdt, dist)[:, self.col_off:self.col_off + self.n] \
                .contiguous().to(dev)
        if beta:
            if weak:
                self.C = host_tensor((m, self.n), TID["C"], tdt, dist, chunk=rank).to(dev)
            else:
                self.C = host_tensor((m, n_total), TID["C"], tdt, dist)[:, self.col_off:self.col_off + self.n] \
                    .contiguous().to(dev)
        else:
            self.C = torch.zeros(m, self.n, device=dev, dtype=tdt)
        bdt = np.uint16 if kind == "hgemm" else self.np_dt
        self.a = b2blas.DeviceBuffer.from_ptr(h, self.A.data_ptr(), m * k, bdt, owner=self.A)
        self.b = b2blas.DeviceBuffer.from_ptr(h, self.B.data_ptr(), k * self.n, bdt, owner=self.B)
        self.c = b2blas.DeviceBuffer.from_ptr(h, self.C.data_ptr(), m * self.n, bdt, owner=self.C)
        self.cfg = b2blas.GemmConfig(m, self.n, k, alpha, beta)
        self.fn = {"hgemm": h.hgemm, "sgemm": h.sgemm_3xtf32 if args.tf32x3 else h.sgemm, "dgemm": h.dgemm}[kind]
        self.simple = {"hgemm": h.hgemm_simple, "dgemm": h.dgemm_simple,
                       "sgemm": h.sgemm_3xtf32_simple if args.tf32x3 else h.sgemm_simple}[kind]
        self.kernel = {"hgemm": "hgemm_tc2_kernel" if m > 128 else "hgemm_tc_kernel",
                       "sgemm": sgemm_kernel_name(m, self.n, k), "dgemm": "dgemm_dmma_ws_kernel<32,3> (persistent)"}[kind]
        self.bound = {"hgemm": "tensor", "sgemm": "fma", "dgemm": "fp64"}[kind]
        if kind == "sgemm" and args.tf32x3:
            self.kernel, self.bound = "sgemm_3xtf32_kernel", "tf32x3"
        # A gathered C: every rank ends each step with the full C.  "fused":
        # the GEMM writes its panel into every rank's C itself
        # (b2b_*gemm_gather through IPC-mapped peer buffers), then a
        # 1-element all-reduce orders the next step behind all ranks' writes.
        # "nccl": GEMM into the panel, NCCL all-gather of the panels,
        # re-layout kernel.
        self.gather = gather_mode(kind, args, world)
        if self.gather == "fused-multicast":
            self.gather = "fused"  # becomes "fused-multicast" below once the multicast object exists
        self.mc = 0
        gemm_kernels = (sgemm_kernels_per_call(m, self.n, k, args.tf32x3) if kind == "sgemm" else
                        dgemm_kernels_per_call(m, self.n, k) if kind == "dgemm" else 1)
        self.launches_per_step = gemm_kernels
        if self.gather == "nccl":
            self.panels = torch.empty(sum(self.widths) * m, device=dev, dtype=tdt)
            self.full = torch.empty(m, sum(self.widths), device=dev, dtype=tdt)
            self.launches_per_step = gemm_kernels + 1  # + the re-layout kernel
        elif self.gather == "fused":
            if args.tf32x3:
                raise SystemExit("--gather with --tf32x3 is not supported")
            if kind == "hgemm" and not beta and args.gather_multicast:
                # NVLink multicast (torch symmetric memory binds one buffer per
                # rank): each output store leaves the GPU once.  Every GPU
                # still receives the (world - 1) other panels, so the step's
                # link bound is the same as with peer stores (measured on 8
                # B200s: 1.67 ms multicast, 1.58 ms peer stores).
                import torch.distributed as dist

                try:
                    import torch.distributed._symmetric_memory as symm

                    self.symm_buf = symm.empty(m * self.global_n, dtype=tdt, device=dev)
                    self.symm_hd = symm.rendezvous(self.symm_buf, dist.group.WORLD.group_name)
                    mc = int(getattr(self.symm_hd, "multicast_ptr", 0) or 0)
                except Exception:  # noqa: BLE001 -- no symmetric memory: peer stores
                    mc = 0
                ok = torch.tensor([1 if mc else 0], device=dev)
                dist.all_reduce(ok, op=dist.ReduceOp.MIN)
                self.mc = mc if ok.item() else 0
            if self.mc:
                self.gather = "fused-multicast"
                self.bar = torch.zeros(1, device=dev)
                self.launches_per_step = 1
                return
            self.peers = shard.PeerBuffers(h, m * self.global_n, bdt)
            if beta:
                host = np.zeros((m, self.global_n), bdt)
                host[:, self.col_off:self.col_off + self.n] = self.C.cpu().numpy().view(bdt)
                h.upload_into(self.peers.buf, host.ravel())
            self.gfn = {"hgemm": h.hgemm_gather, "sgemm": h.sgemm_gather, "dgemm": h.dgemm_gather}[kind]
            self.bar = torch.zeros(1, device=dev)
            # the GEMM's kernels (peer copies of the panel run on copy engines)
            self.launches_per_step = gemm_kernels

    def step(self):
        if self.gather == "fused-multicast":
            import torch.distributed as dist

            self.h.hgemm_gather_multicast(self.cfg, self.a, self.b, self.global_n, self.col_off, self.mc,
                                          self.symm_buf.data_ptr())
            dist.all_reduce(self.bar)
            return
        if self.gather == "fused":
            import torch.distributed as dist

            self.gfn(self.cfg, self.a, self.b, self.global_n, self.col_off, self.peers.ptrs, self.rank)
            dist.all_reduce(self.bar)
            return
        self.fn(self.cfg, self.a, self.b, self.c)
        if self.gather == "nccl":
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.panels, self.C.view(-1))
            esz = self.C.element_size()
            self.h.panels_to_rowmajor(esz, self.m, self.widths, self.panels.data_ptr(), self.full.data_ptr())

    def ref_kernels(self):
        """The reference's kernels for this GEMM (restated in CUDA C), writing
        a scratch copy of C: [(name, launch)]."""
        if self.gather is not None:
            return []
        from baseline import refkernels as R

        self._ref_c = self.C.clone()
        m, n, k, al, be = self.m, self.n, self.k, self.alpha, self.beta
        pa, pb, pc, st = self.A.data_ptr(), self.B.data_ptr(), self._ref_c.data_ptr(), _cur_stream()
        if self.kind == "hgemm":
            return [("hgemm_half", lambda: R.hgemm_half(m, n, k, al, pa, pb, be, pc, st))]
        fn = R.sgemm if self.kind == "sgemm" else R.dgemm
        return [(f"{self.kind}_{name}", (lambda v=v: fn(v, m, n, k, al, pa, pb, be, pc, st)))
                for v, name in R.GEMM_VARIANTS.items()]

    def close(self):
        if self.gather == "fused":
            self.peers.close()
        if self.mc:
            # every rank's stores into the multicast object have landed
            # before any rank releases its buffer
            import torch
            import torch.distributed as dist

            torch.cuda.synchronize()
            dist.barrier()

    def units_per_step(self):
        return 2.0 * self.m * self.n * self.k

    def e2e_setup(self):
        self._hA, self.hA = _pinned_numpy(self.A)
        self._hB, self.hB = _pinned_numpy(self.B)
        self._hC, self.hC = _pinned_numpy(self.C)
        if self.kind == "hgemm":
            self.hA, self.hB, self.hC = (x.view(self.np_dt) for x in (self.hA, self.hB, self.hC))
        self.hA, self.hB, self.hC = (x.reshape(-1) for x in (self.hA, self.hB, self.hC))
        esz = self.A.element_size()
        h2d = (self.m * self.k + self.k * self.n + (self.m * self.n if self.beta else 0)) * esz
        return h2d, self.m * self.n * esz

    def e2e_step(self):
        self.simple(self.cfg, self.hA, self.hB, self.hC)

    def cpu_sample(self, oracle, target_s):
        """Times the host triple loop on a row sample of this rank's problem."""
        import numpy as np

        n, k = self.n, self.k
        B = self.B.cpu().numpy()
        if self.kind == "hgemm":
            B = B.view(np.uint16)
        B = np.ascontiguousarray(B).reshape(-1)
        nt = oracle.num_threads()
        rows = nt
        out = {}
        for attempt in range(2):
            A = np.ascontiguousarray(self.A[:rows].cpu().numpy())
            C = np.ascontiguousarray(self.C[:rows].cpu().numpy())
            if self.kind == "hgemm":
                A, C = A.view(np.uint16).reshape(-1), C.view(np.uint16).reshape(-1)
                bf = np.empty(k * n, np.float32)
                acc = np.empty(rows * n, np.float32)
                t0 = time.perf_counter()
                oracle.cpu_hgemm_rows(rows, n, k, self.alpha, A, B, self.beta, C, bf, acc)
            elif self.kind == "sgemm":
                A, C = A.reshape(-1), C.reshape(-1)
                acc = np.empty(rows * n, np.float32)
                t0 = time.perf_counter()
                oracle.cpu_sgemm_rows(rows, n, k, self.alpha, A, B, self.beta, C, acc)
            else:
                A, C = A.reshape(-1), C.reshape(-1)
                acc = np.empty(rows * n, np.float64)
                t0 = time.perf_counter()
                oracle.cpu_dgemm_rows(rows, n, k, self.alpha, A, B, self.beta, C, acc)
            dt = time.perf_counter() - t0
            out = {"value": 2.0 * rows * n * k / dt / 1e12, "seconds": dt, "rows": rows}
            if attempt == 0:
                per_row = dt / rows
                rows = int(max(nt, min(self.m, target_s / max(per_row, 1e-9))))
                rows = max(nt, rows // nt * nt)
        out["sample"] = (f"first {out['rows']} rows of C ({out['rows']}x{n}x{k}, "
                         f"{2.0 * out['rows'] * n * k / 1e9:.1f} GFLOP), i-k-j host loop")
        return out


class BatchedWorkload(Workload):
    """Strided-batched SGEMM, batch-sharded (no collective)."""

    def __init__(self, h, rank, world, args):
        import torch

        import b2blas
        from b2blas import shard

        self.h = h
        self.name, self.args = "batched", args
        self.total_batch, self.m = getattr(args, "batch", None) or 4096, 256
        b0, b1 = shard.batch_shard(self.total_batch, world, rank)
        self.batch = b1 - b0
        self.world = world
        self.scaling = "strong" if world > 1 else "weak"
        m = self.m
        dev = torch.device("cuda", torch.cuda.current_device())
        self.A = batched_inputs(TID["A"], b0, b1, m).to(dev)
        self.B = batched_inputs(TID["B"], b0, b1, m).to(dev)
        self.C = torch.zeros(self.batch, m, m, device=dev)
        mk = m * m
        self.a = b2blas.DeviceBuffer.from_ptr(h, self.A.data_ptr(), self.batch * mk, "float32", owner=self.A)
        self.b = b2blas.DeviceBuffer.from_ptr(h, self.B.data_ptr(), self.batch * mk, "float32", owner=self.B)
        self.c = b2blas.DeviceBuffer.from_ptr(h, self.C.data_ptr(), self.batch * mk, "float32", owner=self.C)
        self.cfg = b2blas.GemmConfig(m, m, m, 1.0, 0.0)
        self.kernel = "sgemm_tma_rowa_ws_kernel (batched, persistent)"
        self.bound = "fma"

    def step(self):
        mk = self.m * self.m
        self.h.strided_batched_sgemm(self.cfg, self.batch, self.a, mk, self.b, mk, self.c, mk)

    def units_per_step(self):
        return 2.0 * self.batch * self.m ** 3

    def total_units_per_step(self):
        return 2.0 * self.total_batch * self.m ** 3

    def e2e_setup(self):
        self._hA, self.hA = _pinned_numpy(self.A)
        self._hB, self.hB = _pinned_numpy(self.B)
        self._hC, self.hC = _pinned_numpy(self.C)
        self.hA, self.hB, self.hC = (x.reshape(-1) for x in (self.hA, self.hB, self.hC))
        n = self.batch * self.m * self.m * 4
        return 2 * n, n

    def e2e_step(self):
        mk = self.m * self.m
        self.h.strided_batched_sgemm_simple(self.cfg, self.batch, self.hA, mk, self.hB, mk, self.hC, mk)

    def ref_kernels(self):
        from baseline import refkernels as R

        self._ref_c = self.C.clone()
        m, mk, nb = self.m, self.m * self.m, self.batch
        pa, pb, pc, st = self.A.data_ptr(), self.B.data_ptr(), self._ref_c.data_ptr(), _cur_stream()
        return [("strided_batched_sgemm", lambda: R.sgemm_strided_batched(m, m, m, 1.0, pa, mk, pb, mk, 0.0, pc, mk,
                                                                          nb, st))]

    def cpu_sample(self, oracle, target_s):
        import numpy as np

        m = self.m
        nb = 1
        out = {}
        for attempt in range(2):
            A = self.A[:nb].cpu().numpy().reshape(-1)
            B = self.B[:nb].cpu().numpy()
            C = np.zeros(nb * m * m, np.float32)
            acc = np.empty(m * m, np.float32)
            t0 = time.perf_counter()
            for i in range(nb):
                oracle.cpu_sgemm_rows(m, m, m, 1.0, np.ascontiguousarray(A[i * m * m:(i + 1) * m * m]),
                                      np.ascontiguousarray(B[i].reshape(-1)), 0.0, C[i * m * m:(i + 1) * m * m], acc)
            dt = time.perf_counter() - t0
            out = {"value": 2.0 * nb * m ** 3 / dt / 1e12, "seconds": dt, "batches": nb}
            if attempt == 0:
                nb = int(max(1, min(self.batch, target_s / max(dt, 1e-9))))
        out["sample"] = f"first {out['batches']} of the {self.total_batch} 256^3 batches, i-k-j host loop"
        return out


class GemvWorkload(Workload):
    """GEMV 16384 x 16384, N or T, alpha 1, beta 0 (replicas on N GPUs), in
    f32 (sgemv), f64 (dgemv) or f16 with f32 accumulate (hgemv)."""

    unit = "GB/s"
    bound = "hbm"

    def __init__(self, h, rank, world, args, prec="s"):
        import numpy as np
        import torch

        import b2blas

        self.h, self.world, self.prec = h, world, prec
        self.name, self.args = prec + "gemv", args
        self.m = self.n = 16384
        self.trans = 1 if args.trans else 0
        tdt, ndt, self.esize, self.dtype = {"s": (torch.float32, "float32", 4, "f32"),
                                           "d": (torch.float64, "float64", 8, "f64"),
                                           "h": (torch.float16, "uint16", 2, "f16")}[prec]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.A = host_tensor((self.m, self.n), TID["A"], tdt).to(dev)
        xl, yl = (self.n, self.m) if self.trans == 0 else (self.m, self.n)
        self.x = host_tensor((xl,), TID["x"], tdt).to(dev)
        self.y = torch.zeros(yl, device=dev, dtype=tdt)
        buf = lambda t, n: b2blas.DeviceBuffer.from_ptr(h, t.data_ptr(), n, ndt, owner=t)  # noqa: E731
        self.a, self.xd, self.yd = buf(self.A, self.m * self.n), buf(self.x, xl), buf(self.y, yl)
        if prec == "s":
            self.kernel = "sgemv_n_kernel" if self.trans == 0 else "sgemv_t_partial_kernel"
            self.fn = h.sgemv
        else:
            self.kernel = "gemvx_n_kernel" if self.trans == 0 else "gemvx_t_partial_kernel"
            self.fn = h.dgemv if prec == "d" else h.hgemv_dev
        self.launches_per_step = 1 if self.trans == 0 else 2
        self._np = np

    def step(self):
        self.fn(self.trans, self.m, self.n, 1.0, self.a, self.xd, 0.0, self.yd)

    def units_per_step(self):
        return float(self.esize) * (self.m * self.n + self.m + self.n)

    def scale(self, v):
        return v / 1e9

    def e2e_setup(self):
        self._hA, self.hA = _pinned_numpy(self.A)
        self._hx, self.hx = _pinned_numpy(self.x)
        self._hy, self.hy = _pinned_numpy(self.y)
        self.hA = self.hA.reshape(-1)
        if self.prec == "h":  # numpy float16 views of the pinned buffers
            self.hA, self.hx, self.hy = (a.view(self._np.float16) for a in (self.hA, self.hx, self.hy))
        e = self.esize
        return e * (self.m * self.n + len(self.hx)), e * len(self.hy)

    def e2e_step(self):
        fn = {"s": self.h.sgemv_simple, "d": self.h.dgemv_simple, "h": self.h.hgemv}[self.prec]
        fn(self.trans, self.m, self.n, 1.0, self.hA, self.hx, 0.0, self.hy)

    def ref_kernels(self):
        from baseline import refkernels as R

        self._ref_y = self.y.clone()
        t, m, n = self.trans, self.m, self.n
        pa, px, py, st = self.A.data_ptr(), self.x.data_ptr(), self._ref_y.data_ptr(), _cur_stream()
        if self.prec == "s":
            return [(f"sgemv_{name}", (lambda v=v: R.sgemv(v, t, m, n, 1.0, pa, px, 0.0, py, st)))
                    for v, name in ((0, "naive"), (1, "tiled"))]
        if self.prec == "d":
            return [("dgemv", lambda: R.dgemv(t, m, n, 1.0, pa, px, 0.0, py, st))]
        return [("hgemv", lambda: R.hgemv(t, m, n, 1.0, pa, px, 0.0, py, st))]

    def cpu_sample(self, oracle, target_s):
        np = self._np
        n = self.n
        x = self.x.cpu().numpy()
        if self.prec == "h":
            x = x.view(np.uint16)
        xf = np.empty(n, np.float32)
        rows = 256
        out = {}
        for attempt in range(2):
            A = np.ascontiguousarray(self.A[:rows].cpu().numpy()).reshape(-1)
            if self.prec == "h":
                A = A.view(np.uint16)
            y = np.zeros(rows, A.dtype)
            t0 = time.perf_counter()
            reps = 0
            while True:
                if self.prec == "s":
                    oracle.cpu_sgemv_rows(rows, n, 1.0, A, x, 0.0, y)
                elif self.prec == "d":
                    oracle.cpu_dgemv_rows(rows, n, 1.0, A, x, 0.0, y)
                else:
                    oracle.cpu_hgemv_rows(rows, n, 1.0, A, x, 0.0, y, xf)
                reps += 1
                if time.perf_counter() - t0 > (0.2 if attempt == 0 else target_s):
                    break
            dt = time.perf_counter() - t0
            out = {"value": reps * float(self.esize) * (rows * n + n + rows) / dt / 1e9, "seconds": dt,
                   "rows": rows}
            if attempt == 0:
                rows = min(self.m, 4096)
        out["sample"] = f"{out['rows']} rows x {n} (repeated for ~{target_s:.0f} s), row loop"
        return out


class ReduceWorkload(Workload):
    """Level-1 reduction (sdot by default) over 2^28-element f32 vectors
    (1 GiB each), result kept on the device (b2b_sreduce_async)."""

    unit = "GB/s"
    bound = "hbm"
    kernel = "sreduce_kernel"

    def __init__(self, h, rank, world, args):
        import torch

        import b2blas

        self.h, self.world = h, world
        self.name, self.args = "reduce", args
        self.op = args.op
        self.n = args.n or (1 << 28)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.x = host_tensor((self.n,), TID["x"], torch.float32).to(dev)
        self.y = host_tensor((self.n,), TID["y"], torch.float32).to(dev) if self.op == "dot" else None
        self.res = torch.zeros(1, device=dev, dtype=torch.int64 if self.op == "iamax" else torch.float32)
        self.xd = b2blas.DeviceBuffer.from_ptr(h, self.x.data_ptr(), self.n, "float32", owner=self.x)
        self.yd = (b2blas.DeviceBuffer.from_ptr(h, self.y.data_ptr(), self.n, "float32", owner=self.y)
                   if self.y is not None else None)
        self.rd = b2blas.DeviceBuffer.from_ptr(h, self.res.data_ptr(), 1,
                                               "uint64" if self.op == "iamax" else "float32", owner=self.res)
        self.opcode = {"dot": 0, "nrm2": 1, "asum": 2, "iamax": 3}[self.op]
        self.vectors = 2 if self.op == "dot" else 1
        self.dtype = "f32"

    def step(self):
        self.h.sreduce_async(self.opcode, self.n, self.xd, self.yd, self.rd)

    def units_per_step(self):
        return 4.0 * self.n * self.vectors

    def scale(self, v):
        return v / 1e9

    def e2e_setup(self):
        self._hx, self.hx = _pinned_numpy(self.x)
        if self.y is not None:
            self._hy, self.hy = _pinned_numpy(self.y)
        return 4 * self.n * self.vectors, 8 if self.op == "iamax" else 4

    def e2e_step(self):
        h = self.h
        if self.op == "dot":
            h.sdot_simple(self.n, self.hx, self.hy)
        else:
            getattr(h, {"nrm2": "snrm2_simple", "asum": "sasum_simple", "iamax": "isamax_simple"}[self.op])(
                self.n, self.hx)

    def ref_kernels(self):
        import torch

        from baseline import refkernels as R

        self._ref_out = torch.zeros(1, device=self.x.device, dtype=torch.float32)
        n, px, st = self.n, self.x.data_ptr(), _cur_stream()
        py, po, op = (self.y.data_ptr() if self.y is not None else 0), self._ref_out.data_ptr(), self.op
        return [("s" + op if op != "iamax" else "isamax", lambda: R.sreduce(op, n, px, py, po, st))]

    def cpu_sample(self, oracle, target_s):
        import numpy as np

        n = min(self.n, 1 << 26)
        x = self.x[:n].cpu().numpy()
        y = self.y[:n].cpu().numpy() if self.y is not None else x
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < target_s:
            if self.op == "dot":
                oracle.cpu_sdot(n, x, y)
            elif self.op == "iamax":
                oracle.isamax(n, x)
            else:
                oracle.sreduce_ref(self.op, n, x)
            reps += 1
        dt = time.perf_counter() - t0
        threads = oracle.num_threads() if self.op == "dot" else 1
        return {"value": reps * 4.0 * n * self.vectors / dt / 1e9, "seconds": dt, "threads": threads,
                "sample": f"first {n} elements (repeated for ~{target_s:.0f} s), "
                          + ("threaded f32 partial sums" if self.op == "dot" else "single-thread loop")}


def mlp_weight(i, fi, fo):
    """Layer i's weights, normal(0, 1/sqrt(fan_in)), on the host."""
    import torch

    return host_tensor((fi, fo), TID["W"] + i, torch.float32, "normal", std=1.0 / fi ** 0.5)


def mlp_bias(i, fo):
    """Layer i's bias vector, normal(0, 0.01), on the host."""
    import torch

    return host_tensor((fo,), TID["bias"], torch.float32, "normal", std=0.01, chunk=i)


class MlpWorkload(Workload):
    """Resident-weight fp32 MLP forward: 4 x (sgemm + saxpy bias), batch 4096."""

    def __init__(self, h, rank, world, args):
        import torch

        import b2blas

        self.h, self.world = h, world
        self.name, self.args = "mlp", args
        self.dims = [1024, 4096, 4096, 4096, 1024]
        self.batch = 4096
        dev = torch.device("cuda", torch.cuda.current_device())
        self.X = host_tensor((self.batch, self.dims[0]), TID["x"], torch.float32).to(dev)
        self.W, self.bias, self.Z = [], [], []
        for i in range(4):
            fi, fo = self.dims[i], self.dims[i + 1]
            self.W.append(mlp_weight(i, fi, fo).to(dev))
            b = mlp_bias(i, fo).to(dev)
            self.bias.append(b.repeat(self.batch, 1).contiguous())  # pre-broadcast, as the example does
            self.Z.append(torch.empty(self.batch, fo, device=dev))
        wrap = lambda t: b2blas.DeviceBuffer.from_ptr(h, t.data_ptr(), t.numel(), "float32", owner=t)  # noqa
        self.xb = wrap(self.X)
        self.wb = [wrap(t) for t in self.W]
        self.bb = [wrap(t) for t in self.bias]
        self.zb = [wrap(t) for t in self.Z]
        self.bias_vec = [t[0].contiguous() for t in self.bias]
        self.bvec = [wrap(t) for t in self.bias_vec]
        self.fused = bool(args.fused)
        self.algo = b2blas.Algo.Tf32x3 if args.tf32x3 else b2blas.Algo.Default
        # --mlp-streams 2: the batch as two halves, each on its own stream and
        # handle (rows of a GEMM are independent, so the results are the same
        # bits); one half's GEMM tail overlaps the other half's kernels.
        self.streams = 2 if getattr(args, "mlp_streams", 2) == 2 else 1
        self.lanes = [(h, 0, self.batch)]
        if self.streams == 2:
            half = self.batch // 2
            self.s2 = torch.cuda.Stream()
            self.h2 = b2blas.Handle(torch.cuda.current_device())
            self.h2.set_stream(self.s2.cuda_stream)
            self.lanes = [(h, 0, half), (self.h2, half, self.batch - half)]
            self.ev_start, self.ev_done = torch.cuda.Event(), torch.cuda.Event()
        # per lane: (handle, rows) -> buffers over that lane's rows
        self.lane_bufs = []
        for lh, r0, rows in self.lanes:
            lw = lambda t, lh=lh: b2blas.DeviceBuffer.from_ptr(lh, t.data_ptr(), t.numel(), "float32", owner=t)  # noqa
            self.lane_bufs.append({"x": lw(self.X[r0:r0 + rows]), "w": [lw(t) for t in self.W],
                                   "b": [lw(t[r0:r0 + rows]) for t in self.bias], "bv": [lw(t) for t in self.bias_vec],
                                   "z": [lw(t[r0:r0 + rows]) for t in self.Z]})
        self.whole_splits = [h.sgemm_splits(self.batch, self.dims[i + 1], self.dims[i]) for i in range(4)]
        per_gemm = [(1 if args.tf32x3 else
                     sgemm_kernels_per_call(rows, self.dims[i + 1], self.dims[i], splits=self.whole_splits[i])
                     if self.whole_splits[i] > 1 else
                     sgemm_kernels_per_call(rows, self.dims[i + 1], self.dims[i]))
                    for _, _, rows in self.lanes for i in range(4)]
        self.launches_per_step = sum(per_gemm) + (0 if self.fused else 4 * self.streams)  # + a saxpy per layer
        names = sorted({sgemm_kernel_name(rows, self.dims[i + 1], self.dims[i]).split(" (")[0]
                        for _, _, rows in self.lanes for i in range(4)})
        self.kernel = " + ".join(names)
        self.bound = "fma"

    def forward(self, xb):
        import torch

        import b2blas

        if self.streams == 2:  # the second lane starts behind the step's earlier work
            self.ev_start.record(torch.cuda.current_stream())
            self.s2.wait_event(self.ev_start)
        for li, (lh, r0, rows) in enumerate(self.lanes):
            bufs = self.lane_bufs[li]
            inp = xb if self.streams == 1 else bufs["x"]
            for i in range(4):
                fi, fo = self.dims[i], self.dims[i + 1]
                cfg = b2blas.GemmConfig(rows, fo, fi, 1.0, 0.0)
                if self.streams == 2:
                    # each half sums the k ranges of the whole-batch GEMM
                    # (its split-K factor), so two lanes give one lane's bits
                    lh.set_sgemm_splits(self.whole_splits[i])
                if self.fused:
                    # bias (and, for hidden layers, ReLU) in the GEMM epilogue
                    lh.sgemm_bias(cfg, inp, bufs["w"][i], bufs["z"][i], bufs["bv"][i], relu=i < 3, algo=self.algo)
                else:
                    # the example's pattern: sgemm + saxpy of the pre-broadcast bias
                    lh.sgemm_tiled(cfg, inp, bufs["w"][i], bufs["z"][i])
                    lh.saxpy(rows * fo, 1.0, bufs["b"][i], bufs["z"][i])
                inp = bufs["z"][i]
            if self.streams == 2:
                lh.set_sgemm_splits(0)
        if self.streams == 2:  # and the step ends behind it
            self.ev_done.record(self.s2)
            torch.cuda.current_stream().wait_event(self.ev_done)

    def step(self):
        self.forward(self.xb)

    def units_per_step(self):
        return sum(2.0 * self.batch * self.dims[i] * self.dims[i + 1] for i in range(4))

    def e2e_setup(self):
        import torch

        self._hX, self.hX = _pinned_numpy(self.X)
        self._hY = torch.empty(self.Z[-1].shape, dtype=torch.float32, pin_memory=True)
        return self.X.numel() * 4, self.Z[-1].numel() * 4

    def e2e_step(self):
        import torch

        self.X.copy_(torch.from_numpy(self.hX), non_blocking=True)
        self.forward(self.xb)
        self._hY.copy_(self.Z[-1], non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def ref_kernels(self):
        """The example's forward on the reference's kernels: sgemm_tiled + saxpy
        of the pre-broadcast bias per layer, into scratch activations."""
        from baseline import refkernels as R

        self._ref_z = [z.clone() for z in self.Z]
        st, b, d = _cur_stream(), self.batch, self.dims
        ptrs = [self.X.data_ptr()] + [z.data_ptr() for z in self._ref_z]

        def forward():
            for i in range(4):
                R.sgemm(1, b, d[i + 1], d[i], 1.0, ptrs[i], self.W[i].data_ptr(), 0.0, ptrs[i + 1], st)
                R.saxpy(b * d[i + 1], 1.0, self.bias[i].data_ptr(), ptrs[i + 1], st)

        return [("sgemm_tiled + saxpy (mlp forward)", forward)]

    def close(self):
        if self.streams == 2:
            import torch

            torch.cuda.synchronize()
            self.h2.set_stream(None)
            self.h2.close()

    def cpu_sample(self, oracle, target_s):
        import numpy as np

        rows = oracle.num_threads()
        t0 = time.perf_counter()
        flops = 0.0
        inp = np.ascontiguousarray(self.X[:rows].cpu().numpy()).reshape(-1)
        for i in range(4):
            fi, fo = self.dims[i], self.dims[i + 1]
            W = self.W[i].cpu().numpy().reshape(-1)
            z = np.zeros(rows * fo, np.float32)
            acc = np.empty(rows * fo, np.float32)
            oracle.cpu_sgemm_rows(rows, fo, fi, 1.0, inp, W, 0.0, z, acc)
            z += np.tile(self.bias[i][0].cpu().numpy(), rows)
            flops += 2.0 * rows * fi * fo
            inp = z
        dt = time.perf_counter() - t0
        return {"value": flops / dt / 1e12, "seconds": dt,
                "sample": f"{rows} rows of the batch through all 4 layers, i-k-j host loop"}


def make_workload(name, h, rank, world, args):
    if name in GEMM_KINDS:
        return GemmWorkload(h, rank, world, args, name)
    if name == "batched":
        return BatchedWorkload(h, rank, world, args)
    if name in ("sgemv", "dgemv", "hgemv"):
        return GemvWorkload(h, rank, world, args, prec=name[0])
    if name == "reduce":
        return ReduceWorkload(h, rank, world, args)
    if name == "mlp":
        return MlpWorkload(h, rank, world, args)
    raise SystemExit(f"unknown workload {name}")


# ----------------------------------------------------------------- peaks

def roofline_peak(w, peaks, handle_info, mhz=None):
    """(peak value, unit, source) for the workload's dominant kernel.  The
    FP32 / FP64 pipe peaks are computed from the SM count and a clock: `mhz`
    (the median SM clock sampled during the timed region) when given, else
    the maximum SM clock."""
    if w.bound == "tensor":
        return peaks["bf16_tflops"], "TFLOP/s", \
            f"dense f16/bf16 tensor, cuBLAS bf16 burst, {peaks['_source']}"
    if w.bound == "tf32x3":
        # three tf32 MMAs per product: the dense tf32 rate (half the f16/bf16
        # rate) divided by 3, in FP32-equivalent flops
        return peaks["bf16_tflops"] / 2 / 3, "TFLOP/s", \
            f"dense tf32 = bf16/2 of the cuBLAS bf16 burst, /3 for the three MMAs, {peaks['_source']}"
    if w.bound == "hbm":
        return peaks["hbm_gbs"], "GB/s", f"HBM copy bandwidth, {peaks['_source']}"
    sms = handle_info["sm_count"]
    sampled = mhz is not None
    mhz = float(mhz) if sampled else float(peaks.get("sm_max_mhz", 1965.0))
    lanes = 64 if w.dtype == "f64" else 128
    what = "FP64 (DMMA = DFMA rate)" if w.bound == "fp64" else "FP32 FFMA"
    return sms * lanes * 2 * mhz * 1e6 / 1e12, "TFLOP/s", \
        (f"computed {what} peak: {sms} SMs x {lanes} FMA/clk x 2 x {mhz:.0f} MHz "
         + ("(median SM clock sampled during the timed region)" if sampled else "(maximum SM clock)")
         + "; no measured figure for this pipe in MEASURED_PEAKS.json")


# ------------------------------------------------------------ reference

def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the reference's algorithm
    (the oracle's host loops), rank 0 only, a bounded sample per step, on
    the same seeded inputs (host_tensor) and with the same config record as
    the library arm at this world size."""
    if rank != 0:
        return 0
    import numpy as np
    import torch

    from oracle import oracle

    oracle.set_num_threads(os.cpu_count() or 1)
    nt = oracle.num_threads()
    wl = args.workload
    cfg = workload_config(wl, args, world)
    per_step = 1.5  # seconds of CPU work per step
    if wl in GEMM_KINDS:
        m, n, k = cfg["m"], cfg["n"], cfg["k"]
        alpha, beta = GEMM_ALPHA_BETA[wl]
        tdt = {"hgemm": torch.float16, "sgemm": torch.float32, "dgemm": torch.float64}[wl]
        dist = "normal" if wl == "hgemm" else "uniform"
        # The whole problem's B (weak: rank 0's panel, the others' are drawn
        # the same way); A and C are read by row sample.
        weak = cfg.get("scaling") == "weak" and world > 1
        nb = n // world if weak else n
        Afull = host_tensor((m, k), TID["A"], tdt, dist).numpy()
        B = np.ascontiguousarray(host_tensor((k, nb), TID["B"], tdt, dist).numpy()).reshape(-1)
        Cfull = host_tensor((m, nb), TID["C"], tdt, dist).numpy() if beta else np.zeros((m, nb), Afull.dtype)
        if wl == "hgemm":
            Afull, B, Cfull = Afull.view(np.uint16), B.view(np.uint16), Cfull.view(np.uint16)
        n = nb

        def run(rows):
            A = np.ascontiguousarray(Afull[:rows]).reshape(-1)
            C = np.ascontiguousarray(Cfull[:rows]).reshape(-1)
            if wl == "hgemm":
                bf, acc = np.empty(k * n, np.float32), np.empty(rows * n, np.float32)
                t0 = time.perf_counter()
                oracle.cpu_hgemm_rows(rows, n, k, alpha, A, B, beta, C, bf, acc)
            elif wl == "sgemm":
                acc = np.empty(rows * n, np.float32)
                t0 = time.perf_counter()
                oracle.cpu_sgemm_rows(rows, n, k, alpha, A, B, beta, C, acc)
            else:
                acc = np.empty(rows * n)
                t0 = time.perf_counter()
                oracle.cpu_dgemm_rows(rows, n, k, alpha, A, B, beta, C, acc)
            return time.perf_counter() - t0, 2.0 * rows * n * k

        dt, _ = run(nt)
        rows = max(nt, int(per_step / max(dt / nt, 1e-9)) // nt * nt)
        rows = min(rows, m)
        unit = "TFLOP/s"
        sample = f"{rows} of {m} rows of C per step ({rows}x{n}x{k}), i-k-j host loop, {nt} threads"
        step = lambda: run(rows)  # noqa: E731
        scale = 1e12
        dtype = {"hgemm": "f16", "sgemm": "f32", "dgemm": "f64"}[wl]
    elif wl == "batched":
        m = 256
        A = batched_inputs(TID["A"], 0, BATCH_CHUNK, m).numpy()
        B = batched_inputs(TID["B"], 0, BATCH_CHUNK, m).numpy()
        C = np.zeros(m * m, np.float32)
        acc = np.empty(m * m, np.float32)
        state = {"i": 0}

        def run1():
            i = state["i"] % BATCH_CHUNK
            state["i"] += 1
            a, b = np.ascontiguousarray(A[i]).reshape(-1), np.ascontiguousarray(B[i]).reshape(-1)
            t0 = time.perf_counter()
            oracle.cpu_sgemm_rows(m, m, m, 1.0, a, b, 0.0, C, acc)
            return time.perf_counter() - t0

        nb = max(1, min(BATCH_CHUNK, int(per_step / max(run1(), 1e-9))))

        def step():
            state["i"] = 0
            t = sum(run1() for _ in range(nb))
            return t, 2.0 * nb * m ** 3

        unit, scale, dtype = "TFLOP/s", 1e12, "f32"
        sample = f"the first {nb} of the 4096 256^3 batches per step, i-k-j host loop, {nt} threads"
    elif wl in ("sgemv", "dgemv", "hgemv"):
        n = 16384
        rows = 4096 if wl == "sgemv" else 2048
        tdt = {"s": torch.float32, "d": torch.float64, "h": torch.float16}[wl[0]]
        trans = 1 if args.trans else 0
        Afull = host_tensor((16384, n), TID["A"], tdt).numpy()
        x = host_tensor((n,), TID["x"], tdt).numpy()
        # N: the first rows of A; T: y_j = sum_i A[i][j] x[i] over the first
        # columns, i.e. the same row loop over rows of A^T
        A = np.ascontiguousarray(Afull[:, :rows].T if trans else Afull[:rows]).reshape(-1)
        if wl == "hgemv":
            A, x = A.view(np.uint16), x.view(np.uint16)
            y = np.zeros(rows, np.uint16)
            xf = np.empty(n, np.float32)
        else:
            y = np.zeros(rows, A.dtype)
        es = {"s": 4, "d": 8, "h": 2}[wl[0]]

        def step():
            t0 = time.perf_counter()
            if wl == "sgemv":
                oracle.cpu_sgemv_rows(rows, n, 1.0, A, x, 0.0, y)
            elif wl == "dgemv":
                oracle.cpu_dgemv_rows(rows, n, 1.0, A, x, 0.0, y)
            else:
                oracle.cpu_hgemv_rows(rows, n, 1.0, A, x, 0.0, y, xf)
            return time.perf_counter() - t0, float(es) * (rows * n + n + rows)

        unit, scale, dtype = "GB/s", 1e9, {"s": "f32", "d": "f64", "h": "f16"}[wl[0]]
        sample = f"{rows} of 16384 rows per step, row loop, {nt} threads"
    elif wl == "reduce":
        n = min(cfg["n"], 1 << 26)
        x = host_tensor((cfg["n"],), TID["x"], torch.float32)[:n].numpy()
        y = host_tensor((cfg["n"],), TID["y"], torch.float32)[:n].numpy() if args.op == "dot" else x
        op = args.op
        vec = 2 if op == "dot" else 1

        def step():
            t0 = time.perf_counter()
            if op == "dot":
                oracle.cpu_sdot(n, x, y)
            elif op == "iamax":
                oracle.isamax_ref(n, x)
            else:
                oracle.sreduce_ref(op, n, x)
            return time.perf_counter() - t0, 4.0 * n * vec

        unit, scale, dtype = "GB/s", 1e9, "f32"
        if op != "dot":
            nt = 1
        sample = (f"first {n} elements per step, "
                  + (f"threaded f32 partial sums, {nt} threads" if op == "dot" else "the reference's 32-lane loop, 1 thread"))
    else:
        dims = [1024, 4096, 4096, 4096, 1024]
        Ws = [mlp_weight(i, dims[i], dims[i + 1]).numpy().reshape(-1) for i in range(4)]
        bs = [mlp_bias(i, dims[i + 1]).numpy() for i in range(4)]
        rows = nt * 4
        X = host_tensor((4096, dims[0]), TID["x"], torch.float32).numpy()
        state = {"r": 0}

        def step():
            r0 = state["r"] % (4096 // rows) * rows
            state["r"] += 1
            inp = np.ascontiguousarray(X[r0:r0 + rows]).reshape(-1)
            t0 = time.perf_counter()
            fl = 0.0
            for i in range(4):
                z = np.zeros(rows * dims[i + 1], np.float32)
                acc = np.empty_like(z)
                oracle.cpu_sgemm_rows(rows, dims[i + 1], dims[i], 1.0, inp, Ws[i], 0.0, z, acc)
                z += np.tile(bs[i], rows)  # the example's saxpy of the pre-broadcast bias
                fl += 2.0 * rows * dims[i] * dims[i + 1]
                inp = z
            return time.perf_counter() - t0, fl

        unit, scale, dtype = "TFLOP/s", 1e12, "f32"
        sample = f"{rows} rows of the batch-4096 forward per step (sgemm + saxpy bias), i-k-j host loop, {nt} threads"

    for _ in range(args.warmup):
        step()
    tt, uu = 0.0, 0.0
    for _ in range(args.steps):
        t, u = step()
        tt += t
        uu += u
    value = uu / tt / scale
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tt / args.steps * 1e3,
            "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None, "dtype": dtype,
            "data": DATA, "config": cfg,
            "cpu_baseline": {"value": value, "unit": unit, "cores": nt, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference = CPU restatement of cublas-rs's kernels (Rust/cuda-oxide cannot be built here)"}
    print(json.dumps(line), flush=True)
    return 0


def run_e2e(w, h, stream, steps, world, dist, barrier, host_alloc="b2b"):
    """The same metric through the host-slice API: page-locked host inputs
    copied in and the result copied out inside every timed step."""
    import torch

    h2d, d2h = w.e2e_setup()
    # Warm-up: staging allocation, and the host-slice GEMMs' first two large
    # calls, which measure the phased and full-duplex copy schedules.
    w.e2e_step()
    w.e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        w.e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    value = w.scale(w.total_units_per_step() * steps / (float(t.item()) / 1e3))
    return {"value": value, "unit": w.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "api": "host-slice (_simple) calls on page-locked host buffers",
            "host_alloc": "b2b_host_alloc (cudaHostAlloc)" if host_alloc == "b2b" else "torch pin_memory"}


# ------------------------------------------------------------------ main

def time_ref_kernels(w, stream, budget_ms=2500.0, max_launches=10):
    """Times the reference's kernels (restated in CUDA C, baseline/) on this
    workload's resident buffers: one untimed launch, then as many launches as
    fit in about budget_ms (at least one), CUDA events on `stream`."""
    import torch

    try:
        launchers = w.ref_kernels() if hasattr(w, "ref_kernels") else []
    except (OSError, RuntimeError, ImportError) as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}
    if not launchers:
        return None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    for name, fn in launchers:
        fn()
        torch.cuda.synchronize()
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        first = e0.elapsed_time(e1)
        reps = max(1, min(max_launches, int(budget_ms / max(first, 1e-3))))
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        results.append({"kernel": name, "value": w.scale(w.units_per_step() / (ms / 1e3)), "ms_per_launch": ms,
                        "launches": reps})
    best = max(results, key=lambda r: r["value"])
    return {"impl": "the reference's GPU kernels restated in CUDA C (baseline/refkernels.cu), "
                    "same resident device buffers, same B200", "unit": w.unit, "results": results,
            "best_kernel": best["kernel"], "best_value": best["value"]}


def timed_region(w, stream, steps, dist, barrier, local):
    """K steps of `w` between a barrier + synchronize on both sides, CUDA
    events on the launch stream, NVML clocks sampled meanwhile.  Returns
    (this rank's ms, max-over-ranks ms, clock summary)."""
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    with sampler:
        start.record(stream)
        for _ in range(steps):
            w.step()
        end.record(stream)
        torch.cuda.synchronize()
    w.h.synchronize()  # raises if a bounded device wait gave up
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    barrier()
    return ms, ms_max, sampler.summary()


def secondary_names(args, world):
    """The metric's other configurations, measured after the headline one."""
    if args.no_secondary or args.workload != "hgemm" or args.m or args.n or args.k:
        return []
    if world == 1:
        return ["sgemm", "sgemv", "batched", "dgemm"]
    # the column-sharded FP32/FP64 problems (fixed 8192^3 / 4096^3, A
    # replicated), without and with the gathered C
    return ["batched", "hgemm-weak", "sgemm", "sgemm-gather", "dgemm"]


def run_secondary(names, h, stream, rank, world, dist, barrier, local, args, peaks, info):
    """Each secondary configuration in its own timed region: 3 warm-up steps,
    then at least --steps steps and at least ~50 ms of device time."""
    import copy
    import math

    import torch

    out = []
    for name in names:
        sa = copy.copy(args)
        sa.trans = sa.tf32x3 = sa.gather = sa.gather_nccl = sa.gather_multicast = False
        sa.no_gather, sa.weak = True, name == "hgemm-weak"
        if name.endswith("-gather"):
            sa.gather, sa.no_gather = True, False
        sa.m = sa.n = sa.k = sa.batch = None
        wname = name.split("-")[0]
        sa.workload = wname
        w = make_workload(wname, h, rank, world, sa)
        torch.cuda.synchronize()
        for _ in range(3):
            w.step()
        barrier()
        # one step's duration sets the count (the same on every rank)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        w.step()
        e1.record(stream)
        torch.cuda.synchronize()
        est = torch.tensor([e0.elapsed_time(e1)], device="cuda", dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(est, op=dist.ReduceOp.MAX)
        steps = int(min(4000, max(args.steps, math.ceil(50.0 / max(float(est.item()), 1e-3)))))
        ms, ms_max, clocks = timed_region(w, stream, steps, dist, barrier, local)
        value = w.scale(w.total_units_per_step() * steps / (ms_max / 1e3))
        per_launch = ms / steps
        achieved = w.scale(w.units_per_step() / (per_launch / 1e3))
        mhz = clocks.get("sm_mhz") if w.bound in ("fma", "fp64") else None
        peak, punit, psrc = roofline_peak(w, peaks, info, mhz)
        rec = {"name": name, "config": w.config(), "metric": f"{w.unit} ({w.dtype})", "value": value,
               "unit": w.unit, "dtype": w.dtype, "steps": steps, "warmup": 3, "ms_per_step": ms_max / steps,
               "scaling": w.scaling, "kernel": w.kernel, "gpu_launches": w.launches_per_step * steps,
               "roofline": {"bound": {"hbm": "hbm", "tensor": "tensor", "fp64": "fp64"}.get(w.bound, "fma"),
                            "achieved": achieved, "peak": peak, "unit": punit, "frac": achieved / peak,
                            "peak_source": psrc, "ms_per_launch": per_launch,
                            "algorithmic_units_per_launch": w.units_per_step(),
                            "traffic": None if world > 1 and name != "batched" else load_traffic().get(wname)},
               "clocks": clocks}
        if w.bound in ("fma", "fp64"):
            pmax, _, _ = roofline_peak(w, peaks, info)
            rec["roofline"]["frac_at_max_clock"] = achieved / pmax
        if world > 1 and name == "batched" and rec["roofline"]["traffic"]:
            rec["roofline"]["traffic"] = rec["roofline"]["traffic"] * w.batch / w.total_batch
        out.append(rec)
        if hasattr(w, "close"):
            w.close()
        del w
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b2blas", "reference"], default="b2blas")
    ap.add_argument("--workload", choices=["hgemm", "sgemm", "dgemm", "batched", "sgemv", "dgemv", "hgemv", "reduce",
                                           "mlp"], default="hgemm")
    ap.add_argument("--op", choices=["dot", "nrm2", "asum", "iamax"], default="dot", help="reduce: which reduction")
    ap.add_argument("--trans", action="store_true", help="sgemv: A^T x")
    ap.add_argument("--gather", action="store_true",
                    help="column-sharded GEMMs: every rank ends each step with the full C (GEMM with the gather "
                         "fused; the default for HGEMM on N > 1 GPUs)")
    ap.add_argument("--gather-multicast", action="store_true",
                    help="as --gather, HGEMM stores through an NVLink multicast object (torch symmetric memory)")
    ap.add_argument("--gather-nccl", action="store_true",
                    help="as --gather, but GEMM into the panel + NCCL all-gather + re-layout kernel")
    ap.add_argument("--no-gather", action="store_true", help="column-sharded HGEMM on N > 1 GPUs: keep the panels")
    ap.add_argument("--weak", action="store_true",
                    help="HGEMM on N GPUs: every rank its own 8192-column panel of an 8192 x 8192N x 8192 product")
    ap.add_argument("--no-secondary", action="store_true", help="skip the metric's other configurations")
    ap.add_argument("--tf32x3", action="store_true", help="sgemm/mlp: the opt-in 3xTF32 tensor-core kernel")
    ap.add_argument("--fused", action="store_true", help="mlp: bias (+ReLU) fused into the SGEMM epilogue")
    ap.add_argument("--mlp-streams", type=int, choices=[1, 2], default=2,
                    help="mlp: the batch as two halves on two streams (default; same results) or one stream")
    ap.add_argument("--e2e-steps", type=int, default=None, help="0 skips the end-to-end pass")
    ap.add_argument("--e2e-host", choices=["b2b", "torch"], default="b2b",
                    help="page-locked host buffers of the end-to-end pass: b2b_host_alloc or torch pin_memory")
    ap.add_argument("--m", type=int, default=None, help="GEMM size override (profiling small cases)")
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--k", type=int, default=None)
    ap.add_argument("--batch", type=int, default=None,
                    help="batched: batch count override (profiling small cases; default 4096)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-kernels", action="store_true",
                    help="skip timing the reference's GPU kernels (restated in CUDA C) beside the library")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import datetime

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    import b2blas

    h = b2blas.Handle(local)
    # One dedicated stream for torch and the library: the CUDA events that
    # time the steps are recorded on the stream the kernels are launched on.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    h.set_stream(stream.cuda_stream)
    if args.e2e_host == "b2b":
        E2E_HOST["handle"] = h
    w = make_workload(args.workload, h, rank, world, args)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        w.step()
    barrier()
    h.synchronize()

    ms, ms_max, clocks = timed_region(w, stream, args.steps, dist, barrier, local)
    value = w.scale(w.total_units_per_step() * args.steps / (ms_max / 1e3))

    # dominant kernel roofline (per launch, this rank)
    peaks = load_peaks()
    info = h.device_info()
    peak, punit, psrc = roofline_peak(w, peaks, info, clocks.get("sm_mhz") if w.bound in ("fma", "fp64") else None)
    per_launch_ms = ms / args.steps
    if isinstance(w, MlpWorkload):
        # time the GEMMs alone for the kernel figure
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cfgs = [b2blas.GemmConfig(w.batch, w.dims[i + 1], w.dims[i], 1.0, 0.0) for i in range(4)]

        def gemms():
            inp = w.xb
            for i in range(4):
                h.sgemm_tiled(cfgs[i], inp, w.wb[i], w.zb[i])
                inp = w.zb[i]

        # one untimed pass: whole-batch GEMMs may grow the handle's workspace
        # (split-K partial sums) past what the half-batch lanes needed
        gemms()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            gemms()
        e1.record(stream)
        torch.cuda.synchronize()
        per_launch_ms = e0.elapsed_time(e1) / args.steps
    achieved = w.scale(w.units_per_step() / (per_launch_ms / 1e3))
    traffic = load_traffic().get(args.workload) if world == 1 and not (args.m or args.n or args.k) else None
    roof = {"bound": {"hbm": "hbm", "tensor": "tensor", "fp64": "tensor", "tf32x3": "tensor"}.get(w.bound, "fma"),
            "kernel": w.kernel, "achieved": achieved, "peak": peak, "unit": punit, "frac": achieved / peak,
            "peak_source": psrc, "traffic": traffic,
            "algorithmic_units_per_launch": w.units_per_step(),
            "launch_ms": per_launch_ms}
    if isinstance(w, GemmWorkload) and w.gather in ("fused", "fused-multicast"):
        # Fused GEMM + all-gather: the step cannot beat the slower of its
        # math (flops / peak) and its NVLink traffic (the world - 1 panels
        # every GPU receives, at the measured 770 GB/s per direction).
        esz = {"hgemm": 2, "sgemm": 4, "dgemm": 8}[w.kind]
        # Each GPU receives the (world - 1) other panels whatever the sender
        # does (peer stores, or one multicast store replicated by NVSwitch).
        nvl_bytes = (world - 1) * w.m * w.n * esz
        t_math = w.units_per_step() / (peak * 1e12) * 1e3 if punit == "TFLOP/s" else 0.0
        t_link = nvl_bytes / 770e9 * 1e3
        roof["fused_collective"] = {"gather": w.gather, "nvlink_bytes_per_step": nvl_bytes, "link_gbs": 770.0,
                                    "math_ms": t_math, "link_ms": t_link, "target_ms": max(t_math, t_link),
                                    "limiter": "nvlink" if t_link > t_math else "math",
                                    "frac_of_target": max(t_math, t_link) / per_launch_ms}

    # end to end through the host-slice API
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else max(3, min(args.steps, 10))
    e2e = None
    if e2e_steps > 0:
        e2e = run_e2e(w, h, stream, e2e_steps, world, dist, barrier, args.e2e_host)

    refk = None
    if rank == 0 and world == 1 and not args.no_ref_kernels:
        refk = time_ref_kernels(w, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle

        oracle.set_num_threads(os.cpu_count() or 1)
        s = w.cpu_sample(oracle, args.cpu_seconds)
        cpu = {"value": s["value"], "unit": w.unit, "cores": s.get("threads", oracle.num_threads()), "kind": "port",
               "sample": s["sample"], "seconds": round(s["seconds"], 2)}

    launches = w.launches_per_step * args.steps
    config, scaling, wunit, wdtype = w.config(), w.scaling, w.unit, w.dtype
    if hasattr(w, "close"):
        w.close()
    del w
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    secondary = run_secondary(secondary_names(args, world), h, stream, rank, world, dist, barrier, local, args,
                              peaks, info)

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": wunit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": scaling, "vs_baseline": None, "dtype": wdtype,
                "data": DATA, "config": config, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "reference_kernels": refk, "gpu_launches": launches, "clocks": clocks}
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    h.set_stream(None)
    h.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
