"""b2blas.benches -- the reference's bench crate, filled in.

cublas-rs declares a benchmark crate whose every entry point is a todo!
stub (benches/src/lib.rs:1-4): a CUDA-event GpuTimer (timer.rs:6-19), CPU
validation helpers (validator.rs:6-25) and per-routine bench functions that
print a GFLOP/s table against cuBLAS (gemm.rs:6-15, hgemm.rs:3-7,
batched_gemm.rs:3-7, vector_ops.rs:3-19).  This module implements them over
the b2blas C ABI, with the same names and arguments.

    from b2blas import benches
    benches.bench_sgemm(4096, 4096, 4096)

The cuBLAS column comes from torch (torch.mm / bmm / dot, TF32 off), timed
on the same stream with the same events; it is the comparison baseline, not
part of the b2blas path.  `validate_gemm` / `validate_vector` compute their
own CPU reference with numpy in f64 and raise `ValidationError` where the
reference returns Err(String).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import numpy as np

from . import _lib
from . import Algo, GemmConfig, Handle, _check

__all__ = [
    "GpuTimer", "ValidationError", "validate_gemm", "validate_vector", "bench_sgemm", "bench_dgemm", "bench_hgemm",
    "bench_batched_sgemm", "bench_saxpy", "bench_dot", "bench_nrm2",
]


class GpuTimer:
    """GpuTimer (timer.rs:6-19): `start` records a CUDA event on the handle's
    stream, `stop` records the end event, waits for it and returns the
    elapsed milliseconds.  A timer is used once."""

    def __init__(self, raw: ctypes.c_void_p):
        self._t = raw

    @classmethod
    def start(cls, handle: Handle) -> "GpuTimer":
        t = ctypes.c_void_p()
        _check(_lib.load().b2b_gpu_timer_start(handle._h, ctypes.byref(t)))
        return cls(t)

    def stop(self) -> float:
        if not self._t:
            raise RuntimeError("GpuTimer.stop called twice")
        ms = ctypes.c_double()
        t, self._t = self._t, None
        _check(_lib.load().b2b_gpu_timer_stop(t, ctypes.byref(ms)))
        return ms.value


class ValidationError(Exception):
    """Err(String) of validate_gemm / validate_vector."""


def validate_gemm(m: int, n: int, k: int, alpha: float, a, b, beta: float, expected, actual,
                  tolerance: float) -> None:
    """validate_gemm (validator.rs:6-20): recompute alpha*A*B + beta*C on the
    CPU (f64) and check max |actual - reference| <= tolerance.  `expected`
    is C as it was before the call (the matrix beta scales); `actual` is C
    after it.  Row-major, A m x k, B k x n, C m x n."""
    a = np.asarray(a, dtype=np.float64).reshape(-1)
    b = np.asarray(b, dtype=np.float64).reshape(-1)
    c0 = np.asarray(expected, dtype=np.float64).reshape(-1)
    got = np.asarray(actual, dtype=np.float64).reshape(-1)
    for name, arr, want in (("A", a, m * k), ("B", b, k * n), ("expected", c0, m * n), ("actual", got, m * n)):
        if arr.size != want:
            raise ValidationError(f"{name} has {arr.size} elements, expected {want}")
    ref = alpha * (a.reshape(m, k) @ b.reshape(k, n)).reshape(-1)
    if beta != 0.0:
        ref = ref + beta * c0
    _check_close(ref, got, tolerance, lambda i: f"C[{i // n}][{i % n}]" if n else f"C[{i}]")


def validate_vector(expected, actual, tolerance: float) -> None:
    """validate_vector (validator.rs:22-25): element-wise max |actual -
    expected| <= tolerance, equal lengths."""
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    if e.size != a.size:
        raise ValidationError(f"length mismatch: expected {e.size}, actual {a.size}")
    _check_close(e, a, tolerance, lambda i: f"[{i}]")


def _check_close(ref: np.ndarray, got: np.ndarray, tol: float, where: Callable[[int], str]) -> None:
    if ref.size == 0:
        return
    bad = np.isnan(got) & ~np.isnan(ref)
    if bad.any():
        i = int(np.argmax(bad))
        raise ValidationError(f"NaN at {where(i)} (reference {ref[i]})")
    err = np.abs(got - ref)
    err[np.isnan(err)] = 0.0  # NaN in both
    i = int(np.argmax(err))
    if err[i] > tol:
        raise ValidationError(f"max abs error {err[i]:.6g} at {where(i)} exceeds tolerance {tol:g} "
                              f"(got {got[i]:.9g}, reference {ref[i]:.9g})")


# ---------------------------------------------------------------- benches

def _torch_stream(handle: Handle):
    """A torch stream shared with the handle, so one pair of events times
    both sides."""
    import torch

    s = torch.cuda.Stream(device=handle.device)
    handle.set_stream(s.cuda_stream)
    return s


def _time(handle: Handle, fn: Callable[[], None], reps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    t = GpuTimer.start(handle)
    for _ in range(reps):
        fn()
    return t.stop() / reps


def _print_table(title: str, rows: list, unit: str) -> None:
    print(title)
    print(f"  {'variant':<22}{'ms':>10}{unit:>12}{'vs cuBLAS':>11}")
    base = next((r["rate"] for r in rows if r["variant"].startswith("cuBLAS")), None)
    for r in rows:
        rel = f"{r['rate'] / base:10.2f}x" if base else ""
        print(f"  {r['variant']:<22}{r['ms']:>10.4f}{r['rate']:>12.1f}{rel:>11}")


def _gemm_bench(kind: str, m: int, n: int, k: int, reps: int, warmup: int, handle: Optional[Handle],
                print_table: bool) -> list:
    import torch

    h = handle or Handle(torch.cuda.current_device())
    s = _torch_stream(h)
    dev = torch.device("cuda", h.device)
    dt = {"s": np.float32, "d": np.float64, "h": np.float16}[kind]
    tdt = {"s": torch.float32, "d": torch.float64, "h": torch.float16}[kind]
    rng = np.random.default_rng(0)
    A = (rng.standard_normal(m * k) * (0.1 if kind == "h" else 1.0)).astype(dt)
    B = (rng.standard_normal(k * n) * (0.1 if kind == "h" else 1.0)).astype(dt)
    a, b = h.upload(A), h.upload(B)
    c = h.zeroed(m * n, np.uint16 if kind == "h" else dt)
    cfg = GemmConfig(m, n, k, 1.0, 0.0)
    flops = 2.0 * m * n * k
    rows = []
    with torch.cuda.stream(s):
        if kind == "h":
            variants = [("hgemm_tensor_core", lambda: h.hgemm(cfg, a, b, c))]
        else:
            fn = h.sgemm if kind == "s" else h.dgemm
            names = [("naive", Algo.Naive), ("tiled", Algo.Tiled), ("vectorized", Algo.Vectorized),
                     ("double_buf", Algo.DoubleBuf)]
            variants = [(f"{kind}gemm_{nm}", (lambda al=al: fn(cfg, a, b, c, al))) for nm, al in names]
            if kind == "s":
                variants.append(("sgemm_3xtf32", lambda: h.sgemm(cfg, a, b, c, Algo.Tf32x3)))
        for name, f in variants:
            ms = _time(h, f, reps, warmup)
            rows.append({"variant": name, "ms": ms, "rate": flops / ms / 1e6})
        ta = torch.from_numpy(A).to(dev).reshape(m, k)
        tb = torch.from_numpy(B).to(dev).reshape(k, n)
        tc = torch.empty(m, n, dtype=tdt, device=dev)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            ms = _time(h, lambda: torch.mm(ta, tb, out=tc), reps, warmup)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        rows.append({"variant": f"cuBLAS {kind}gemm", "ms": ms, "rate": flops / ms / 1e6})
    h.synchronize()
    h.set_stream(None)
    if print_table:
        _print_table(f"{kind.upper()}GEMM {m}x{n}x{k} (GFLOP/s)", rows, "GFLOP/s")
    return rows


def bench_sgemm(m: int, n: int, k: int, reps: int = 10, warmup: int = 3, handle: Optional[Handle] = None,
                print_table: bool = True) -> list:
    """bench_sgemm (gemm.rs:3-10): every SGEMM variant against cuBLAS
    SGEMM (TF32 off); returns the rows it prints."""
    return _gemm_bench("s", m, n, k, reps, warmup, handle, print_table)


def bench_dgemm(m: int, n: int, k: int, reps: int = 10, warmup: int = 3, handle: Optional[Handle] = None,
                print_table: bool = True) -> list:
    """bench_dgemm (gemm.rs:12-15)."""
    return _gemm_bench("d", m, n, k, reps, warmup, handle, print_table)


def bench_hgemm(m: int, n: int, k: int, reps: int = 10, warmup: int = 3, handle: Optional[Handle] = None,
                print_table: bool = True) -> list:
    """bench_hgemm (hgemm.rs:3-7): the tcgen05 HGEMM against cuBLAS HGEMM."""
    return _gemm_bench("h", m, n, k, reps, warmup, handle, print_table)


def bench_batched_sgemm(m: int, n: int, k: int, batch_count: int, reps: int = 10, warmup: int = 3,
                        handle: Optional[Handle] = None, print_table: bool = True) -> list:
    """bench_batched_sgemm (batched_gemm.rs:3-7): strided-batched SGEMM
    against torch.bmm (cuBLAS strided-batched SGEMM)."""
    import torch

    h = handle or Handle(torch.cuda.current_device())
    s = _torch_stream(h)
    dev = torch.device("cuda", h.device)
    rng = np.random.default_rng(0)
    A = rng.standard_normal(batch_count * m * k).astype(np.float32)
    B = rng.standard_normal(batch_count * k * n).astype(np.float32)
    a, b, c = h.upload(A), h.upload(B), h.zeroed(batch_count * m * n)
    cfg = GemmConfig(m, n, k, 1.0, 0.0)
    flops = 2.0 * m * n * k * batch_count
    rows = []
    with torch.cuda.stream(s):
        ms = _time(h, lambda: h.strided_batched_sgemm(cfg, batch_count, a, m * k, b, k * n, c, m * n), reps,
                   warmup)
        rows.append({"variant": "strided_batched_sgemm", "ms": ms, "rate": flops / ms / 1e6})
        ta = torch.from_numpy(A).to(dev).reshape(batch_count, m, k)
        tb = torch.from_numpy(B).to(dev).reshape(batch_count, k, n)
        tc = torch.empty(batch_count, m, n, device=dev)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            ms = _time(h, lambda: torch.bmm(ta, tb, out=tc), reps, warmup)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        rows.append({"variant": "cuBLAS bmm", "ms": ms, "rate": flops / ms / 1e6})
    h.synchronize()
    h.set_stream(None)
    if print_table:
        _print_table(f"batched SGEMM {batch_count} x {m}x{n}x{k} (GFLOP/s)", rows, "GFLOP/s")
    return rows


def _vector_bench(op: str, n: int, reps: int, warmup: int, handle: Optional[Handle], print_table: bool) -> list:
    import torch

    h = handle or Handle(torch.cuda.current_device())
    s = _torch_stream(h)
    dev = torch.device("cuda", h.device)
    rng = np.random.default_rng(0)
    X = rng.standard_normal(n).astype(np.float32)
    Y = rng.standard_normal(n).astype(np.float32)
    x, y = h.upload(X), h.upload(Y)
    res = h.zeroed(1)
    nbytes = {"saxpy": 12.0 * n, "dot": 8.0 * n, "nrm2": 4.0 * n}[op]
    rows = []
    with torch.cuda.stream(s):
        if op == "saxpy":
            ours = lambda: h.saxpy(n, 2.0, x, y)  # noqa: E731
        elif op == "dot":
            ours = lambda: h.sreduce_async(Handle.ReduceOp.Dot, n, x, y, res)  # noqa: E731
        else:
            ours = lambda: h.sreduce_async(Handle.ReduceOp.Nrm2, n, x, None, res)  # noqa: E731
        ms = _time(h, ours, reps, warmup)
        rows.append({"variant": f"b2blas {op}", "ms": ms, "rate": nbytes / ms / 1e6})
        tx, ty = torch.from_numpy(X).to(dev), torch.from_numpy(Y).to(dev)
        if op == "saxpy":
            theirs = lambda: ty.add_(tx, alpha=2.0)  # noqa: E731
        elif op == "dot":
            theirs = lambda: torch.dot(tx, ty)  # noqa: E731
        else:
            theirs = lambda: torch.linalg.vector_norm(tx)  # noqa: E731
        ms = _time(h, theirs, reps, warmup)
        rows.append({"variant": f"cuBLAS/torch {op}", "ms": ms, "rate": nbytes / ms / 1e6})
    h.synchronize()
    h.set_stream(None)
    if print_table:
        _print_table(f"{op} n={n} (GB/s)", rows, "GB/s")
    return rows


def bench_saxpy(n: int, reps: int = 20, warmup: int = 3, handle: Optional[Handle] = None,
                print_table: bool = True) -> list:
    """bench_saxpy (vector_ops.rs:3-7), in GB/s (12 bytes per element)."""
    return _vector_bench("saxpy", n, reps, warmup, handle, print_table)


def bench_dot(n: int, reps: int = 20, warmup: int = 3, handle: Optional[Handle] = None,
              print_table: bool = True) -> list:
    """bench_dot (vector_ops.rs:9-13), in GB/s (8 bytes per element)."""
    return _vector_bench("dot", n, reps, warmup, handle, print_table)


def bench_nrm2(n: int, reps: int = 20, warmup: int = 3, handle: Optional[Handle] = None,
               print_table: bool = True) -> list:
    """bench_nrm2 (vector_ops.rs:15-19), in GB/s (4 bytes per element)."""
    return _vector_bench("nrm2", n, reps, warmup, handle, print_table)
