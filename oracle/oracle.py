"""ctypes/numpy front end of the CPU oracle (liboracle.so, built from oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker.  The product library never
calls into this module.

Every function here forwards to oracle.c; the reference file:line each one
restates is given there.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_LIB_PATH_V3 = os.path.join(_HERE, "liboracle_v3.so")
_lib = None


def _cpu_has_avx2_fma() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return "avx2" in flags and "fma" in flags
    except OSError:
        pass
    return False

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_d = ctypes.c_double
_f = ctypes.c_float


def build() -> str:
    """Compile liboracle.so (gcc + OpenMP) if it is missing or stale."""
    src = os.path.join(_HERE, "oracle.c")
    stale = [p for p in (_LIB_PATH, _LIB_PATH_V3)
             if not os.path.exists(p) or os.path.getmtime(p) < os.path.getmtime(src)]
    if stale:
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    path = _LIB_PATH_V3 if (_cpu_has_avx2_fma() and os.path.exists(_LIB_PATH_V3)) else _LIB_PATH
    L = ctypes.CDLL(path)
    sig = {
        "oracle_pcg32_first": (ctypes.c_uint32, [_u64, _u64, _u32p, _sz]),
        "oracle_fill_uniform_f32": (None, [_f32p, _sz, _u64, _u64, _d, _d]),
        "oracle_fill_uniform_f64": (None, [_f64p, _sz, _u64, _u64, _d, _d]),
        "oracle_fill_normal_f32": (None, [_f32p, _sz, _u64, _u64, _d, _d]),
        "oracle_fill_normal_f16": (None, [_u16p, _sz, _u64, _u64, _d, _d]),
        "oracle_fill_uniform_f16": (None, [_u16p, _sz, _u64, _u64, _d, _d]),
        "oracle_ref_f16_to_f32": (_f, [ctypes.c_uint16]),
        "oracle_ref_f32_to_f16": (ctypes.c_uint16, [_f]),
        "oracle_f16_to_f64": (_d, [ctypes.c_uint16]),
        "oracle_f64_to_f16_rne": (ctypes.c_uint16, [_d]),
        "oracle_sgemm_rows_f64": (None, [_sz, _sz, _sz, _sz, _sz, _d, _f32p, _f32p, _d, ctypes.c_void_p, _f64p]),
        "oracle_dgemm_rows_f64": (None, [_sz, _sz, _sz, _sz, _sz, _d, _f64p, _f64p, _d, ctypes.c_void_p, _f64p]),
        "oracle_hgemm_rows_f64": (None, [_sz, _sz, _sz, _sz, _sz, _d, _u16p, _u16p, _d, ctypes.c_void_p, _f64p]),
        "oracle_sgemm_strided_batched_f64": (
            None, [_sz, _sz, _sz, _d, _f32p, _sz, _f32p, _sz, _d, ctypes.c_void_p, _sz, _sz, _f64p]),
        "oracle_sgemv_f64": (None, [ctypes.c_int, _sz, _sz, _d, _f32p, _f32p, _d, _f32p, _f64p]),
        "oracle_dgemv_f64": (None, [ctypes.c_int, _sz, _sz, _d, _f64p, _f64p, _d, _f64p, _f64p]),
        "oracle_hgemv_f64": (None, [ctypes.c_int, _sz, _sz, _d, _u16p, _u16p, _d, _u16p, _f64p]),
        "oracle_hgemv_ref": (None, [ctypes.c_int, _sz, _sz, _f, _u16p, _u16p, _f, _u16p]),
        "oracle_saxpy_f64": (None, [_sz, _d, _f32p, _f32p, _f64p]),
        "oracle_sdot_f64": (_d, [_sz, _f32p, _f32p]),
        "oracle_snrm2_f64": (_d, [_sz, _f32p]),
        "oracle_sasum_f64": (_d, [_sz, _f32p]),
        "oracle_isamax": (_sz, [_sz, _f32p]),
        "oracle_sreduce_ref": (_f, [ctypes.c_int, _sz, _f32p, ctypes.c_void_p]),
        "oracle_isamax_ref": (_sz, [_sz, _f32p]),
        "oracle_sgemm_ref_f32": (None, [_sz, _sz, _sz, _f, _f32p, _f32p, _f, _f32p]),
        "oracle_hgemm_ref": (None, [_sz, _sz, _sz, _f, _u16p, _u16p, _f, _u16p]),
        "oracle_rel_fro_err_f32": (_d, [_f32p, _f64p, _sz]),
        "oracle_rel_fro_err_f64": (_d, [_f64p, _f64p, _sz]),
        "oracle_rel_fro_err_f16": (_d, [_u16p, _f64p, _sz]),
        "oracle_num_threads": (ctypes.c_int, []),
        "oracle_set_num_threads": (None, [ctypes.c_int]),
        "oracle_cpu_sgemm_ikj": (None, [_sz, _sz, _sz, _f, _f32p, _f32p, _f, _f32p, _f32p]),
        "oracle_cpu_dgemm_ikj": (None, [_sz, _sz, _sz, _d, _f64p, _f64p, _d, _f64p, _f64p]),
        "oracle_cpu_hgemm_ikj": (None, [_sz, _sz, _sz, _f, _u16p, _u16p, _f, _u16p, _f32p, _f32p]),
        "oracle_cpu_sgemv_n": (None, [_sz, _sz, _f, _f32p, _f32p, _f, _f32p]),
        "oracle_cpu_dgemv_n": (None, [_sz, _sz, _d, _f64p, _f64p, _d, _f64p]),
        "oracle_cpu_hgemv_n": (None, [_sz, _sz, _f, _u16p, _u16p, _f, _u16p, _f32p]),
        "oracle_cpu_sdot": (_f, [_sz, _f32p, _f32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def _cptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- inputs

def pcg32(seed: int, stream: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().oracle_pcg32_first(seed, stream, out, n)
    return out


def uniform_f32(n, seed=42, stream=1, lo=-1.0, hi=1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oracle_fill_uniform_f32(out, n, seed, stream, lo, hi)
    return out


def uniform_f64(n, seed=42, stream=1, lo=-1.0, hi=1.0) -> np.ndarray:
    out = np.empty(n, np.float64)
    lib().oracle_fill_uniform_f64(out, n, seed, stream, lo, hi)
    return out


def normal_f32(n, seed=42, stream=1, mean=0.0, std=1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oracle_fill_normal_f32(out, n, seed, stream, mean, std)
    return out


def normal_f16(n, seed=42, stream=1, mean=0.0, std=1.0) -> np.ndarray:
    """f16 bit patterns (uint16) of normal(mean, std) rounded to nearest even."""
    out = np.empty(n, np.uint16)
    lib().oracle_fill_normal_f16(out, n, seed, stream, mean, std)
    return out


def uniform_f16(n, seed=42, stream=1, lo=-1.0, hi=1.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().oracle_fill_uniform_f16(out, n, seed, stream, lo, hi)
    return out


# ------------------------------------------------------------ conversions

def ref_f16_to_f32(h: int) -> float:
    return lib().oracle_ref_f16_to_f32(h)


def ref_f32_to_f16(f: float) -> int:
    return lib().oracle_ref_f32_to_f16(f)


def f16_to_f64(h: int) -> float:
    return lib().oracle_f16_to_f64(h)


def f64_to_f16_rne(x: float) -> int:
    return lib().oracle_f64_to_f16_rne(x)


# ------------------------------------------------------- FP64 evaluations

def sgemm_f64(m, n, k, alpha, A, B, beta=0.0, C=None, row0=0, nrows=None) -> np.ndarray:
    nrows = m - row0 if nrows is None else nrows
    A, B = _c(A, np.float32).ravel(), _c(B, np.float32).ravel()
    C = None if C is None else _c(C, np.float32).ravel()
    out = np.empty(nrows * n, np.float64)
    lib().oracle_sgemm_rows_f64(m, n, k, row0, nrows, alpha, A, B, beta, _cptr(C), out)
    return out


def dgemm_f64(m, n, k, alpha, A, B, beta=0.0, C=None, row0=0, nrows=None) -> np.ndarray:
    nrows = m - row0 if nrows is None else nrows
    A, B = _c(A, np.float64).ravel(), _c(B, np.float64).ravel()
    C = None if C is None else _c(C, np.float64).ravel()
    out = np.empty(nrows * n, np.float64)
    lib().oracle_dgemm_rows_f64(m, n, k, row0, nrows, alpha, A, B, beta, _cptr(C), out)
    return out


def hgemm_f64(m, n, k, alpha, A, B, beta=0.0, C=None, row0=0, nrows=None) -> np.ndarray:
    """A, B, C are f16 bit patterns (uint16)."""
    nrows = m - row0 if nrows is None else nrows
    A, B = _c(A, np.uint16).ravel(), _c(B, np.uint16).ravel()
    C = None if C is None else _c(C, np.uint16).ravel()
    out = np.empty(nrows * n, np.float64)
    lib().oracle_hgemm_rows_f64(m, n, k, row0, nrows, alpha, A, B, beta, _cptr(C), out)
    return out


def sgemm_strided_batched_f64(m, n, k, alpha, A, sa, B, sb, beta, C, sc, batch) -> np.ndarray:
    A, B = _c(A, np.float32).ravel(), _c(B, np.float32).ravel()
    C = None if C is None else _c(C, np.float32).ravel()
    out = np.empty(batch * m * n, np.float64)
    lib().oracle_sgemm_strided_batched_f64(m, n, k, alpha, A, sa, B, sb, beta, _cptr(C), sc, batch, out)
    return out


def sgemv_f64(trans: int, m, n, alpha, A, x, beta, y) -> np.ndarray:
    A, x, y = _c(A, np.float32).ravel(), _c(x, np.float32).ravel(), _c(y, np.float32).ravel()
    out = np.empty(n if trans else m, np.float64)
    lib().oracle_sgemv_f64(int(trans), m, n, alpha, A, x, beta, y, out)
    return out


def dgemv_f64(trans: int, m, n, alpha, A, x, beta, y) -> np.ndarray:
    """DGEMV with Dot2-compensated dot products (oracle error ~ eps_f64)."""
    A, x, y = _c(A, np.float64).ravel(), _c(x, np.float64).ravel(), _c(y, np.float64).ravel()
    out = np.empty(n if trans else m, np.float64)
    lib().oracle_dgemv_f64(int(trans), m, n, alpha, A, x, beta, y, out)
    return out


def hgemv_f64(trans: int, m, n, alpha, A, x, beta, y) -> np.ndarray:
    """HGEMV of f16 bit patterns, evaluated in f64 from the exact inputs."""
    A, x, y = _c(A, np.uint16).ravel(), _c(x, np.uint16).ravel(), _c(y, np.uint16).ravel()
    out = np.empty(n if trans else m, np.float64)
    lib().oracle_hgemv_f64(int(trans), m, n, alpha, A, x, beta, y, out)
    return out


def saxpy_f64(n, alpha, x, y) -> np.ndarray:
    x, y = _c(x, np.float32).ravel(), _c(y, np.float32).ravel()
    out = np.empty(n, np.float64)
    lib().oracle_saxpy_f64(n, alpha, x, y, out)
    return out


def sdot_f64(n, x, y) -> float:
    return lib().oracle_sdot_f64(n, _c(x, np.float32).ravel(), _c(y, np.float32).ravel())


def snrm2_f64(n, x) -> float:
    return lib().oracle_snrm2_f64(n, _c(x, np.float32).ravel())


def sasum_f64(n, x) -> float:
    return lib().oracle_sasum_f64(n, _c(x, np.float32).ravel())


def isamax(n, x) -> int:
    """Smallest index of the largest |x[i]| (NaN skipped; 0 if none)."""
    return lib().oracle_isamax(n, _c(x, np.float32).ravel())


# ------------------------------------------- reference arithmetic (f32/f16)

def sgemm_ref_f32(m, n, k, alpha, A, B, beta, C) -> np.ndarray:
    C = _c(C, np.float32).ravel().copy()
    lib().oracle_sgemm_ref_f32(m, n, k, alpha, _c(A, np.float32).ravel(), _c(B, np.float32).ravel(), beta, C)
    return C


def hgemm_ref(m, n, k, alpha, A, B, beta, C) -> np.ndarray:
    C = _c(C, np.uint16).ravel().copy()
    lib().oracle_hgemm_ref(m, n, k, alpha, _c(A, np.uint16).ravel(), _c(B, np.uint16).ravel(), beta, C)
    return C


def hgemv_ref(trans: int, m, n, alpha, A, x, beta, y) -> np.ndarray:
    """The reference's own HGEMV arithmetic (flushing decode, f32 sums,
    truncating encode); returns the new y as f16 bit patterns."""
    y = _c(y, np.uint16).ravel().copy()
    lib().oracle_hgemv_ref(int(trans), m, n, alpha, _c(A, np.uint16).ravel(), _c(x, np.uint16).ravel(), beta, y)
    return y


def sreduce_ref(op: str, n, x, y=None) -> float:
    """The reference's 32-lane f32 reduction (op 'dot', 'nrm2' or 'asum')."""
    code = {"dot": 0, "nrm2": 1, "asum": 2}[op]
    x = _c(x, np.float32).ravel()
    yp = None
    if code == 0:
        y = _c(y, np.float32).ravel()
        yp = y.ctypes.data
    return lib().oracle_sreduce_ref(code, n, x, yp)


def isamax_ref(n, x) -> int:
    """The reference's ISAMAX, tie order included."""
    return lib().oracle_isamax_ref(n, _c(x, np.float32).ravel())


# ------------------------------------------------------------------ norms

def rel_err(got, ref: np.ndarray) -> float:
    """Normwise relative error ||got - ref||_F / ||ref||_F."""
    ref = _c(ref, np.float64).ravel()
    if got.dtype == np.float32:
        return lib().oracle_rel_fro_err_f32(_c(got, np.float32).ravel(), ref, ref.size)
    if got.dtype == np.float64:
        return lib().oracle_rel_fro_err_f64(_c(got, np.float64).ravel(), ref, ref.size)
    if got.dtype == np.uint16:
        return lib().oracle_rel_fro_err_f16(_c(got, np.uint16).ravel(), ref, ref.size)
    raise TypeError(got.dtype)


EPS = {"f32": float(np.finfo(np.float32).eps), "f64": float(np.finfo(np.float64).eps)}


def tol_normwise(k: int, dtype: str) -> float:
    """The parity bound 4*K*eps(dtype) for FP32/FP64 GEMM/GEMV."""
    return 4.0 * k * EPS[dtype]


HGEMM_TOL = 2e-2  # relative, FP16 in / FP32 accumulate


# ---------------------------------------------------------- CPU baselines

def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(t: int) -> None:
    lib().oracle_set_num_threads(t)


def cpu_sgemm_rows(rows, n, k, alpha, A, B, beta, C, scratch) -> None:
    lib().oracle_cpu_sgemm_ikj(rows, n, k, alpha, A, B, beta, C, scratch)


def cpu_dgemm_rows(rows, n, k, alpha, A, B, beta, C, scratch) -> None:
    lib().oracle_cpu_dgemm_ikj(rows, n, k, alpha, A, B, beta, C, scratch)


def cpu_hgemm_rows(rows, n, k, alpha, A, B, beta, C, bf_scratch, row_scratch) -> None:
    lib().oracle_cpu_hgemm_ikj(rows, n, k, alpha, A, B, beta, C, bf_scratch, row_scratch)


def cpu_sgemv_rows(rows, n, alpha, A, x, beta, y) -> None:
    lib().oracle_cpu_sgemv_n(rows, n, alpha, A, x, beta, y)


def cpu_dgemv_rows(rows, n, alpha, A, x, beta, y) -> None:
    lib().oracle_cpu_dgemv_n(rows, n, alpha, A, x, beta, y)


def cpu_hgemv_rows(rows, n, alpha, A, x, beta, y, xf) -> None:
    lib().oracle_cpu_hgemv_n(rows, n, alpha, A, x, beta, y, xf)


def cpu_sdot(n, x, y) -> float:
    return lib().oracle_cpu_sdot(n, x, y)
