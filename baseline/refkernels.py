"""ctypes loader for librefkernels.so: the reference's GPU kernels (naive /
tiled / vectorized / double_buf GEMMs, hgemm_half, strided-batched SGEMM,
GEMVs, saxpy, the 32-thread L1 reductions) restated in CUDA C.

A reported baseline for bench.py, timed on the same resident buffers as the
library; the library never calls it.  Every function takes raw device
pointers (ints) and a CUDA stream handle, launches asynchronously, and raises
RuntimeError on a launch error.  Variant numbers follow the reference's
Handle methods: 0 naive, 1 tiled, 2 vectorized, 3 double_buf
(crates/cublas-rs/src/lib.rs:439-612)."""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "librefkernels.so")
_lib = None

GEMM_VARIANTS = {0: "naive", 1: "tiled", 2: "vectorized", 3: "double_buf"}
SYMBOLS = ("refk_sgemm", "refk_dgemm", "refk_hgemm_half", "refk_sgemm_strided_batched", "refk_sgemv",
           "refk_dgemv", "refk_hgemv", "refk_sreduce", "refk_saxpy")


def build() -> str:
    import subprocess

    subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"{_LIB_PATH} is not built (make -C baseline)")
        L = ctypes.CDLL(_LIB_PATH)
        i, f, d, p, i64 = ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_void_p, ctypes.c_int64
        sig = {
            "refk_sgemm": [i, i, i, i, f, p, p, f, p, p],
            "refk_dgemm": [i, i, i, i, d, p, p, d, p, p],
            "refk_hgemm_half": [i, i, i, f, p, p, f, p, p],
            "refk_sgemm_strided_batched": [i, i, i, f, p, i64, p, i64, f, p, i64, i, p],
            "refk_sgemv": [i, i, i, i, f, p, p, f, p, p],
            "refk_dgemv": [i, i, i, d, p, p, d, p, p],
            "refk_hgemv": [i, i, i, f, p, p, f, p, p],
            "refk_sreduce": [i, i, p, p, p, p],
            "refk_saxpy": [i, f, p, p, p],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, i
        _lib = L
    return _lib


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def sgemm(variant, m, n, k, alpha, a, b, beta, c, stream=0):
    _check(lib().refk_sgemm(variant, m, n, k, alpha, a, b, beta, c, stream), "refk_sgemm")


def dgemm(variant, m, n, k, alpha, a, b, beta, c, stream=0):
    _check(lib().refk_dgemm(variant, m, n, k, alpha, a, b, beta, c, stream), "refk_dgemm")


def hgemm_half(m, n, k, alpha, a, b, beta, c, stream=0):
    _check(lib().refk_hgemm_half(m, n, k, alpha, a, b, beta, c, stream), "refk_hgemm_half")


def sgemm_strided_batched(m, n, k, alpha, a, sa, b, sb, beta, c, sc, batch, stream=0):
    _check(lib().refk_sgemm_strided_batched(m, n, k, alpha, a, sa, b, sb, beta, c, sc, batch, stream),
           "refk_sgemm_strided_batched")


def sgemv(variant, trans, m, n, alpha, a, x, beta, y, stream=0):
    _check(lib().refk_sgemv(variant, trans, m, n, alpha, a, x, beta, y, stream), "refk_sgemv")


def dgemv(trans, m, n, alpha, a, x, beta, y, stream=0):
    _check(lib().refk_dgemv(trans, m, n, alpha, a, x, beta, y, stream), "refk_dgemv")


def hgemv(trans, m, n, alpha, a, x, beta, y, stream=0):
    _check(lib().refk_hgemv(trans, m, n, alpha, a, x, beta, y, stream), "refk_hgemv")


REDUCE_OPS = {"dot": 0, "nrm2": 1, "asum": 2, "iamax": 3}


def sreduce(op, n, x, y, out, stream=0):
    """op: "dot" | "nrm2" (writes the sum of squares) | "asum" | "iamax" (uint32, 0-based)."""
    _check(lib().refk_sreduce(REDUCE_OPS[op], n, x, y or 0, out, stream), "refk_sreduce")


def saxpy(n, alpha, x, y, stream=0):
    _check(lib().refk_saxpy(n, alpha, x, y, stream), "refk_saxpy")
