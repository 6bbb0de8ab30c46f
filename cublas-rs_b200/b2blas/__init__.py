"""b2blas -- Python mirror of cublas-rs's `Handle` API over the B200 C ABI.

The method names, argument order, row-major layout and alpha/beta semantics
are those of `cublas_rs::Handle` (crates/cublas-rs/src/lib.rs:42-710); the
device-buffer flavour takes `DeviceBuffer`s and is asynchronous on the
handle's stream, the `_simple` flavour takes host numpy arrays, copies in and
out and blocks.  Errors raise `CublasError`, whose `kind` names the
`cublas_core::CublasError` variant (crates/cublas-core/src/error.rs:7-24).
Where the reference panics on a host-slice length mismatch
(crates/cublas-l3/src/sgemm.rs:469-471), this raises
`CublasError(kind="DimensionMismatch")`.

Every call goes through libb2blas.so (hand-written sm_100a kernels); there is
no CPU fallback.
"""
from __future__ import annotations

import ctypes
import enum
import weakref
from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np

from . import _lib

__all__ = [
    "Algo", "CublasError", "DeviceBuffer", "GemmConfig", "Handle", "Transpose", "load_library", "version",
]

load_library = _lib.load

# b2b_status -> CublasError variant
_KIND = {
    1: "Driver",
    2: "DimensionMismatch",
    3: "InvalidArgument",
    4: "Driver",  # device wait timeout, surfaced as a driver-level failure
    5: "InvalidArgument",
    6: "Driver",
}


class CublasError(RuntimeError):
    """Error from a b2blas call; `kind` is the cublas_core::CublasError variant
    and `status` the b2b_status code."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = _KIND.get(status, "Driver")
        super().__init__(f"{self.kind}: {message}")


class Transpose(enum.IntEnum):
    """cublas_core::Transpose (crates/cublas-core/src/config.rs:20-23)."""

    NoTrans = 0
    Trans = 1


class Algo(enum.IntEnum):
    """Kernel variant the call was made as (see b2b_algo in b2blas.h)."""

    Default = 0
    Naive = 1
    Tiled = 2
    Vectorized = 3
    DoubleBuf = 4
    Tf32x3 = 5


@dataclass
class GemmConfig:
    """cublas_core::GemmConfig<T> (crates/cublas-core/src/config.rs:3-9):
    C = alpha * A * B + beta * C with A m x k, B k x n, C m x n."""

    m: int
    n: int
    k: int
    alpha: float = 1.0
    beta: float = 0.0


def version() -> int:
    return _lib.load().b2b_version()


def _check(rc: int) -> None:
    if rc != 0:
        lib = _lib.load()
        raise CublasError(rc, lib.b2b_last_error().decode(errors="replace"))


_DT = {
    np.dtype(np.float32): np.float32,
    np.dtype(np.float64): np.float64,
    np.dtype(np.float16): np.uint16,
    np.dtype(np.uint16): np.uint16,
}


def _host(a: np.ndarray, dtype) -> np.ndarray:
    if not isinstance(a, np.ndarray):
        raise TypeError("host slices must be numpy arrays")
    if a.dtype == np.float16 and dtype == np.uint16:
        a = a.view(np.uint16)
    if a.dtype != np.dtype(dtype):
        raise TypeError(f"expected {np.dtype(dtype)}, got {a.dtype}")
    if not a.flags.c_contiguous:
        raise ValueError("host slices must be C-contiguous")
    return a


def _hp(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


class DeviceBuffer:
    """Typed device allocation, the stand-in for cuda_core::DeviceBuffer<T>
    (re-exported as cublas_rs::DeviceBuf, crates/cublas-rs/src/lib.rs:34).

    Owns its memory unless created with `from_ptr` (a view of someone
    else's allocation, e.g. a torch tensor's storage)."""

    def __init__(self, handle: "Handle", ptr: int, length: int, dtype, owner: Any = None, owned: bool = True):
        self.handle = handle
        self.ptr = int(ptr)
        self._len = int(length)
        self.dtype = np.dtype(dtype)
        self._owner = owner
        self._owned = owned

    def __len__(self) -> int:
        return self._len

    def len(self) -> int:
        return self._len

    @property
    def nbytes(self) -> int:
        return self._len * self.dtype.itemsize

    @classmethod
    def zeroed(cls, handle: "Handle", length: int, dtype=np.float32) -> "DeviceBuffer":
        """DeviceBuffer::zeroed(stream, n)."""
        buf = handle.alloc(length, dtype)
        _check(_lib.load().b2b_memset(handle._h, ctypes.c_void_p(buf.ptr), 0, buf.nbytes))
        return buf

    @classmethod
    def from_host(cls, handle: "Handle", host: np.ndarray) -> "DeviceBuffer":
        """DeviceBuffer::from_host(stream, &[T])."""
        return handle.upload(host)

    @classmethod
    def from_ptr(cls, handle: "Handle", ptr: int, length: int, dtype, owner: Any = None) -> "DeviceBuffer":
        """Non-owning view of existing device memory (kept alive by `owner`)."""
        return cls(handle, ptr, length, dtype, owner=owner, owned=False)

    def to_host_vec(self) -> np.ndarray:
        return self.handle.download(self)

    def free(self) -> None:
        if self._owned and self.ptr:
            _lib.load().b2b_free(self.handle._h, ctypes.c_void_p(self.ptr))
        self.ptr = 0
        self._owned = False

    def __del__(self):
        try:
            if self._owned and self.ptr and self.handle._h:
                self.free()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.free()


class Handle:
    """Mirror of cublas_rs::Handle (crates/cublas-rs/src/lib.rs:42-710)."""

    def __init__(self, device: int = 0):
        lib = _lib.load()
        h = ctypes.c_void_p()
        _check(lib.b2b_create(int(device), ctypes.byref(h)))
        self._h = h
        self._lib = lib
        self.device = int(device)

    # ---- lifecycle (lib.rs:53-97)
    @classmethod
    def new(cls) -> "Handle":
        return cls(0)

    @classmethod
    def with_device(cls, device_idx: int) -> "Handle":
        return cls(device_idx)

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self._lib.b2b_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _check(self._lib.b2b_get_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def set_stream(self, stream: int | None) -> None:
        """Issue subsequent work on a caller-owned cudaStream_t.  None selects
        the handle's own stream; 0 (what torch reports for its default
        stream) selects the legacy default stream."""
        if stream is None:
            ptr = 0
        elif int(stream) == 0:
            ptr = 1  # cudaStreamLegacy
        else:
            ptr = int(stream)
        _check(self._lib.b2b_set_stream(self._h, ctypes.c_void_p(ptr)))

    def synchronize(self) -> None:
        _check(self._lib.b2b_synchronize(self._h))

    def device_info(self) -> dict:
        d, s, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _check(self._lib.b2b_device_info(self._h, ctypes.byref(d), ctypes.byref(s), ctypes.byref(c)))
        return {"device": d.value, "sm_count": s.value, "sm_clock_khz": c.value}

    # ---- memory
    def alloc(self, length: int, dtype=np.float32) -> DeviceBuffer:
        p = ctypes.c_void_p()
        nbytes = int(length) * np.dtype(dtype).itemsize
        _check(self._lib.b2b_malloc(self._h, nbytes, ctypes.byref(p)))
        return DeviceBuffer(self, p.value or 0, length, dtype)

    def host_empty(self, length: int, dtype=np.float32) -> np.ndarray:
        """A numpy array in page-locked host memory from b2b_host_alloc
        (cudaHostAlloc), freed when the array is garbage-collected.  Host
        slices in such memory copy at full PCIe rate in both directions."""
        nbytes = max(int(length) * np.dtype(dtype).itemsize, 1)
        p = ctypes.c_void_p()
        _check(self._lib.b2b_host_alloc(nbytes, ctypes.byref(p)))
        raw = (ctypes.c_char * nbytes).from_address(p.value)
        weakref.finalize(raw, _lib.load().b2b_host_free, ctypes.c_void_p(p.value))
        return np.frombuffer(raw, dtype=dtype, count=int(length))

    def upload(self, host: np.ndarray) -> DeviceBuffer:
        host = np.ascontiguousarray(host)
        dt = np.uint16 if host.dtype == np.float16 else host.dtype
        buf = self.alloc(host.size, dt)
        _check(self._lib.b2b_memcpy_h2d(self._h, ctypes.c_void_p(buf.ptr), _hp(host), host.nbytes))
        return buf

    def upload_into(self, dev: DeviceBuffer, host: np.ndarray) -> None:
        """Copy a host array into an existing device buffer (its first bytes)."""
        host = np.ascontiguousarray(host)
        if host.nbytes > dev.nbytes:
            raise CublasError(2, f"{host.nbytes} bytes do not fit a {dev.nbytes}-byte buffer")
        _check(self._lib.b2b_memcpy_h2d(self._h, ctypes.c_void_p(dev.ptr), _hp(host), host.nbytes))

    def download(self, dev: DeviceBuffer) -> np.ndarray:
        out = np.empty(len(dev), dev.dtype)
        _check(self._lib.b2b_memcpy_d2h(self._h, _hp(out), ctypes.c_void_p(dev.ptr), dev.nbytes))
        return out

    def memset(self, buf: DeviceBuffer, value: int = 0) -> None:
        """Set every byte of `buf` to `value`, ordered on the handle's stream."""
        _check(self._lib.b2b_memset(self._h, ctypes.c_void_p(buf.ptr), int(value), buf.nbytes))

    def zeroed(self, length: int, dtype=np.float32) -> DeviceBuffer:
        return DeviceBuffer.zeroed(self, length, dtype)

    # ---- helpers
    @staticmethod
    def _need(buf: DeviceBuffer, n: int, what: str, dtype) -> None:
        if buf.dtype != np.dtype(dtype):
            raise CublasError(3, f"{what} has dtype {buf.dtype}, expected {np.dtype(dtype)}")
        if len(buf) < n:
            raise CublasError(2, f"dimension mismatch in {what}: expected {n}, got {len(buf)}")

    def _gemm_dev(self, fn, algo, cfg: GemmConfig, a, b, c, dtype):
        m, n, k = cfg.m, cfg.n, cfg.k
        if m and n and k:
            self._need(a, m * k, "A", dtype)
            self._need(b, k * n, "B", dtype)
            self._need(c, m * n, "C", dtype)
        args = [self._h] + ([int(algo)] if algo is not None else []) + [
            m, n, k, cfg.alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(b.ptr), cfg.beta, ctypes.c_void_p(c.ptr)]
        _check(fn(*args))

    def _gemm_host(self, fn, algo, cfg: GemmConfig, a, b, c, dtype):
        a, b, c = _host(a, dtype), _host(b, dtype), _host(c, dtype)
        args = [self._h] + ([int(algo)] if algo is not None else []) + [
            cfg.m, cfg.n, cfg.k, cfg.alpha, _hp(a), a.size, _hp(b), b.size, cfg.beta, _hp(c), c.size]
        _check(fn(*args))

    # ---- Level 3: SGEMM (lib.rs:439-524)
    def sgemm(self, config, a, b, c, algo=Algo.Default):
        self._gemm_dev(self._lib.b2b_sgemm, algo, config, a, b, c, np.float32)

    def sgemm_simple(self, config, a, b, c, algo=Algo.Default):
        self._gemm_host(self._lib.b2b_sgemm_simple, algo, config, a, b, c, np.float32)

    def sgemm_naive(self, config, a, b, c):
        self.sgemm(config, a, b, c, Algo.Naive)

    def sgemm_naive_simple(self, config, a, b, c):
        self.sgemm_simple(config, a, b, c, Algo.Naive)

    def sgemm_tiled(self, config, a, b, c):
        self.sgemm(config, a, b, c, Algo.Tiled)

    def sgemm_tiled_simple(self, config, a, b, c):
        self.sgemm_simple(config, a, b, c, Algo.Tiled)

    def sgemm_vectorized(self, config, a, b, c):
        self.sgemm(config, a, b, c, Algo.Vectorized)

    def sgemm_vectorized_simple(self, config, a, b, c):
        self.sgemm_simple(config, a, b, c, Algo.Vectorized)

    def sgemm_double_buf(self, config, a, b, c):
        self.sgemm(config, a, b, c, Algo.DoubleBuf)

    def sgemm_double_buf_simple(self, config, a, b, c):
        self.sgemm_simple(config, a, b, c, Algo.DoubleBuf)

    def sgemm_bias(self, config, a, b, c, bias=None, relu=False, algo=Algo.Default):
        """C = act(alpha*A*B + beta*C + bias[col]) with the bias broadcast and
        the optional ReLU in the GEMM epilogue (the mlp example's
        sgemm + saxpy(pre-broadcast bias) pair in one kernel)."""
        m, n, k = config.m, config.n, config.k
        if m and n and k:
            self._need(a, m * k, "A", np.float32)
            self._need(b, k * n, "B", np.float32)
            self._need(c, m * n, "C", np.float32)
            if bias is not None:
                self._need(bias, n, "bias", np.float32)
        _check(self._lib.b2b_sgemm_bias(self._h, int(algo), m, n, k, config.alpha, ctypes.c_void_p(a.ptr),
                                        ctypes.c_void_p(b.ptr), config.beta, ctypes.c_void_p(c.ptr),
                                        ctypes.c_void_p(bias.ptr if bias is not None else 0), 1 if relu else 0))

    def sgemm_splits(self, m: int, n: int, k: int) -> int:
        """Number of k ranges the FFMA SGEMM sums separately for an m x n x k
        call (b2b_sgemm_splits; 1 = no split-K)."""
        out = ctypes.c_int(0)
        _check(self._lib.b2b_sgemm_splits(self._h, m, n, k, ctypes.byref(out)))
        return out.value

    def set_sgemm_splits(self, splits: int) -> None:
        """Fix the split-K factor of this handle's later SGEMMs
        (b2b_set_sgemm_splits): 0 = per call (default), 1 = never."""
        _check(self._lib.b2b_set_sgemm_splits(self._h, int(splits)))

    def sgemm_3xtf32(self, config, a, b, c):
        """Opt-in split-precision tensor-core SGEMM (no reference counterpart)."""
        self.sgemm(config, a, b, c, Algo.Tf32x3)

    def sgemm_3xtf32_simple(self, config, a, b, c):
        self.sgemm_simple(config, a, b, c, Algo.Tf32x3)

    # ---- Level 3: DGEMM (lib.rs:527-612)
    def dgemm(self, config, a, b, c, algo=Algo.Default):
        self._gemm_dev(self._lib.b2b_dgemm, algo, config, a, b, c, np.float64)

    def dgemm_simple(self, config, a, b, c, algo=Algo.Default):
        self._gemm_host(self._lib.b2b_dgemm_simple, algo, config, a, b, c, np.float64)

    def dgemm_naive(self, config, a, b, c):
        self.dgemm(config, a, b, c, Algo.Naive)

    def dgemm_naive_simple(self, config, a, b, c):
        self.dgemm_simple(config, a, b, c, Algo.Naive)

    def dgemm_tiled(self, config, a, b, c):
        self.dgemm(config, a, b, c, Algo.Tiled)

    def dgemm_tiled_simple(self, config, a, b, c):
        self.dgemm_simple(config, a, b, c, Algo.Tiled)

    def dgemm_vectorized(self, config, a, b, c):
        self.dgemm(config, a, b, c, Algo.Vectorized)

    def dgemm_vectorized_simple(self, config, a, b, c):
        self.dgemm_simple(config, a, b, c, Algo.Vectorized)

    def dgemm_double_buf(self, config, a, b, c):
        self.dgemm(config, a, b, c, Algo.DoubleBuf)

    def dgemm_double_buf_simple(self, config, a, b, c):
        self.dgemm_simple(config, a, b, c, Algo.DoubleBuf)

    # ---- Level 3: HGEMM (lib.rs:616-635); f16 as np.float16 or its uint16 bits
    def hgemm(self, config, a, b, c):
        """Device-buffer HGEMM (uint16 bit patterns of f16)."""
        self._gemm_dev(self._lib.b2b_hgemm, None, config, a, b, c, np.uint16)

    def hgemm_simple(self, config, a, b, c):
        self._gemm_host(self._lib.b2b_hgemm_simple, None, config, a, b, c, np.uint16)

    def hgemm_half(self, config, a, b, c):
        """Handle::hgemm_half: host slices only, like the reference."""
        self.hgemm_simple(config, a, b, c)

    def hgemm_tensor_core(self, config, a, b, c):
        """Handle::hgemm_tensor_core: the tcgen05 path (a todo! in the reference)."""
        self.hgemm_simple(config, a, b, c)

    # ---- batched (lib.rs:639-709)
    def strided_batched_sgemm(self, config, batch_count, a, stride_a, b, stride_b, c, stride_c):
        m, n, k = config.m, config.n, config.k
        if m and n and k and batch_count:
            self._need(a, (batch_count - 1) * stride_a + m * k, "A", np.float32)
            self._need(b, (batch_count - 1) * stride_b + k * n, "B", np.float32)
            self._need(c, (batch_count - 1) * stride_c + m * n, "C", np.float32)
        _check(self._lib.b2b_sgemm_strided_batched(
            self._h, m, n, k, config.alpha, ctypes.c_void_p(a.ptr), stride_a, ctypes.c_void_p(b.ptr), stride_b,
            config.beta, ctypes.c_void_p(c.ptr), stride_c, batch_count))

    def strided_batched_sgemm_simple(self, config, batch_count, a, stride_a, b, stride_b, c, stride_c):
        a, b, c = _host(a, np.float32), _host(b, np.float32), _host(c, np.float32)
        _check(self._lib.b2b_sgemm_strided_batched_simple(
            self._h, config.m, config.n, config.k, config.alpha, _hp(a), a.size, stride_a, _hp(b), b.size, stride_b,
            config.beta, _hp(c), c.size, stride_c, batch_count))

    def batched_sgemm(self, config, batch_count, a: Sequence[np.ndarray], b: Sequence[np.ndarray],
                      c: Sequence[np.ndarray]):
        if len(a) != batch_count or len(b) != batch_count or len(c) != batch_count:
            # batched.rs:222-224 asserts the slice counts.
            raise CublasError(2, f"slice counts must equal batch_count={batch_count}: "
                                 f"got {len(a)}, {len(b)}, {len(c)}")
        a = [_host(x, np.float32) for x in a]
        b = [_host(x, np.float32) for x in b]
        c = [_host(x, np.float32) for x in c]
        n = batch_count
        pa = (ctypes.c_void_p * max(n, 1))(*[x.ctypes.data for x in a])
        pb = (ctypes.c_void_p * max(n, 1))(*[x.ctypes.data for x in b])
        pc = (ctypes.c_void_p * max(n, 1))(*[x.ctypes.data for x in c])
        la = (ctypes.c_size_t * max(n, 1))(*[x.size for x in a])
        lb = (ctypes.c_size_t * max(n, 1))(*[x.size for x in b])
        lc = (ctypes.c_size_t * max(n, 1))(*[x.size for x in c])
        cast = lambda arr: ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))  # noqa: E731
        _check(self._lib.b2b_sgemm_batched_simple(
            self._h, config.m, config.n, config.k, config.alpha, cast(pa), la, cast(pb), lb, config.beta, cast(pc),
            lc, n))

    # ---- Level 2: SGEMV (lib.rs:230-309)
    def sgemv(self, trans, m, n, alpha, a, x, beta, y, algo=Algo.Default):
        xl, yl = (n, m) if int(trans) == 0 else (m, n)
        if m and n:
            self._need(a, m * n, "A", np.float32)
            self._need(x, xl, "x", np.float32)
            self._need(y, yl, "y", np.float32)
        _check(self._lib.b2b_sgemv(self._h, int(algo), int(trans), m, n, alpha, ctypes.c_void_p(a.ptr),
                                   ctypes.c_void_p(x.ptr), beta, ctypes.c_void_p(y.ptr)))

    def sgemv_simple(self, trans, m, n, alpha, a, x, beta, y, algo=Algo.Default):
        a, x, y = _host(a, np.float32), _host(x, np.float32), _host(y, np.float32)
        _check(self._lib.b2b_sgemv_simple(self._h, int(algo), int(trans), m, n, alpha, _hp(a), a.size, _hp(x),
                                          x.size, beta, _hp(y), y.size))

    def sgemv_tiled(self, trans, m, n, alpha, a, x, beta, y):
        self.sgemv(trans, m, n, alpha, a, x, beta, y, Algo.Tiled)

    def sgemv_tiled_simple(self, trans, m, n, alpha, a, x, beta, y):
        self.sgemv_simple(trans, m, n, alpha, a, x, beta, y, Algo.Tiled)

    # ---- Level 2: DGEMV, HGEMV (lib.rs:312-366)
    def dgemv(self, trans, m, n, alpha, a, x, beta, y):
        xl, yl = (n, m) if int(trans) == 0 else (m, n)
        if m and n:
            self._need(a, m * n, "A", np.float64)
            self._need(x, xl, "x", np.float64)
            self._need(y, yl, "y", np.float64)
        _check(self._lib.b2b_dgemv(self._h, int(trans), m, n, alpha, ctypes.c_void_p(a.ptr),
                                   ctypes.c_void_p(x.ptr), beta, ctypes.c_void_p(y.ptr)))

    def dgemv_simple(self, trans, m, n, alpha, a, x, beta, y):
        a, x, y = _host(a, np.float64), _host(x, np.float64), _host(y, np.float64)
        _check(self._lib.b2b_dgemv_simple(self._h, int(trans), m, n, alpha, _hp(a), a.size, _hp(x), x.size, beta,
                                          _hp(y), y.size))

    def hgemv(self, trans, m, n, alpha, a, x, beta, y):
        """Handle::hgemv: host slices of f16 (np.float16 or uint16 bit
        patterns).  alpha and beta are f16 values in the reference, so they
        are rounded to f16 first and passed on as f32 (gemv.rs:651-652)."""
        a, x, y = _host(a, np.uint16), _host(x, np.uint16), _host(y, np.uint16)
        _check(self._lib.b2b_hgemv_simple(self._h, int(trans), m, n, float(np.float16(alpha)), _hp(a), a.size,
                                          _hp(x), x.size, float(np.float16(beta)), _hp(y), y.size))

    def hgemv_dev(self, trans, m, n, alpha, a, x, beta, y):
        """Device-buffer HGEMV (f16 bit patterns, f32 alpha/beta)."""
        xl, yl = (n, m) if int(trans) == 0 else (m, n)
        if m and n:
            self._need(a, m * n, "A", np.uint16)
            self._need(x, xl, "x", np.uint16)
            self._need(y, yl, "y", np.uint16)
        _check(self._lib.b2b_hgemv(self._h, int(trans), m, n, alpha, ctypes.c_void_p(a.ptr),
                                   ctypes.c_void_p(x.ptr), beta, ctypes.c_void_p(y.ptr)))

    # ---- Level 1: SAXPY (lib.rs:110-129)
    def saxpy(self, n, alpha, x, y):
        if n:
            self._need(x, n, "x", np.float32)
            self._need(y, n, "y", np.float32)
        _check(self._lib.b2b_saxpy(self._h, n, alpha, ctypes.c_void_p(x.ptr), ctypes.c_void_p(y.ptr)))

    def saxpy_simple(self, n, alpha, x, y):
        x, y = _host(x, np.float32), _host(y, np.float32)
        _check(self._lib.b2b_saxpy_simple(self._h, n, alpha, _hp(x), x.size, _hp(y), y.size))

    # ---- Level 1 reductions (lib.rs:157-195)
    class ReduceOp(enum.IntEnum):
        Dot = 0
        Nrm2 = 1
        Asum = 2
        Iamax = 3

    def _reduce_dev(self, fn, n, x, y=None):
        if n:
            self._need(x, n, "x", np.float32)
            if y is not None:
                self._need(y, n, "y", np.float32)
        out = ctypes.c_float()
        args = [self._h, n, ctypes.c_void_p(x.ptr)] + ([ctypes.c_void_p(y.ptr)] if y is not None else [])
        _check(fn(*args, ctypes.byref(out)))
        return out.value

    def _reduce_host(self, fn, n, x, y=None):
        x = _host(x, np.float32)
        args = [self._h, n, _hp(x), x.size]
        if y is not None:
            y = _host(y, np.float32)
            args += [_hp(y), y.size]
        out = ctypes.c_float()
        _check(fn(*args, ctypes.byref(out)))
        return out.value

    def sdot(self, n, x, y) -> float:
        return self._reduce_dev(self._lib.b2b_sdot, n, x, y)

    def sdot_simple(self, n, x, y) -> float:
        return self._reduce_host(self._lib.b2b_sdot_simple, n, x, y)

    def snrm2(self, n, x) -> float:
        return self._reduce_dev(self._lib.b2b_snrm2, n, x)

    def snrm2_simple(self, n, x) -> float:
        return self._reduce_host(self._lib.b2b_snrm2_simple, n, x)

    def sasum(self, n, x) -> float:
        return self._reduce_dev(self._lib.b2b_sasum, n, x)

    def sasum_simple(self, n, x) -> float:
        return self._reduce_host(self._lib.b2b_sasum_simple, n, x)

    def isamax(self, n, x) -> int:
        if n:
            self._need(x, n, "x", np.float32)
        out = ctypes.c_size_t()
        _check(self._lib.b2b_isamax(self._h, n, ctypes.c_void_p(x.ptr), ctypes.byref(out)))
        return out.value

    def isamax_simple(self, n, x) -> int:
        x = _host(x, np.float32)
        out = ctypes.c_size_t()
        _check(self._lib.b2b_isamax_simple(self._h, n, _hp(x), x.size, ctypes.byref(out)))
        return out.value

    def sreduce_async(self, op, n, x, y, result) -> None:
        """Stream-ordered reduction into device memory: `result` is a float32
        DeviceBuffer (Dot, Nrm2, Asum) or a uint64 one (Iamax)."""
        want = np.uint64 if int(op) == 3 else np.float32
        self._need(result, 1, "result", want)
        if n:
            self._need(x, n, "x", np.float32)
            if int(op) == 0:
                self._need(y, n, "y", np.float32)
        _check(self._lib.b2b_sreduce_async(self._h, int(op), n, ctypes.c_void_p(x.ptr if x is not None else 0),
                                           ctypes.c_void_p(y.ptr if y is not None else 0),
                                           ctypes.c_void_p(result.ptr)))

    # ---- self-test of the bounded device waits
    def selftest_bounded_wait(self, limit_ns: int) -> None:
        """Queues a kernel whose wait can never complete; it gives up after
        limit_ns.  The following synchronize() raises CublasError(status=4)."""
        _check(self._lib.b2b_selftest_bounded_wait(self._h, int(limit_ns)))

    # ---- multi-GPU: GEMM with the all-gather folded in
    def _gather(self, fn, dtype, config, a, b, ldc, col_off, dst_ptrs, self_index):
        m, n, k = config.m, config.n, config.k
        if m and n and k:
            self._need(a, m * k, "A", dtype)
            self._need(b, k * n, "B", dtype)
        arr = (ctypes.c_void_p * len(dst_ptrs))(*[int(p) for p in dst_ptrs])
        _check(fn(self._h, m, n, k, config.alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(b.ptr), config.beta,
                  int(ldc), int(col_off), ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), len(dst_ptrs),
                  int(self_index)))

    def hgemm_gather(self, config, a, b, ldc, col_off, dst_ptrs, self_index):
        """This rank's column panel of C = alpha*A*B (+ beta*C) written into
        every rank's full m x ldc C (dst_ptrs, b2b_hgemm_gather)."""
        self._gather(self._lib.b2b_hgemm_gather, np.uint16, config, a, b, ldc, col_off, dst_ptrs, self_index)

    def hgemm_gather_multicast(self, config, a, b, ldc, col_off, mc_ptr, own_ptr):
        """b2b_hgemm_gather_multicast: the gather through an NVLink multicast
        address bound to every rank's C (beta must be 0)."""
        m, n, k = config.m, config.n, config.k
        if config.beta != 0.0:
            raise CublasError(3, "hgemm_gather_multicast needs beta == 0")
        if m and n and k:
            self._need(a, m * k, "A", np.uint16)
            self._need(b, k * n, "B", np.uint16)
        _check(self._lib.b2b_hgemm_gather_multicast(self._h, m, n, k, config.alpha, ctypes.c_void_p(a.ptr),
                                                    ctypes.c_void_p(b.ptr), int(ldc), int(col_off),
                                                    ctypes.c_void_p(int(mc_ptr)), ctypes.c_void_p(int(own_ptr))))

    def sgemm_gather(self, config, a, b, ldc, col_off, dst_ptrs, self_index):
        self._gather(self._lib.b2b_sgemm_gather, np.float32, config, a, b, ldc, col_off, dst_ptrs, self_index)

    def dgemm_gather(self, config, a, b, ldc, col_off, dst_ptrs, self_index):
        self._gather(self._lib.b2b_dgemm_gather, np.float64, config, a, b, ldc, col_off, dst_ptrs, self_index)

    def ipc_get_handle(self, buf: DeviceBuffer) -> bytes:
        """64-byte CUDA IPC handle of a library allocation (its base pointer)."""
        out = ctypes.create_string_buffer(64)
        _check(self._lib.b2b_ipc_get_handle(self._h, ctypes.c_void_p(buf.ptr), out))
        return out.raw

    def ipc_open_handle(self, handle: bytes) -> int:
        """Device pointer (in this process) to the allocation behind `handle`."""
        p = ctypes.c_void_p()
        _check(self._lib.b2b_ipc_open_handle(self._h, ctypes.create_string_buffer(bytes(handle), 64),
                                             ctypes.byref(p)))
        return p.value

    def ipc_close_handle(self, ptr: int) -> None:
        _check(self._lib.b2b_ipc_close_handle(self._h, ctypes.c_void_p(int(ptr))))

    # ---- multi-GPU helper
    def panels_to_rowmajor(self, elem_bytes: int, m: int, widths: Sequence[int], panels_ptr: int, c_ptr: int):
        w = (ctypes.c_size_t * len(widths))(*widths)
        _check(self._lib.b2b_panels_to_rowmajor(self._h, elem_bytes, m, len(widths), w, ctypes.c_void_p(panels_ptr),
                                                ctypes.c_void_p(c_ptr)))
