"""b2b_sgemv_noalloc: the SGEMV entry point that allocates no device memory,
for callers that cannot call cudaMalloc/cudaFree (their device memory is
owned by another allocator, or fixed at start-up, or they cannot afford the
synchronisation cudaFree implies).  Its transposed path keeps the split-row
partial sums in a fixed device array built into the library instead of
handle workspace.

Checked through the C ABI:
  * against b2b_sgemv (the existing entry point), bit for bit -- both slice
    the rows the same way -- and against the FP64 oracle within the SGEMV
    tolerance 4*len*eps(f32) normwise, on two calls in a row with different
    inputs, so a stale partial from the first call would show in the second;
  * that a fresh handle's noalloc calls leave the device's memory pool (the
    one the handle workspace grows from) untouched, while b2b_sgemv on the
    same handle grows it (the check can see an allocation);
  * the rejection of a shape whose partials do not fit the array: before any
    launch, with B2B_ERR_INVALID_ARG and a message naming the sizes, and y
    unchanged.  No shape exceeds the 2^18-float array on a 148-SM GPU, so the
    case uses a handle created with a lower limit (B2B_NOALLOC_SCRATCH_FLOATS)
    and real device buffers.
Collected last (file name), and self-contained: every test makes its own
handle, so the file passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

B2B_ERR_INVALID_ARG = 3


def _call(lib, h, fn, trans, m, n, alpha, a, xd, beta, yd):
    if fn == "noalloc":
        return lib.b2b_sgemv_noalloc(h._h, trans, m, n, alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(xd.ptr),
                                     beta, ctypes.c_void_p(yd.ptr))
    return lib.b2b_sgemv(h._h, 0, trans, m, n, alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(xd.ptr), beta,
                         ctypes.c_void_p(yd.ptr))


def _run(lib, h, fn, trans, m, n, alpha, A, x, beta, y0):
    a, xd, yd = h.upload(A), h.upload(x), h.upload(y0)
    rc = _call(lib, h, fn, trans, m, n, alpha, a, xd, beta, yd)
    assert rc == 0, lib.b2b_last_error()
    h.synchronize()
    out = h.download(yd)
    for buf in (a, xd, yd):
        buf.free()
    return out


def _pool_used_bytes(device=0):
    """Bytes in use from the device's current memory pool, the pool the
    library's stream-ordered workspace allocations come from (driver API:
    cuDeviceGetMemPool + CU_MEMPOOL_ATTR_USED_MEM_CURRENT)."""
    cu = ctypes.CDLL("libcuda.so.1")
    dev = ctypes.c_int()
    assert cu.cuDeviceGet(ctypes.byref(dev), device) == 0
    pool = ctypes.c_void_p()
    assert cu.cuDeviceGetMemPool(ctypes.byref(pool), dev) == 0
    used = ctypes.c_uint64()
    CU_MEMPOOL_ATTR_USED_MEM_CURRENT = 7
    assert cu.cuMemPoolGetAttribute(pool, CU_MEMPOOL_ATTR_USED_MEM_CURRENT, ctypes.byref(used)) == 0
    return used.value


@pytest.mark.parametrize("trans,m,n", [(1, 4096, 16384), (1, 3000, 1000), (0, 2048, 4096)])
def test_noalloc_matches_sgemv_two_calls_in_a_row(trans, m, n):
    import b2blas

    lib = b2blas.load_library()
    h = b2blas.Handle(0)
    try:
        rng = np.random.default_rng(1234)
        tol = oracle.tol_normwise(n if trans == 0 else m, "f32")
        xl, yl = (n, m) if trans == 0 else (m, n)
        for call in range(2):
            A = rng.uniform(-1, 1, m * n).astype(np.float32)
            x = rng.uniform(-1, 1, xl).astype(np.float32)
            y = rng.uniform(-1, 1, yl).astype(np.float32)
            alpha, beta = (1.0, 0.0) if call == 0 else (1.5, -0.5)
            ref = _run(lib, h, "sgemv", trans, m, n, alpha, A, x, beta, y)
            got = _run(lib, h, "noalloc", trans, m, n, alpha, A, x, beta, y)
            assert np.array_equal(got, ref), (call, "noalloc and b2b_sgemv differ in bits")
            exact = oracle.sgemv_f64(trans, m, n, alpha, A, x, beta, y)
            err = oracle.rel_err(got, exact)
            assert err <= tol, (call, err, tol)
    finally:
        h.close()


def test_noalloc_leaves_the_memory_pool_untouched():
    import b2blas

    lib = b2blas.load_library()
    h = b2blas.Handle(0)  # fresh handle: its workspace has never grown
    try:
        m, n = 4096, 16384  # T: 5 slices of partials on 148 SMs
        rng = np.random.default_rng(99)
        A = rng.uniform(-1, 1, m * n).astype(np.float32)
        x = rng.uniform(-1, 1, m).astype(np.float32)
        y = np.zeros(n, np.float32)
        a, xd, yd = h.upload(A), h.upload(x), h.upload(y)
        h.synchronize()
        before = _pool_used_bytes()
        for _ in range(2):
            assert _call(lib, h, "noalloc", 1, m, n, 1.0, a, xd, 0.0, yd) == 0, lib.b2b_last_error()
        h.synchronize()
        assert _pool_used_bytes() == before
        # control: the allocating entry point grows the handle's workspace
        # from the same pool, which this check sees
        assert _call(lib, h, "sgemv", 1, m, n, 1.0, a, xd, 0.0, yd) == 0, lib.b2b_last_error()
        h.synchronize()
        assert _pool_used_bytes() > before
        for buf in (a, xd, yd):
            buf.free()
    finally:
        h.close()


def test_noalloc_rejects_a_shape_beyond_the_limit(monkeypatch):
    import b2blas

    lib = b2blas.load_library()
    monkeypatch.setenv("B2B_NOALLOC_SCRATCH_FLOATS", "1024")
    h = b2blas.Handle(0)  # reads the lower limit at creation
    monkeypatch.delenv("B2B_NOALLOC_SCRATCH_FLOATS")
    try:
        m, n = 4096, 16384  # T: 5 x 16384 partials > 1024
        rng = np.random.default_rng(7)
        A = rng.uniform(-1, 1, m * n).astype(np.float32)
        x = rng.uniform(-1, 1, m).astype(np.float32)
        y = rng.uniform(-1, 1, n).astype(np.float32)
        a, xd, yd = h.upload(A), h.upload(x), h.upload(y)
        rc = _call(lib, h, "noalloc", 1, m, n, 1.5, a, xd, 0.5, yd)
        assert rc == B2B_ERR_INVALID_ARG
        msg = lib.b2b_last_error()
        msg = msg.decode() if isinstance(msg, bytes) else str(msg)
        assert "16384" in msg and "1024" in msg, msg
        h.synchronize()
        assert np.array_equal(h.download(yd), y)  # nothing ran
        # N needs no scratch and is unaffected by the limit; a T shape whose
        # single slice writes y directly is too
        assert _call(lib, h, "noalloc", 0, 64, 16, 1.0, a, xd, 0.0, yd) == 0, lib.b2b_last_error()
        for buf in (a, xd, yd):
            buf.free()
    finally:
        h.close()
