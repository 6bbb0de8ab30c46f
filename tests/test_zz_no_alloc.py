"""b2b_sgemv_noalloc: the SGEMV entry point that allocates no device memory,
for callers that cannot call cudaMalloc/cudaFree (their device memory is
owned by another allocator, or fixed at start-up, or they cannot afford the
synchronisation cudaFree implies).  Its transposed path keeps the split-row
partial sums in a fixed device array built into the library instead of
handle workspace.

Checked through the C ABI against b2b_sgemv (the existing entry point) on
two calls in a row, with the SGEMV tolerance 4*m*eps(f32) normwise; the two
calls use different inputs, so a stale partial from the first call would
show up in the second.  Collected last (file name), and self-contained: it
makes its own handle, so it passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(lib, h, fn, trans, m, n, alpha, A, x, beta, y0):
    import b2blas

    a, xd, yd = h.upload(A), h.upload(x), h.upload(y0)
    if fn == "noalloc":
        rc = lib.b2b_sgemv_noalloc(h._h, trans, m, n, alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(xd.ptr), beta,
                                   ctypes.c_void_p(yd.ptr))
    else:
        rc = lib.b2b_sgemv(h._h, 0, trans, m, n, alpha, ctypes.c_void_p(a.ptr), ctypes.c_void_p(xd.ptr), beta,
                           ctypes.c_void_p(yd.ptr))
    assert rc == 0, lib.b2b_last_error()
    h.synchronize()
    out = h.download(yd)
    for buf in (a, xd, yd):
        buf.free()
    return out


@pytest.mark.parametrize("trans,m,n", [(1, 4096, 16384), (1, 3000, 1000), (0, 2048, 4096)])
def test_noalloc_matches_sgemv_two_calls_in_a_row(trans, m, n):
    import b2blas

    lib = b2blas.load_library()
    h = b2blas.Handle(0)
    try:
        rng = np.random.default_rng(1234)
        tol = 4.0 * (n if trans == 0 else m) * np.finfo(np.float32).eps
        xl, yl = (n, m) if trans == 0 else (m, n)
        for call in range(2):
            A = rng.uniform(-1, 1, m * n).astype(np.float32)
            x = rng.uniform(-1, 1, xl).astype(np.float32)
            y = rng.uniform(-1, 1, yl).astype(np.float32)
            alpha, beta = (1.0, 0.0) if call == 0 else (1.5, -0.5)
            ref = _run(lib, h, "sgemv", trans, m, n, alpha, A, x, beta, y)
            got = _run(lib, h, "noalloc", trans, m, n, alpha, A, x, beta, y)
            err = np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref.astype(np.float64))
            assert err <= tol, (call, err)
    finally:
        h.close()
