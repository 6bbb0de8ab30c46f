"""SGEMV (N and T) and SAXPY parity on the GPU, through the C ABI, against
the CPU oracle.  SGEMV tolerance: 4*n_inner*eps(f32) normwise."""
import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu


def test_sgemv_known_answers(handle):
    import b2blas

    for case in load_golden("known_answers.json")["cases"]:
        if case["op"] != "sgemv":
            continue
        m, n = case["m"], case["n"]
        t = b2blas.Transpose.NoTrans if case["trans"] == "N" else b2blas.Transpose.Trans
        xl, yl = (n, m) if case["trans"] == "N" else (m, n)
        for fn in (handle.sgemv_simple, handle.sgemv_tiled_simple):
            y = np.zeros(yl, np.float32)
            fn(t, m, n, 1.0, np.ones(m * n, np.float32), np.ones(xl, np.float32), 0.0, y)
            assert np.max(np.abs(y - case["expect"])) <= case["tol_abs"]


SHAPES = [(1, 1), (16, 24), (33, 65), (1000, 999), (4096, 4100), (5, 20000), (20000, 5), (16384, 1024),
          (300, 130)]


@pytest.mark.parametrize("m,n", SHAPES)
@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, -0.5)])
def test_sgemv_random_parity(handle, oracle, m, n, trans, alpha, beta):
    A = oracle.uniform_f32(m * n, 42, 1)
    xl, yl = (n, m) if trans == 0 else (m, n)
    x = oracle.uniform_f32(xl, 42, 4)
    y = oracle.uniform_f32(yl, 42, 5)
    ref = oracle.sgemv_f64(trans, m, n, alpha, A, x, beta, y)
    a, xd, yd = handle.upload(A), handle.upload(x), handle.upload(y)
    handle.sgemv(trans, m, n, alpha, a, xd, beta, yd)
    handle.synchronize()
    got = handle.download(yd)
    inner = n if trans == 0 else m
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(inner, "f32")
    host = y.copy()
    handle.sgemv_simple(trans, m, n, alpha, A, x, beta, host)
    assert np.array_equal(host, got)


def test_sgemv_16384_full_size(handle, oracle):
    # The decode configuration: 16384 x 16384, N, alpha 1, beta 0, full check.
    m = n = 16384
    A = oracle.uniform_f32(m * n, 42, 1)
    x = oracle.uniform_f32(n, 42, 4)
    ref = oracle.sgemv_f64(0, m, n, 1.0, A, x, 0.0, np.zeros(m, np.float32))
    a, xd, yd = handle.upload(A), handle.upload(x), handle.zeroed(m)
    handle.sgemv(0, m, n, 1.0, a, xd, 0.0, yd)
    handle.synchronize()
    assert oracle.rel_err(handle.download(yd), ref) <= oracle.tol_normwise(n, "f32")
    # and the transposed product of the same matrix
    refT = oracle.sgemv_f64(1, m, n, 1.0, A, x, 0.0, np.zeros(n, np.float32))
    handle.sgemv(1, m, n, 1.0, a, xd, 0.0, yd)
    handle.synchronize()
    assert oracle.rel_err(handle.download(yd), refT) <= oracle.tol_normwise(m, "f32")


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 1 << 20, (1 << 20) + 3])
def test_saxpy_parity(handle, oracle, n):
    x = oracle.uniform_f32(n, 5, 1)
    y = oracle.uniform_f32(n, 5, 2)
    ref = oracle.saxpy_f64(n, 2.5, x, y)
    xd, yd = handle.upload(x), handle.upload(y)
    handle.saxpy(n, 2.5, xd, yd)
    handle.synchronize()
    got = handle.download(yd)
    # one fused multiply-add per element: within 1 ulp of the exact value
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)) <= 2 * np.finfo(np.float32).eps
    host = y.copy()
    handle.saxpy_simple(n, 2.5, x, host)
    assert np.array_equal(host, got)


def test_saxpy_known_answer_bias_pattern(handle):
    # The mlp example's bias step: Z += broadcast(bias) via saxpy
    # (examples/mlp/src/main.rs:140-145).
    rows, cols = 128, 256
    z = np.zeros(rows * cols, np.float32)
    bias = np.tile(np.full(cols, 0.1, np.float32), rows)
    handle.saxpy_simple(rows * cols, 1.0, bias, z)
    assert np.allclose(z, 0.1)
