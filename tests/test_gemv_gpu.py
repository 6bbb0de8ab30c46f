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


# ------------------------------------------------------------ DGEMV, HGEMV
# DGEMV: 4*n_inner*eps(f64) normwise against the Dot2-compensated oracle.
# HGEMV: f16 output rounding (2^-11 relative) plus f32 accumulation,
# 2^-11 + 4*n_inner*eps(f32) normwise against the exact f64 evaluation.

XSHAPES = [(1, 1), (16, 24), (33, 65), (1000, 999), (4096, 4104), (5, 20000), (20000, 5), (300, 130), (7, 4096)]


def _hgemv_tol(inner):
    return 2.0 ** -11 + 4 * inner * float(np.finfo(np.float32).eps)


@pytest.mark.parametrize("m,n", XSHAPES)
@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, -0.5)])
def test_dgemv_random_parity(handle, oracle, m, n, trans, alpha, beta):
    A = oracle.uniform_f64(m * n, 43, 1)
    xl, yl = (n, m) if trans == 0 else (m, n)
    x = oracle.uniform_f64(xl, 43, 4)
    y = oracle.uniform_f64(yl, 43, 5)
    ref = oracle.dgemv_f64(trans, m, n, alpha, A, x, beta, y)
    a, xd, yd = handle.upload(A), handle.upload(x), handle.upload(y)
    handle.dgemv(trans, m, n, alpha, a, xd, beta, yd)
    handle.synchronize()
    got = handle.download(yd)
    inner = n if trans == 0 else m
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(inner, "f64")
    host = y.copy()
    handle.dgemv_simple(trans, m, n, alpha, A, x, beta, host)
    assert np.array_equal(host, got)


@pytest.mark.parametrize("m,n", XSHAPES)
@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, -0.5)])
def test_hgemv_random_parity(handle, oracle, m, n, trans, alpha, beta):
    A = oracle.uniform_f16(m * n, 44, 1)
    xl, yl = (n, m) if trans == 0 else (m, n)
    x = oracle.uniform_f16(xl, 44, 4)
    y = oracle.uniform_f16(yl, 44, 5)
    ref = oracle.hgemv_f64(trans, m, n, alpha, A, x, beta, y)
    inner = n if trans == 0 else m
    host = y.copy()
    handle.hgemv(trans, m, n, alpha, A, x, beta, host)  # host slices, as Handle::hgemv
    assert oracle.rel_err(host, ref) <= _hgemv_tol(inner)
    a, xd, yd = handle.upload(A), handle.upload(x), handle.upload(y)
    handle.hgemv_dev(trans, m, n, alpha, a, xd, beta, yd)
    handle.synchronize()
    assert np.array_equal(handle.download(yd), host)
    # The reference's own arithmetic truncates on encode (up to an f16 ulp,
    # 2^-10, where round-to-nearest gives half of it): within that bound.
    refarith = oracle.hgemv_ref(trans, m, n, alpha, A, x, beta, y)
    assert oracle.rel_err(refarith, ref) <= 2.0 ** -10 + 4 * inner * float(np.finfo(np.float32).eps)


def test_hgemv_known_answer(handle, oracle):
    from test_oracle import hgemv_ramp, hgemv_ramp_expect

    case = [c for c in load_golden("known_answers.json")["cases"] if c["op"] == "hgemv"][0]
    m, n = case["m"], case["n"]
    a16, x16 = hgemv_ramp(m, n)
    y = np.zeros(m, np.float16)
    handle.hgemv(0, m, n, 1.0, a16.view(np.float16), x16.view(np.float16), 0.0, y)
    expect = hgemv_ramp_expect(a16, x16, m, n)
    err = np.abs(y.astype(np.float32) - expect) / np.maximum(np.abs(expect), 1e-6)
    assert np.max(err) <= case["tol_rel"]


@pytest.mark.parametrize("prec", ["d", "h"])
def test_gemv_ext_beta_zero_ignores_y_and_unaligned(handle, oracle, prec):
    # beta == 0 never reads y (NaN stays out); pointers offset by one element
    # take the scalar path and agree with the aligned result.
    m, n = 257, 264
    dt = np.float64 if prec == "d" else np.uint16
    A = oracle.uniform_f64(m * n + 1, 45, 1) if prec == "d" else oracle.uniform_f16(m * n + 1, 45, 1)
    x = oracle.uniform_f64(n + 1, 45, 2) if prec == "d" else oracle.uniform_f16(n + 1, 45, 2)
    nan = np.full(m + 1, np.nan, np.float64) if prec == "d" else np.full(m + 1, 0x7E00, np.uint16)
    a, xd = handle.upload(A), handle.upload(x)
    for off in (0, 1):
        yd = handle.upload(nan)
        av = type(a).from_ptr(handle, a.ptr + off * a.dtype.itemsize, m * n, dt, owner=a)
        xv = type(xd).from_ptr(handle, xd.ptr + off * xd.dtype.itemsize, n, dt, owner=xd)
        yv = type(yd).from_ptr(handle, yd.ptr, m, dt, owner=yd)
        (handle.dgemv if prec == "d" else handle.hgemv_dev)(0, m, n, 1.0, av, xv, 0.0, yv)
        handle.synchronize()
        got = handle.download(yd)[:m]
        Ao, xo = A[off:off + m * n], x[off:off + n]
        ref = (oracle.dgemv_f64 if prec == "d" else oracle.hgemv_f64)(0, m, n, 1.0, Ao, xo, 0.0, nan[:m])
        assert oracle.rel_err(got, ref) <= (oracle.tol_normwise(n, "f64") if prec == "d" else _hgemv_tol(n))


def test_gemv_ext_host_length_checks(handle):
    import b2blas

    with pytest.raises(b2blas.CublasError) as e:
        handle.dgemv_simple(0, 4, 5, 1.0, np.zeros(19), np.zeros(5), 0.0, np.zeros(4))
    assert e.value.kind == "DimensionMismatch"
    with pytest.raises(b2blas.CublasError) as e:
        handle.hgemv(1, 4, 5, 1.0, np.zeros(20, np.float16), np.zeros(3, np.float16), 0.0, np.zeros(5, np.float16))
    assert e.value.kind == "DimensionMismatch"
    with pytest.raises(b2blas.CublasError) as e:
        handle.hgemv(0, 4, 5, 1.0, np.zeros(20, np.float16), np.zeros(5, np.float16), 0.0, np.zeros(3, np.float16))
    assert e.value.kind == "DimensionMismatch"
    # zero dimensions: Ok, y untouched (gemv.rs:497-499)
    y = np.full(3, 7.0)
    handle.dgemv_simple(0, 0, 5, 1.0, np.zeros(0), np.zeros(5), 0.0, y)
    assert np.all(y == 7.0)


def test_dgemv_hgemv_full_size(handle, oracle):
    # 8192 x 8192 f64 (512 MiB) and 16384 x 16384 f16 (512 MiB), both shapes.
    m = n = 8192
    A = oracle.uniform_f64(m * n, 46, 1)
    x = oracle.uniform_f64(n, 46, 2)
    a, xd, yd = handle.upload(A), handle.upload(x), handle.alloc(n, np.float64)
    for trans in (0, 1):
        ref = oracle.dgemv_f64(trans, m, n, 1.0, A, x, 0.0, np.zeros(n))
        handle.dgemv(trans, m, n, 1.0, a, xd, 0.0, yd)
        handle.synchronize()
        assert oracle.rel_err(handle.download(yd), ref) <= oracle.tol_normwise(n, "f64")
    del a
    m = n = 16384
    A = oracle.uniform_f16(m * n, 46, 3)
    x = oracle.uniform_f16(n, 46, 4)
    a, xd, yd = handle.upload(A), handle.upload(x), handle.alloc(n, np.uint16)
    for trans in (0, 1):
        ref = oracle.hgemv_f64(trans, m, n, 1.0, A, x, 0.0, np.zeros(n, np.uint16))
        handle.hgemv_dev(trans, m, n, 1.0, a, xd, 0.0, yd)
        handle.synchronize()
        assert oracle.rel_err(handle.download(yd), ref) <= _hgemv_tol(n)
