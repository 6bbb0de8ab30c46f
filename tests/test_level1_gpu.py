"""Level-1 reductions (SDOT, SNRM2, SASUM, ISAMAX) on the GPU, through the C
ABI, against the CPU oracle.

The kernels sum in f64, so the bound is the f32 rounding of the result plus
an f64 accumulation term: |got - exact| <= 2^-24 |exact| + 2 n eps64 S, with
S = sum |x y| (|x|^2, |x|).  ISAMAX is exact: the smallest index of the
largest |x|."""
import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu

EPS64 = float(np.finfo(np.float64).eps)
SIZES = [1, 3, 4, 5, 31, 1000, 4096, 4097, 65537, 1 << 20, (1 << 22) + 3]


def _bound(exact, s, n):
    return 2.0 ** -24 * abs(exact) + 2 * n * EPS64 * s + 1e-38


def test_reduction_known_answers(handle):
    for case in load_golden("known_answers.json")["cases"]:
        op = case["op"]
        if op not in ("sdot", "snrm2", "sasum", "isamax"):
            continue
        n = case["n"]
        x = np.arange(n, dtype=np.float32)
        if op == "isamax":
            assert handle.isamax_simple(n, x) == case["expect"]
            continue
        got = handle.sdot_simple(n, x, x) if op == "sdot" else getattr(handle, f"{op}_simple")(n, x)
        assert abs(got - case["expect"]) / case["expect"] <= case["tol_rel"]
        # and, summing in f64, within an f32 rounding of the closed form
        assert abs(got - case["expect"]) <= 2.0 ** -24 * case["expect"]


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("offset", [0, 1])
def test_reductions_random_parity(handle, oracle, n, offset):
    # offset 1 shifts both vectors off 16-byte alignment (scalar-load path)
    x = oracle.normal_f32(n + offset, 21, 1)
    y = oracle.normal_f32(n + offset, 21, 2)
    xb, yb = handle.upload(x), handle.upload(y)
    xd = type(xb).from_ptr(handle, xb.ptr + 4 * offset, n, np.float32, owner=xb)
    yd = type(yb).from_ptr(handle, yb.ptr + 4 * offset, n, np.float32, owner=yb)
    xs, ys = x[offset:], y[offset:]
    x64, y64 = xs.astype(np.float64), ys.astype(np.float64)

    exact = oracle.sdot_f64(n, xs, ys)
    got = handle.sdot(n, xd, yd)
    assert abs(got - exact) <= _bound(exact, float(np.abs(x64 * y64).sum()), n)
    assert handle.sdot_simple(n, xs, ys) == got

    exact = oracle.snrm2_f64(n, xs)
    got = handle.snrm2(n, xd)
    assert abs(got - exact) <= 2.0 ** -23 * exact
    assert handle.snrm2_simple(n, xs) == got

    exact = oracle.sasum_f64(n, xs)
    got = handle.sasum(n, xd)
    assert abs(got - exact) <= _bound(exact, exact, n)
    assert handle.sasum_simple(n, xs) == got

    want = oracle.isamax(n, xs)
    assert handle.isamax(n, xd) == want
    assert handle.isamax_simple(n, xs) == want


def test_reductions_repeatable_and_async(handle, oracle):
    import b2blas

    n = (1 << 24) + 5
    x = oracle.normal_f32(n, 22, 1)
    y = oracle.normal_f32(n, 22, 2)
    xd, yd = handle.upload(x), handle.upload(y)
    first = [handle.sdot(n, xd, yd), handle.snrm2(n, xd), handle.sasum(n, xd), handle.isamax(n, xd)]
    for _ in range(3):  # fixed partial sets and a fixed final order: bitwise repeatable
        again = [handle.sdot(n, xd, yd), handle.snrm2(n, xd), handle.sasum(n, xd), handle.isamax(n, xd)]
        assert again == first
    # the stream-ordered flavour writes the same values to device memory
    f = handle.zeroed(1, np.float32)
    u = handle.zeroed(1, np.uint64)
    Op = b2blas.Handle.ReduceOp
    for op, want in ((Op.Dot, first[0]), (Op.Nrm2, first[1]), (Op.Asum, first[2])):
        handle.sreduce_async(op, n, xd, yd if op == Op.Dot else None, f)
        handle.synchronize()
        assert float(handle.download(f)[0]) == want
    handle.sreduce_async(Op.Iamax, n, xd, None, u)
    handle.synchronize()
    assert int(handle.download(u)[0]) == first[3]
    # n == 0 writes a zero result
    handle.sreduce_async(Op.Iamax, 0, xd, None, u)
    handle.synchronize()
    assert int(handle.download(u)[0]) == 0


def test_reductions_special_values(handle, oracle):
    # |x| up to 1e30: the f32 sum of squares the reference forms overflows;
    # the f64 one here does not.
    x = np.array([3e30, -4e30] + [0.0] * 1000, np.float32)
    assert handle.snrm2_simple(x.size, x) == pytest.approx(5e30, rel=2 ** -23)
    # tiny values: no underflow to zero either
    x = np.array([3e-30, 4e-30], np.float32)
    assert handle.snrm2_simple(2, x) == pytest.approx(5e-30, rel=2 ** -23)
    # ISAMAX: ties -> smallest index (in different blocks and lanes), NaN skipped
    n = 1 << 20
    x = np.zeros(n, np.float32)
    x[n - 7] = -9.0
    x[12345] = 9.0
    x[777777] = 9.0
    assert handle.isamax_simple(n, x) == 12345
    x[100] = np.nan
    assert handle.isamax_simple(n, x) == 12345
    assert handle.isamax_simple(5, np.full(5, np.nan, np.float32)) == 0
    # inf wins; a NaN operand of dot gives NaN
    x[999] = -np.inf
    assert handle.isamax_simple(n, x) == 999
    assert np.isnan(handle.sdot_simple(4, np.array([1, np.nan, 2, 3], np.float32), np.ones(4, np.float32)))


def test_reductions_lengths_and_empty(handle):
    import b2blas

    assert handle.sdot_simple(0, np.zeros(0, np.float32), np.zeros(0, np.float32)) == 0.0
    assert handle.isamax_simple(0, np.zeros(0, np.float32)) == 0
    assert handle.snrm2_simple(0, np.zeros(3, np.float32)) == 0.0
    with pytest.raises(b2blas.CublasError) as e:
        handle.sdot_simple(5, np.zeros(5, np.float32), np.zeros(4, np.float32))
    assert e.value.kind == "DimensionMismatch"
    with pytest.raises(b2blas.CublasError) as e:
        handle.isamax_simple(5, np.zeros(4, np.float32))
    assert e.value.kind == "DimensionMismatch"
    # only x[..n] counts (dot.rs:93-94): a larger tail is ignored
    x = np.array([1, 2, 3, 100], np.float32)
    assert handle.sasum_simple(3, x) == 6.0
    assert handle.isamax_simple(3, x) == 2
