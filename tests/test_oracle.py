"""The CPU oracle against the golden vectors (CPU only).

Pins: the PCG32 published known-answer sequence, the reference's own f16
conversion branches (crates/cublas-l3/src/hgemm.rs:20-51), and every
all-ones known answer of the reference's example binaries.  Also checks that
the tolerance machinery rejects a planted error.
"""
import math

import numpy as np
import pytest

from conftest import load_golden


def test_pcg32_known_answer(oracle):
    kat = load_golden("pcg32_kat.json")
    got = oracle.pcg32(kat["seed"], kat["stream"], len(kat["outputs"]))
    assert [int(v) for v in got] == kat["outputs"]


def _dec(x):
    return {"nan": float("nan"), "inf": float("inf"), "-inf": float("-inf")}.get(x, x)


def test_reference_f32_to_f16_branches(oracle):
    for row in load_golden("f16_conversions.json")["f32_to_f16"]:
        x = np.float32(_dec(row["x"]))
        assert oracle.ref_f32_to_f16(float(x)) == row["bits"], row["why"]


def test_reference_f16_to_f32_branches(oracle):
    for row in load_golden("f16_conversions.json")["f16_to_f32"]:
        got = oracle.ref_f16_to_f32(row["bits"])
        want = _dec(row["x"])
        assert got == want, row["why"]
        if want == 0.0:
            assert math.copysign(1.0, got) == (-1.0 if row["negzero"] else 1.0), row["why"]


def test_rne_f16_matches_numpy(oracle):
    # The round-to-nearest-even encoder used for inputs agrees with numpy's
    # IEEE float16 conversion on a sweep including subnormals and ties.
    xs = np.concatenate([
        np.linspace(-70000, 70000, 4001),
        np.linspace(-1e-4, 1e-4, 4001),
        (np.arange(-2048, 2049) * 2.0 ** -25),
        np.array([65504.0, 65519.99, 65520.0, 1 + 2 ** -11, 1 + 3 * 2 ** -11, 2 ** -24, 2 ** -25, 3 * 2 ** -26]),
    ])
    for x in xs:
        assert oracle.f64_to_f16_rne(float(x)) == int(np.float16(x).view(np.uint16)), x
    # Exact widening round-trips every finite f16.
    bits = np.arange(0, 0x10000, dtype=np.uint32).astype(np.uint16)
    finite = bits[(bits & 0x7C00) != 0x7C00]
    want = finite.view(np.float16).astype(np.float64)
    got = np.array([oracle.f16_to_f64(int(b)) for b in finite[::7]])
    assert np.array_equal(got, want[::7])


def hgemv_ramp(m, n):
    """The saxpy example's HGEMV inputs: a[i] = f16(0.01 i), x[j] = f16(0.1 j)
    (examples/saxpy/src/main.rs:133-137), as f16 bit patterns."""
    a16 = (np.arange(m * n, dtype=np.float32) * np.float32(0.01)).astype(np.float16).view(np.uint16)
    x16 = (np.arange(n, dtype=np.float32) * np.float32(0.1)).astype(np.float16).view(np.uint16)
    return a16, x16


def hgemv_ramp_expect(a16, x16, m, n):
    """The example's check value: f32 sum in j order of the f16 products
    (examples/saxpy/src/main.rs:151-157)."""
    a = a16.view(np.float16).astype(np.float32).reshape(m, n)
    x = x16.view(np.float16).astype(np.float32)
    out = np.zeros(m, np.float32)
    for j in range(n):
        out += a[:, j] * x[j]
    return out


def _ones(n, dt=np.float32):
    return np.ones(n, dt)


@pytest.mark.parametrize("case", [c for c in load_golden("known_answers.json")["cases"]],
                         ids=lambda c: f"{c['op']}-{c.get('m', 1)}x{c['n']}")
def test_known_answers_through_oracle(oracle, case):
    op, m, n = case["op"], case.get("m", 1), case["n"]
    if op in ("sgemm", "dgemm"):
        k = case["k"]
        dt = np.float32 if op == "sgemm" else np.float64
        f = oracle.sgemm_f64 if op == "sgemm" else oracle.dgemm_f64
        out = f(m, n, k, case["alpha"], _ones(m * k, dt), _ones(k * n, dt), case["beta"], _ones(m * n, dt))
        assert np.max(np.abs(out - case["expect"])) <= case["tol_abs"]
        if op == "sgemm" and m <= 512:
            ref = oracle.sgemm_ref_f32(m, n, k, case["alpha"], _ones(m * k), _ones(k * n), case["beta"],
                                       np.zeros(m * n, np.float32))
            assert np.max(np.abs(ref - case["expect"])) <= case["tol_abs"]
    elif op in ("strided_batched_sgemm", "batched_sgemm"):
        b, k = case["batch"], case["k"]
        out = oracle.sgemm_strided_batched_f64(m, n, k, 1.0, _ones(b * m * k), m * k, _ones(b * k * n), k * n, 0.0,
                                               None, m * n, b)
        assert np.max(np.abs(out - case["expect"])) <= case["tol_abs"]
    elif op == "hgemm":
        k = case["k"]
        one = np.full(m * k, 0x3C00, np.uint16)
        c = oracle.hgemm_ref(m, n, k, 1.0, one, np.full(k * n, 0x3C00, np.uint16), 0.0, np.zeros(m * n, np.uint16))
        vals = c.view(np.float16).astype(np.float64)
        assert np.max(np.abs(vals - case["expect"]) / case["expect"]) <= case["tol_rel"]
    elif op == "sgemv":
        trans = 0 if case["trans"] == "N" else 1
        xl, yl = (n, m) if trans == 0 else (m, n)
        out = oracle.sgemv_f64(trans, m, n, 1.0, _ones(m * n), _ones(xl), 0.0, np.zeros(yl, np.float32))
        assert np.max(np.abs(out - case["expect"])) <= case["tol_abs"]
    elif op == "hgemv":
        a16, x16 = hgemv_ramp(m, n)
        got = oracle.hgemv_ref(0, m, n, 1.0, a16, x16, 0.0, np.zeros(m, np.uint16)).view(np.float16)
        expect = hgemv_ramp_expect(a16, x16, m, n)
        err = np.abs(got.astype(np.float32) - expect) / np.maximum(np.abs(expect), 1e-6)
        assert np.max(err) <= case["tol_rel"]
        exact = oracle.hgemv_f64(0, m, n, 1.0, a16, x16, 0.0, np.zeros(m, np.uint16))
        np.testing.assert_allclose(expect, exact, rtol=1e-5)
    elif op in ("sdot", "snrm2", "sasum"):
        x = np.arange(n, dtype=np.float32)
        exact = {"sdot": lambda: oracle.sdot_f64(n, x, x), "snrm2": lambda: oracle.snrm2_f64(n, x),
                 "sasum": lambda: oracle.sasum_f64(n, x)}[op]()
        assert exact == pytest.approx(case["expect"], rel=1e-15)
        ref = oracle.sreduce_ref({"sdot": "dot", "snrm2": "nrm2", "sasum": "asum"}[op], n, x, x)
        assert abs(ref - case["expect"]) / case["expect"] <= case["tol_rel"]
    elif op == "isamax":
        x = np.arange(n, dtype=np.float32)
        assert oracle.isamax(n, x) == case["expect"]
        assert oracle.isamax_ref(n, x) == case["expect"]
    else:
        raise AssertionError(op)


def test_reference_f32_arithmetic_within_bound(oracle):
    # The reference's f32 loop (sum += a*b in k order) lands within the
    # 4*K*eps normwise bound of the FP64 evaluation on random data.
    m, n, k = 64, 48, 512
    A = oracle.uniform_f32(m * k, 42, 1)
    B = oracle.uniform_f32(k * n, 42, 2)
    C = oracle.uniform_f32(m * n, 42, 3)
    ref64 = oracle.sgemm_f64(m, n, k, 1.5, A, B, 0.5, C)
    ref32 = oracle.sgemm_ref_f32(m, n, k, 1.5, A, B, 0.5, C)
    assert oracle.rel_err(ref32, ref64) <= oracle.tol_normwise(k, "f32")


def test_planted_error_is_caught(oracle):
    # A mistake planted in the oracle's output (one element off by 1%) must
    # push the normwise error over the FP32 bound at K=512.
    m, n, k = 32, 32, 512
    A = oracle.uniform_f32(m * k, 7, 1)
    B = oracle.uniform_f32(k * n, 7, 2)
    ref = oracle.sgemm_f64(m, n, k, 1.0, A, B)
    bad = ref.astype(np.float32)
    bad[5] *= 1.25
    assert oracle.rel_err(bad, ref) > oracle.tol_normwise(k, "f32")


def test_hgemm_reference_arithmetic_within_tolerance(oracle):
    m, n, k = 48, 40, 256
    A = oracle.normal_f16(m * k, 42, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 42, 2, 0.0, 0.1)
    ref64 = oracle.hgemm_f64(m, n, k, 1.0, A, B)
    refc = oracle.hgemm_ref(m, n, k, 1.0, A, B, 0.0, np.zeros(m * n, np.uint16))
    assert oracle.rel_err(refc, ref64) <= oracle.HGEMM_TOL


def test_strided_batched_offsets(oracle):
    # Batch b reads A + b*stride_a etc. (crates/cublas-l3/src/batched.rs:55-58).
    m, n, k, batch = 5, 7, 3, 4
    sa, sb, sc = m * k + 2, k * n + 1, m * n + 3
    A = oracle.uniform_f32(batch * sa, 1, 1)
    B = oracle.uniform_f32(batch * sb, 1, 2)
    C = oracle.uniform_f32(batch * sc, 1, 3)
    out = oracle.sgemm_strided_batched_f64(m, n, k, 2.0, A, sa, B, sb, 0.5, C, sc, batch).reshape(batch, m, n)
    for b in range(batch):
        a = A[b * sa:b * sa + m * k].astype(np.float64).reshape(m, k)
        bb = B[b * sb:b * sb + k * n].astype(np.float64).reshape(k, n)
        c = C[b * sc:b * sc + m * n].astype(np.float64).reshape(m, n)
        np.testing.assert_allclose(out[b], 2.0 * a @ bb + 0.5 * c, rtol=1e-12, atol=1e-12)


def test_dgemv_oracle_formulas_and_compensation(oracle):
    m, n = 11, 17
    A = oracle.uniform_f64(m * n, 3, 1)
    a = A.reshape(m, n)
    xn, xt = oracle.uniform_f64(n, 3, 2), oracle.uniform_f64(m, 3, 3)
    yn, yt = oracle.uniform_f64(m, 3, 4), oracle.uniform_f64(n, 3, 5)
    np.testing.assert_allclose(oracle.dgemv_f64(0, m, n, 1.5, A, xn, 0.25, yn), 1.5 * a @ xn + 0.25 * yn,
                               rtol=1e-13, atol=1e-14)
    np.testing.assert_allclose(oracle.dgemv_f64(1, m, n, 1.5, A, xt, 0.25, yt), 1.5 * a.T @ xt + 0.25 * yt,
                               rtol=1e-13, atol=1e-14)
    # Dot2 recovers a sum that plain f64 accumulation loses entirely:
    # 1e16 + 1 - 1e16 (+ 1) = 2, where the naive left-to-right sum gives 1.
    A2 = np.array([1e16, 1.0, -1e16, 1.0])
    out = oracle.dgemv_f64(0, 1, 4, 1.0, A2, np.ones(4), 0.0, np.zeros(1))
    assert out[0] == 2.0


def test_hgemv_oracles_agree(oracle):
    # The exact f64 evaluation and the reference's own arithmetic (flushing
    # decode, f32 sums, truncating encode) agree within an f16 ulp or two on
    # normal-range data, for both shapes.
    m, n = 40, 56
    A = oracle.uniform_f16(m * n, 9, 1)
    for trans in (0, 1):
        xl, yl = (n, m) if trans == 0 else (m, n)
        x, y = oracle.uniform_f16(xl, 9, 2), oracle.uniform_f16(yl, 9, 3)
        a = A.view(np.float16).astype(np.float64).reshape(m, n)
        op = a if trans == 0 else a.T
        want = 0.75 * op @ x.view(np.float16).astype(np.float64) + 0.5 * y.view(np.float16).astype(np.float64)
        np.testing.assert_allclose(oracle.hgemv_f64(trans, m, n, 0.75, A, x, 0.5, y), want, rtol=1e-12,
                                   atol=1e-12)
        ref = oracle.hgemv_ref(trans, m, n, 0.75, A, x, 0.5, y).view(np.float16).astype(np.float64)
        assert np.max(np.abs(ref - want) / np.maximum(np.abs(want), 2.0 ** -10)) <= 2.0 ** -9


def test_sgemv_index_formulas(oracle):
    m, n = 9, 13
    A = oracle.uniform_f32(m * n, 3, 1)
    xn = oracle.uniform_f32(n, 3, 2)
    xt = oracle.uniform_f32(m, 3, 3)
    yn = oracle.uniform_f32(m, 3, 4)
    yt = oracle.uniform_f32(n, 3, 5)
    a = A.astype(np.float64).reshape(m, n)
    np.testing.assert_allclose(oracle.sgemv_f64(0, m, n, 1.5, A, xn, 0.25, yn), 1.5 * a @ xn + 0.25 * yn, rtol=1e-12)
    np.testing.assert_allclose(oracle.sgemv_f64(1, m, n, 1.5, A, xt, 0.25, yt), 1.5 * a.T @ xt + 0.25 * yt,
                               rtol=1e-12)


def test_reductions_oracle_vs_numpy(oracle):
    for n in (0, 1, 31, 32, 33, 1000, 4099):
        x = oracle.uniform_f32(n, 12, 1)
        y = oracle.uniform_f32(n, 12, 2)
        xd, yd = x.astype(np.float64), y.astype(np.float64)
        assert oracle.sdot_f64(n, x, y) == pytest.approx(float(xd @ yd), rel=1e-13, abs=1e-13)
        assert oracle.snrm2_f64(n, x) == pytest.approx(float(np.sqrt(xd @ xd)), rel=1e-13, abs=1e-13)
        assert oracle.sasum_f64(n, x) == pytest.approx(float(np.abs(xd).sum()), rel=1e-13, abs=1e-13)
        if n:
            assert oracle.isamax(n, x) == int(np.argmax(np.abs(x)))
            # a unique maximum: the reference's lane tree finds the same index
            assert oracle.isamax_ref(n, x) == oracle.isamax(n, x)
        # the reference's f32 arithmetic is within 4*n*eps(f32) * sum|x y|
        if n:
            bound = 4 * n * float(np.finfo(np.float32).eps) * float(np.abs(xd * yd).sum())
            assert abs(oracle.sreduce_ref("dot", n, x, y) - float(xd @ yd)) <= bound


def test_isamax_ties_and_nan(oracle):
    # ties: the BLAS answer is the smallest index
    x = np.zeros(64, np.float32)
    x[40] = -5.0
    x[7] = 5.0
    assert oracle.isamax(64, x) == 7
    # NaN never wins; all-NaN gives 0
    x = np.array([np.nan, 1.0, np.nan, -3.0], np.float32)
    assert oracle.isamax(4, x) == 3 and oracle.isamax_ref(4, x) == 3
    assert oracle.isamax(3, np.full(3, np.nan, np.float32)) == 0
    assert oracle.isamax_ref(3, np.full(3, np.nan, np.float32)) == 0
    # The reference's lane tree settles ties by lane slot: index 32 (lane 0)
    # and index 1 (lane 1) meet at stride 1, and slot 0 keeps its own value
    # unless the other is strictly greater, so it answers 32 where the BLAS
    # answer is 1.
    x = np.zeros(64, np.float32)
    x[32] = 2.0
    x[1] = -2.0
    assert oracle.isamax(64, x) == 1
    assert oracle.isamax_ref(64, x) == 32
