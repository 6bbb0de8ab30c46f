"""SGEMM / DGEMM / strided-batched / batched parity on the GPU, through the C
ABI, against the CPU oracle.  Tolerance: normwise relative error
||C - C*||_F / ||C*||_F <= 4*K*eps(dtype) against the FP64 evaluation."""
import ctypes

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu

VARIANTS = ["naive", "tiled", "vectorized", "double_buf"]


def _cfg(m, n, k, alpha, beta):
    import b2blas

    return b2blas.GemmConfig(m, n, k, alpha, beta)


def _gemm_dev(handle, op, variant, cfg, A, B, C):
    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    getattr(handle, f"{op}_{variant}" if variant else op)(cfg, a, b, c)
    handle.synchronize()
    return handle.download(c)


# ------------------------------------------------------------ known answers

@pytest.mark.parametrize("case", [c for c in load_golden("known_answers.json")["cases"]
                                  if c["op"] in ("sgemm", "dgemm")], ids=lambda c: f"{c['op']}-{c['m']}")
def test_known_answer_all_variants(handle, case):
    dt = np.float32 if case["op"] == "sgemm" else np.float64
    m, n, k = case["m"], case["n"], case["k"]
    cfg = _cfg(m, n, k, case["alpha"], case["beta"])
    for v in case["variants"]:
        # host-slice flavour, as the reference example calls it
        c = np.zeros(m * n, dt)
        getattr(handle, f"{case['op']}_{v}_simple")(cfg, np.ones(m * k, dt), np.ones(k * n, dt), c)
        assert np.max(np.abs(c - case["expect"])) <= case["tol_abs"], v
        # device-buffer flavour, as gemm_bench calls it
        c2 = _gemm_dev(handle, case["op"], v, cfg, np.ones(m * k, dt), np.ones(k * n, dt), np.zeros(m * n, dt))
        assert np.max(np.abs(c2 - case["expect"])) <= case["tol_abs"], v


def test_known_answer_strided_and_batched(handle):
    import b2blas

    for case in load_golden("known_answers.json")["cases"]:
        if case["op"] not in ("strided_batched_sgemm", "batched_sgemm"):
            continue
        b, m, n, k = case["batch"], case["m"], case["n"], case["k"]
        cfg = b2blas.GemmConfig(m, n, k, 1.0, 0.0)
        if case["op"] == "strided_batched_sgemm":
            c = np.zeros(b * m * n, np.float32)
            handle.strided_batched_sgemm_simple(cfg, b, np.ones(b * m * k, np.float32), m * k,
                                                np.ones(b * k * n, np.float32), k * n, c, m * n)
            assert np.max(np.abs(c - case["expect"])) <= case["tol_abs"]
        else:
            cs = [np.zeros(m * n, np.float32) for _ in range(b)]
            handle.batched_sgemm(cfg, b, [np.ones(m * k, np.float32)] * b, [np.ones(k * n, np.float32)] * b, cs)
            assert max(np.max(np.abs(x - case["expect"])) for x in cs) <= case["tol_abs"]


# --------------------------------------------------------- random parity

SHAPES = [(512, 512, 512), (1, 1, 1), (15, 17, 33), (129, 257, 65), (300, 200, 100), (128, 128, 8), (64, 96, 1000),
          (1000, 8, 16), (7, 1023, 9)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, 0.5), (-0.75, 2.0)])
def test_sgemm_random_parity(handle, oracle, m, n, k, alpha, beta):
    A = oracle.uniform_f32(m * k, 42, 1)
    B = oracle.uniform_f32(k * n, 42, 2)
    C = oracle.uniform_f32(m * n, 42, 3)
    ref = oracle.sgemm_f64(m, n, k, alpha, A, B, beta, C)
    got = _gemm_dev(handle, "sgemm", None, _cfg(m, n, k, alpha, beta), A, B, C)
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(k, "f32")


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, 0.5)])
def test_dgemm_random_parity(handle, oracle, m, n, k, alpha, beta):
    A = oracle.uniform_f64(m * k, 42, 1)
    B = oracle.uniform_f64(k * n, 42, 2)
    C = oracle.uniform_f64(m * n, 42, 3)
    ref = oracle.dgemm_f64(m, n, k, alpha, A, B, beta, C)
    got = _gemm_dev(handle, "dgemm", None, _cfg(m, n, k, alpha, beta), A, B, C)
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(k, "f64")


def test_sgemm_unaligned_pointers_take_scalar_path(handle, oracle):
    # Operands that start one element past a 16-byte boundary must still be
    # correct (the vector path needs 16-byte alignment).
    import b2blas

    m, n, k = 70, 90, 50
    A = oracle.uniform_f32(m * k + 1, 5, 1)
    B = oracle.uniform_f32(k * n + 1, 5, 2)
    C = oracle.uniform_f32(m * n + 1, 5, 3)
    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    av = b2blas.DeviceBuffer.from_ptr(handle, a.ptr + 4, m * k, np.float32)
    bv = b2blas.DeviceBuffer.from_ptr(handle, b.ptr + 4, k * n, np.float32)
    cv = b2blas.DeviceBuffer.from_ptr(handle, c.ptr + 4, m * n, np.float32)
    handle.sgemm(_cfg(m, n, k, 1.25, -0.5), av, bv, cv)
    handle.synchronize()
    got = handle.download(c)[1:]
    ref = oracle.sgemm_f64(m, n, k, 1.25, A[1:], B[1:], -0.5, C[1:])
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(k, "f32")


def test_beta_zero_does_not_read_c(handle, oracle):
    # beta == 0: C is write-only, so NaN in C does not propagate.
    m, n, k = 64, 64, 64
    A = oracle.uniform_f32(m * k, 1, 1)
    B = oracle.uniform_f32(k * n, 1, 2)
    C = np.full(m * n, np.nan, np.float32)
    got = _gemm_dev(handle, "sgemm", None, _cfg(m, n, k, 1.0, 0.0), A, B, C)
    assert np.all(np.isfinite(got))


def test_zero_dims_leave_c_untouched(handle):
    c = handle.upload(np.full(16, 7.0, np.float32))
    z = handle.upload(np.zeros(16, np.float32))
    handle.sgemm(_cfg(4, 4, 0, 1.0, 0.0), z, z, c)
    handle.synchronize()
    assert np.all(handle.download(c) == 7.0)


def test_simple_equals_device_flavour_bitwise(handle, oracle):
    m, n, k = 200, 160, 96
    A = oracle.uniform_f32(m * k, 9, 1)
    B = oracle.uniform_f32(k * n, 9, 2)
    C = oracle.uniform_f32(m * n, 9, 3)
    cfg = _cfg(m, n, k, 1.5, 0.5)
    dev = _gemm_dev(handle, "sgemm", None, cfg, A, B, C)
    host = C.copy()
    handle.sgemm_simple(cfg, A, B, host)
    assert np.array_equal(dev, host)


@pytest.mark.parametrize("col_panels", ["1", "2", "3"])
@pytest.mark.parametrize("prec", ["s", "d", "h"])
def test_large_simple_tiled_pipeline(oracle, monkeypatch, col_panels, prec):
    # Host slices above 64 MiB take the pipelined path: row panels of A times
    # column panels of B, gathered and scattered with 2-D copies.  Ragged
    # sizes leave short last panels in both directions; beta != 0 uploads C
    # tiles too.  The result equals the device-buffer flavour bit for bit
    # (same kernel per output element), and is checked against FP64 rows.
    import b2blas

    monkeypatch.setenv("B2B_HOST_COL_PANELS", col_panels)
    m, n, k = 3000, 2600, 3000  # f32: 98 MB of operands
    if prec == "d":
        m, n, k = 2100, 1800, 2100
    if prec == "h":
        m, n, k = 4100, 4104, 4096
    h = b2blas.Handle(0)
    try:
        if prec == "h":
            A = oracle.normal_f16(m * k, 11, 1, 0.0, 0.1)
            B = oracle.normal_f16(k * n, 11, 2, 0.0, 0.1)
            C = oracle.normal_f16(m * n, 11, 3, 0.0, 0.1)
        else:
            f = oracle.uniform_f32 if prec == "s" else oracle.uniform_f64
            A, B, C = f(m * k, 11, 1), f(k * n, 11, 2), f(m * n, 11, 3)
        cfg = b2blas.GemmConfig(m, n, k, 1.25, -0.5)
        host = C.copy()
        getattr(h, f"{prec}gemm_simple")(cfg, A, B, host)
        a, b, c = h.upload(A), h.upload(B), h.upload(C)
        getattr(h, f"{prec}gemm")(cfg, a, b, c)
        h.synchronize()
        dev = h.download(c)
        ref_fn = {"s": oracle.sgemm_f64, "d": oracle.dgemm_f64, "h": oracle.hgemm_f64}[prec]
        rows = [0, 383, 384, m - 1]
        for r in rows:
            ref = ref_fn(m, n, k, 1.25, A, B, -0.5, C, row0=r, nrows=1)
            got = np.ascontiguousarray(host.reshape(m, n)[r])
            tol = 2e-2 if prec == "h" else oracle.tol_normwise(k, "f32" if prec == "s" else "f64")
            assert oracle.rel_err(got, ref) <= tol, r
        if prec != "h":
            assert np.array_equal(dev, host)
        else:  # tile shapes may pick another tcgen05 variant: within an f16 ulp
            d = np.abs(dev.view(np.float16).astype(np.float64) - host.view(np.float16).astype(np.float64))
            assert np.max(d) <= 2 * np.max(np.abs(host.view(np.float16).astype(np.float64))) * 2 ** -10
    finally:
        h.close()


def test_sgemm_8192_full_size_sampled(handle, oracle):
    # The 8192^3 configuration (alpha 1.5, beta 0.5): sampled rows against the
    # FP64 oracle, plus a column check C[:, j] against A @ B[:, j].
    import b2blas

    m = n = k = 8192
    A = oracle.uniform_f32(m * k, 42, 1)
    B = oracle.uniform_f32(k * n, 42, 2)
    C = oracle.uniform_f32(m * n, 42, 3)
    got = _gemm_dev(handle, "sgemm", None, b2blas.GemmConfig(m, n, k, 1.5, 0.5), A, B, C).reshape(m, n)
    tol = oracle.tol_normwise(k, "f32")
    for r in (0, 1, 4095, 8191):
        ref = oracle.sgemm_f64(m, n, k, 1.5, A, B, 0.5, C, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= tol, r
    A2 = A.reshape(m, k).astype(np.float64)
    for j in (0, 777, 8191):
        ref = 1.5 * (A2 @ B.reshape(k, n)[:, j].astype(np.float64)) + 0.5 * C.reshape(m, n)[:, j]
        assert oracle.rel_err(np.ascontiguousarray(got[:, j]), ref) <= tol, j


def test_dgemm_4096_full_size_sampled(handle, oracle):
    import b2blas

    m = n = k = 4096
    A = oracle.uniform_f64(m * k, 42, 1)
    B = oracle.uniform_f64(k * n, 42, 2)
    C = oracle.uniform_f64(m * n, 42, 3)
    got = _gemm_dev(handle, "dgemm", None, b2blas.GemmConfig(m, n, k, 1.5, 0.5), A, B, C).reshape(m, n)
    for r in (0, 2049, 4095):
        ref = oracle.dgemm_f64(m, n, k, 1.5, A, B, 0.5, C, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= oracle.tol_normwise(k, "f64"), r


@pytest.mark.parametrize("m,n,k,beta", [(1000, 1002, 998, 0.5), (2176, 2048, 512, 0.0), (130, 4096, 64, 0.5)])
def test_dgemm_persistent_kernel_bit_identical(monkeypatch, oracle, m, n, k, beta):
    # The persistent warp-specialised DMMA kernel (the default) against the
    # one-CTA-per-tile kernel (variant 8): same per-element arithmetic, so the
    # same bits.  2176 x 2048 is 272 tiles, so CTAs take two tiles each and the
    # producer streams across a tile boundary; ragged edges in M, N and K.
    import b2blas

    A = oracle.uniform_f64(m * k, 31, 1)
    B = oracle.uniform_f64(k * n, 31, 2)
    C = oracle.uniform_f64(m * n, 31, 3)
    monkeypatch.setenv("B2B_DGEMM_KSPLIT", "1")  # the one-CTA-per-tile kernel does not split
    cfg = b2blas.GemmConfig(m, n, k, 1.5, beta)
    outs = {}
    for v in ("0", "8"):
        monkeypatch.setenv("B2B_DGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            outs[v] = _gemm_dev(h, "dgemm", None, cfg, A, B, C)
        finally:
            h.close()
    assert np.array_equal(outs["0"], outs["8"])
    got = outs["0"].reshape(m, n)
    for r in (0, m // 2 + 1, m - 1):
        ref = oracle.dgemm_f64(m, n, k, 1.5, A, B, beta, C, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= oracle.tol_normwise(k, "f64"), r


@pytest.mark.parametrize("m,n,k,ks,beta", [(1024, 1024, 1024, None, 0.5), (2048, 2048, 2048, "4", 0.0),
                                            (1000, 1002, 998, "3", 0.5), (130, 4096, 4096, "8", -1.0)])
def test_dgemm_split_k(oracle, monkeypatch, m, n, k, ks, beta):
    # Split-K on the persistent DMMA kernel (chosen for 1024^3: 64 tiles under
    # one wave, S = 2; forced for the others, including K whose last range is
    # short): raw sums per k range in workspace, then a fixed-order reduce
    # applying alpha and beta.  Within the FP64 bound of the FP64 evaluation,
    # and the same bits on a second call.
    import b2blas

    if ks is None:
        monkeypatch.delenv("B2B_DGEMM_KSPLIT", raising=False)
    else:
        monkeypatch.setenv("B2B_DGEMM_KSPLIT", ks)
    A = oracle.uniform_f64(m * k, 33, 1)
    B = oracle.uniform_f64(k * n, 33, 2)
    C = oracle.uniform_f64(m * n, 33, 3)
    h = b2blas.Handle(0)
    try:
        cfg = b2blas.GemmConfig(m, n, k, 1.5, beta)
        a, b = h.upload(A), h.upload(B)
        outs = []
        for _ in range(2):
            c = h.upload(C)
            h.dgemm(cfg, a, b, c)
            h.synchronize()
            outs.append(h.download(c))
        assert np.array_equal(outs[0], outs[1])
        got = outs[0].reshape(m, n)
        for r in (0, m // 2 + 1, m - 1):
            ref = oracle.dgemm_f64(m, n, k, 1.5, A, B, beta, C, row0=r, nrows=1)
            assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= oracle.tol_normwise(k, "f64"), r
    finally:
        h.close()


def test_dgemm_split_k_simple_matches_device_bits(oracle):
    # 1024 x 1024 x 8192 splits in two (64 tiles, under one wave).  Its
    # 64 MiB operands make the host-slice call pipelined and tiled; the call
    # forces the whole GEMM's split on every tile, so every output sums the
    # same k ranges in the same order: the device call's bits.
    import b2blas

    m, n, k = 1024, 1024, 8192
    A = oracle.uniform_f64(m * k, 34, 1)
    B = oracle.uniform_f64(k * n, 34, 2)
    C = oracle.uniform_f64(m * n, 34, 3)
    h = b2blas.Handle(0)
    try:
        cfg = b2blas.GemmConfig(m, n, k, 1.25, -0.5)
        host = C.copy()
        h.dgemm_simple(cfg, A, B, host)
        a, b, c = h.upload(A), h.upload(B), h.upload(C)
        h.dgemm(cfg, a, b, c)
        h.synchronize()
        dev = h.download(c)
        assert np.array_equal(dev, host)
        for r in (0, 513, m - 1):
            ref = oracle.dgemm_f64(m, n, k, 1.25, A, B, -0.5, C, row0=r, nrows=1)
            assert oracle.rel_err(np.ascontiguousarray(host.reshape(m, n)[r]), ref) <= oracle.tol_normwise(k, "f64")
    finally:
        h.close()


# ------------------------------------------------------- batched family

@pytest.mark.parametrize("batch,m,n,k,gap", [(8, 64, 64, 64, 0), (33, 17, 29, 13, 3), (4, 256, 256, 256, 0),
                                             (70000, 2, 3, 4, 1)])
def test_strided_batched_parity(handle, oracle, batch, m, n, k, gap):
    import b2blas

    sa, sb, sc = m * k + gap, k * n + 2 * gap, m * n + gap
    A = oracle.uniform_f32(batch * sa, 11, 1)
    B = oracle.uniform_f32(batch * sb, 11, 2)
    C = oracle.uniform_f32(batch * sc, 11, 3)
    cfg = b2blas.GemmConfig(m, n, k, 0.75, 0.25)
    ref = oracle.sgemm_strided_batched_f64(m, n, k, 0.75, A, sa, B, sb, 0.25, C, sc, batch)
    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    handle.strided_batched_sgemm(cfg, batch, a, sa, b, sb, c, sc)
    handle.synchronize()
    got = handle.download(c)
    gotp = np.concatenate([got[i * sc:i * sc + m * n] for i in range(batch)]) if gap else got
    assert oracle.rel_err(gotp, ref) <= oracle.tol_normwise(k, "f32")
    if gap:  # elements between batches are untouched
        for i in range(min(batch, 50)):
            assert np.array_equal(got[i * sc + m * n:(i + 1) * sc], C[i * sc + m * n:(i + 1) * sc])
    # the host-slice flavour gives the same bits
    host = C.copy()
    handle.strided_batched_sgemm_simple(cfg, batch, A, sa, B, sb, host, sc)
    assert np.array_equal(host, got)


def test_strided_batched_4096x256_sampled(handle, oracle):
    import b2blas

    batch, m = 4096, 256
    A = oracle.uniform_f32(batch * m * m, 42, 1)
    B = oracle.uniform_f32(batch * m * m, 42, 2)
    a, b = handle.upload(A), handle.upload(B)
    c = handle.zeroed(batch * m * m)
    handle.strided_batched_sgemm(b2blas.GemmConfig(m, m, m, 1.0, 0.0), batch, a, m * m, b, m * m, c, m * m)
    handle.synchronize()
    got = handle.download(c)
    for bi in (0, 1, 2047, 4095):
        s = bi * m * m
        ref = oracle.sgemm_f64(m, m, m, 1.0, A[s:s + m * m], B[s:s + m * m])
        assert oracle.rel_err(got[s:s + m * m], ref) <= oracle.tol_normwise(m, "f32"), bi


def test_batched_sgemm_list_api(handle, oracle):
    import b2blas

    batch, m, n, k = 5, 31, 40, 23
    As = [oracle.uniform_f32(m * k, 20 + i, 1) for i in range(batch)]
    Bs = [oracle.uniform_f32(k * n, 20 + i, 2) for i in range(batch)]
    Cs = [oracle.uniform_f32(m * n, 20 + i, 3) for i in range(batch)]
    refs = [oracle.sgemm_f64(m, n, k, 2.0, As[i], Bs[i], -1.0, Cs[i]) for i in range(batch)]
    outs = [c.copy() for c in Cs]
    handle.batched_sgemm(b2blas.GemmConfig(m, n, k, 2.0, -1.0), batch, As, Bs, outs)
    for o, r in zip(outs, refs):
        assert oracle.rel_err(o, r) <= oracle.tol_normwise(k, "f32")


# ------------------------------------------------- opt-in 3xTF32 SGEMM

@pytest.mark.parametrize("m,n,k", [(256, 256, 32), (512, 512, 512), (300, 264, 72), (1, 4, 4), (129, 260, 1000),
                                   (1024, 768, 4096), (15, 17, 33)])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.5, 0.5)])
def test_sgemm_3xtf32_parity(handle, oracle, m, n, k, alpha, beta):
    # Same FP32 bound as the FFMA kernel: ||C - C*|| / ||C*|| <= 4*K*eps(f32).
    A = oracle.uniform_f32(m * k, 43, 1)
    B = oracle.uniform_f32(k * n, 43, 2)
    C = oracle.uniform_f32(m * n, 43, 3)
    ref = oracle.sgemm_f64(m, n, k, alpha, A, B, beta, C)
    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    handle.sgemm_3xtf32(_cfg(m, n, k, alpha, beta), a, b, c)
    handle.synchronize()
    got = handle.download(c)
    err = oracle.rel_err(got, ref)
    assert err <= oracle.tol_normwise(k, "f32"), err
    # Far tighter than a plain TF32 GEMM (~1e-3 at K=4096): the three-term
    # split leaves the tensor core's f32 accumulation as the main error
    # (measured ~3e-5 at K=4096; the FFMA kernel is ~1e-6).
    assert err <= 1e-4, err


def test_sgemm_3xtf32_8192_sampled(handle, oracle):
    import b2blas

    m = n = k = 8192
    A = oracle.uniform_f32(m * k, 42, 1)
    B = oracle.uniform_f32(k * n, 42, 2)
    C = oracle.uniform_f32(m * n, 42, 3)
    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    handle.sgemm_3xtf32(b2blas.GemmConfig(m, n, k, 1.5, 0.5), a, b, c)
    handle.synchronize()
    got = handle.download(c).reshape(m, n)
    for r in (0, 255, 256, 8191):
        ref = oracle.sgemm_f64(m, n, k, 1.5, A, B, 0.5, C, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= oracle.tol_normwise(k, "f32"), r


# -------------------------------------------- fused bias + ReLU epilogue

@pytest.mark.parametrize("algo", [0, 5])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 200, 100), (4096, 1024, 1024), (15, 17, 33), (130, 264, 72)])
@pytest.mark.parametrize("relu", [False, True])
def test_sgemm_bias_relu(handle, oracle, algo, m, n, k, relu):
    # C = act(alpha*A*B + beta*C + bias[col]), the mlp layer in one kernel;
    # same FP32 bound as SGEMM.
    import b2blas

    A = oracle.uniform_f32(m * k, 61, 1)
    B = oracle.uniform_f32(k * n, 61, 2)
    C = oracle.uniform_f32(m * n, 61, 3)
    bias = oracle.normal_f32(n, 61, 5, 0.0, 0.5)
    ref = oracle.sgemm_f64(m, n, k, 1.25, A, B, 0.5, C).reshape(m, n) + bias.astype(np.float64)[None, :]
    if relu:
        ref = np.maximum(ref, 0.0)
    a, b, c, bd = handle.upload(A), handle.upload(B), handle.upload(C), handle.upload(bias)
    handle.sgemm_bias(_cfg(m, n, k, 1.25, 0.5), a, b, c, bd, relu=relu, algo=b2blas.Algo(algo))
    handle.synchronize()
    got = handle.download(c)
    assert oracle.rel_err(got, ref.ravel()) <= oracle.tol_normwise(k, "f32")
    if relu:
        assert np.all(got >= 0.0)


def test_sgemm_bias_equals_sgemm_plus_saxpy(handle, oracle):
    # The fused layer matches the reference's two-call pattern
    # (examples/mlp/src/main.rs:130-144): sgemm then saxpy of the
    # pre-broadcast bias.
    import b2blas

    m, n, k = 256, 512, 128
    A = oracle.uniform_f32(m * k, 3, 1)
    B = oracle.uniform_f32(k * n, 3, 2)
    bias = oracle.normal_f32(n, 3, 5, 0.0, 0.01)
    cfg = b2blas.GemmConfig(m, n, k, 1.0, 0.0)
    a, b, bd = handle.upload(A), handle.upload(B), handle.upload(bias)
    c1, c2 = handle.zeroed(m * n), handle.zeroed(m * n)
    handle.sgemm_tiled(cfg, a, b, c1)
    handle.saxpy(m * n, 1.0, handle.upload(np.tile(bias, m)), c1)
    handle.sgemm_bias(cfg, a, b, c2, bd)
    handle.synchronize()
    np.testing.assert_allclose(handle.download(c2), handle.download(c1), rtol=0, atol=1e-5)


# ------------------------------------------- FFMA kernel forms, same bits

@pytest.mark.parametrize("m,n,k,alpha,beta", [(1000, 1028, 1000, 1.5, 0.5), (300, 1024, 96, 1.0, 0.0),
                                              (256, 2048, 64, 0.75, 0.25)])
def test_sgemm_ffma_kernels_bit_identical(monkeypatch, oracle, m, n, k, alpha, beta):
    # Every FP32 FFMA kernel sums each output over k in order with one fma per
    # step, so the forms must agree bit for bit: the cp.async kernel (variant
    # 11), the TMA-fed kernel on a transposed A with scalar FFMA (20), FFMA2
    # on row pairs (21), FFMA2 on column pairs (22), and the persistent
    # TMA-fed kernel on row-major A (23, which the default 0 takes for these
    # shapes).  Split-K is off here (it sums k ranges separately, so a split
    # call has other bits by design).
    import b2blas

    monkeypatch.setenv("B2B_SGEMM_KSPLIT", "1")
    A = oracle.uniform_f32(m * k, 21, 1)
    B = oracle.uniform_f32(k * n, 21, 2)
    C = oracle.uniform_f32(m * n, 21, 3)
    cfg = b2blas.GemmConfig(m, n, k, alpha, beta)
    outs = {}
    for v in ("0", "11", "20", "21", "22", "23"):
        monkeypatch.setenv("B2B_SGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            outs[v] = _gemm_dev(h, "sgemm", None, cfg, A, B, C)
        finally:
            h.close()
    ref = oracle.sgemm_f64(m, n, k, alpha, A, B, beta, C)
    assert oracle.rel_err(outs["11"], ref) <= oracle.tol_normwise(k, "f32")
    for v in ("0", "20", "21", "22", "23"):
        assert np.array_equal(outs[v], outs["11"]), v


@pytest.mark.parametrize("splits", [2, 3])
@pytest.mark.parametrize("m,n,k,beta", [(1000, 1028, 1000, 0.5), (2048, 1024, 4096, 0.0)])
def test_sgemm_split_k_persistent_matches_transposed_a_kernel(monkeypatch, oracle, splits, m, n, k, beta):
    # A split GEMM on the persistent row-major-A kernel (the default) and on
    # the transposed-A kernel (variant 21) sums the same k ranges in the same
    # order and adds the partials in split order: the same bits, with and
    # without the fused bias + ReLU epilogue.
    import b2blas

    monkeypatch.setenv("B2B_SGEMM_KSPLIT", str(splits))
    A = oracle.uniform_f32(m * k, 23, 1)
    B = oracle.uniform_f32(k * n, 23, 2)
    C = oracle.uniform_f32(m * n, 23, 3)
    bias = oracle.uniform_f32(n, 23, 5)
    cfg = b2blas.GemmConfig(m, n, k, 1.5, beta)
    outs = {}
    for v in ("0", "21"):
        monkeypatch.setenv("B2B_SGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            outs[v] = _gemm_dev(h, "sgemm", None, cfg, A, B, C)
            a, b, c, bb = h.upload(A), h.upload(B), h.upload(C), h.upload(bias)
            h.sgemm_bias(cfg, a, b, c, bb, relu=True)
            h.synchronize()
            outs[v + "b"] = h.download(c)
        finally:
            h.close()
    assert np.array_equal(outs["0"], outs["21"])
    assert np.array_equal(outs["0b"], outs["21b"])
    got = outs["0"].reshape(m, n)
    for r in (0, m // 2 + 3, m - 1):
        ref = oracle.sgemm_f64(m, n, k, 1.5, A, B, beta, C, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= oracle.tol_normwise(k, "f32"), r


@pytest.mark.parametrize("batch", [12, 300])
def test_strided_batched_tma_kernel_bit_identical(monkeypatch, oracle, batch):
    # The batched default (TMA-fed on row-major A, 3-D tensor maps) against
    # the cp.async kernel (variant 11) and the TMA kernel's 128 x 256 and
    # 128 x 128 (two CTAs per SM) forms (variants 24, 25) and the form that
    # transposes A in shared memory (26), and its persistent warp-specialised
    # forms (27: the FFMA warps transpose A; 28 and the default: the producer
    # warpgroup does; 300 batches give each CTA several tiles), with gaps between batches and
    # ragged M/N edges.
    import b2blas

    m, n, k = 200, 136, 100
    sa, sb, sc = m * k + 4, k * n + 8, m * n + 12
    A = oracle.uniform_f32(batch * sa, 22, 1)
    B = oracle.uniform_f32(batch * sb, 22, 2)
    C = oracle.uniform_f32(batch * sc, 22, 3)
    cfg = b2blas.GemmConfig(m, n, k, 1.5, 0.5)
    outs = {}
    for v in ("0", "11", "24", "25", "26", "27", "28"):
        monkeypatch.setenv("B2B_SGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            a, b, c = h.upload(A), h.upload(B), h.upload(C)
            h.strided_batched_sgemm(cfg, batch, a, sa, b, sb, c, sc)
            h.synchronize()
            outs[v] = h.download(c)
        finally:
            h.close()
    assert np.array_equal(outs["0"], outs["11"])
    assert np.array_equal(outs["0"], outs["24"])
    assert np.array_equal(outs["0"], outs["25"])
    assert np.array_equal(outs["0"], outs["26"])
    assert np.array_equal(outs["0"], outs["27"])
    assert np.array_equal(outs["0"], outs["28"])
    ref = oracle.sgemm_strided_batched_f64(m, n, k, 1.5, A, sa, B, sb, 0.5, C, sc, batch)
    got = np.concatenate([outs["0"][i * sc:i * sc + m * n] for i in range(batch)])
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(k, "f32")
    for i in range(batch):
        assert np.array_equal(outs["0"][i * sc + m * n:(i + 1) * sc], C[i * sc + m * n:(i + 1) * sc])


@pytest.mark.parametrize("gap,beta", [(0, 0.0), (0, 0.5), (3, 0.0), (3, 0.5)])
def test_strided_batched_simple_pipelined(monkeypatch, oracle, gap, beta):
    # Large host-slice calls run in chunks of batches over three streams
    # (upload / compute / download); both copy schedules must give the bits
    # of the device-buffer call, leave the gaps between batches untouched
    # and not write past the last batch.
    import b2blas

    batch, m, n, k = 1000, 128, 128, 128  # 197 MB of operands: pipelined
    sa, sb, sc = m * k + 4 * gap, k * n + 8 * gap, m * n + 4 * gap
    A = oracle.uniform_f32(batch * sa, 23, 1)
    B = oracle.uniform_f32(batch * sb, 23, 2)
    C = oracle.uniform_f32(batch * sc + 5, 23, 3)  # 5 elements past the last batch's stride
    cfg = b2blas.GemmConfig(m, n, k, 1.25, beta)
    h = b2blas.Handle(0)
    try:
        a, b, c = h.upload(A), h.upload(B), h.upload(C)
        h.strided_batched_sgemm(cfg, batch, a, sa, b, sb, c, sc)
        h.synchronize()
        want = h.download(c)
    finally:
        h.close()
    for mode in ("0", "1"):
        monkeypatch.setenv("B2B_COPY_MODE", mode)
        h = b2blas.Handle(0)
        try:
            host = C.copy()
            h.strided_batched_sgemm_simple(cfg, batch, A, sa, B, sb, host, sc)
        finally:
            h.close()
        assert np.array_equal(host, want), mode
        assert np.array_equal(host[batch * sc:], C[batch * sc:])
    ref = oracle.sgemm_strided_batched_f64(m, n, k, 1.25, A[:3 * sa], sa, B[:3 * sb], sb, beta, C[:3 * sc], sc, 3)
    got = np.concatenate([want[i * sc:i * sc + m * n] for i in range(3)])
    assert oracle.rel_err(got, ref) <= oracle.tol_normwise(k, "f32")


def test_strided_batched_simple_pipelined_shared_a(monkeypatch, oracle):
    # stride_a = 0: one A for every batch (the slice holds a single m x k
    # matrix).  The pipelined host-slice call uploads it once and must give
    # the device-buffer call's bits in both copy schedules.
    import b2blas

    batch, m, n, k = 1000, 128, 128, 128
    A = oracle.uniform_f32(m * k, 24, 1)
    B = oracle.uniform_f32(batch * k * n, 24, 2)
    C = oracle.uniform_f32(batch * m * n, 24, 3)
    cfg = b2blas.GemmConfig(m, n, k, 1.0, 0.5)
    h = b2blas.Handle(0)
    try:
        a, b, c = h.upload(A), h.upload(B), h.upload(C)
        h.strided_batched_sgemm(cfg, batch, a, 0, b, k * n, c, m * n)
        h.synchronize()
        want = h.download(c)
    finally:
        h.close()
    for mode in ("0", "1"):
        monkeypatch.setenv("B2B_COPY_MODE", mode)
        h = b2blas.Handle(0)
        try:
            host = C.copy()
            h.strided_batched_sgemm_simple(cfg, batch, A, 0, B, k * n, host, m * n)
        finally:
            h.close()
        assert np.array_equal(host, want), mode
    ref = oracle.sgemm_strided_batched_f64(m, n, k, 1.0, A, 0, B[:2 * k * n], k * n, 0.5, C[:2 * m * n], m * n, 2)
    assert oracle.rel_err(want[:2 * m * n], ref) <= oracle.tol_normwise(k, "f32")


@pytest.mark.parametrize("m,n,k,ks", [(1024, 1024, 1024, None), (1000, 1024, 1000, "3"), (4096, 1028, 512, "2"),
                                      (256, 2048, 4096, "8"), (128, 1024, 300, "2")])
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_sgemm_split_k(oracle, monkeypatch, m, n, k, ks, beta):
    # Split-K on the TMA-fed SGEMM (chosen for 1024^3: 32 tiles under one
    # wave; forced through B2B_SGEMM_KSPLIT for the others, including a K
    # whose last range is short): raw sums per k range in workspace, then a
    # fixed-order reduce applying alpha, beta, bias and ReLU.  Within the
    # FP32 bound of the FP64 evaluation; the same bits on a second call; the
    # bias + ReLU epilogue equals sgemm followed by the bias and ReLU on the
    # host (both round alpha*sum + beta*c the same way before adding bias).
    import b2blas

    if ks is None:
        monkeypatch.delenv("B2B_SGEMM_KSPLIT", raising=False)
    else:
        monkeypatch.setenv("B2B_SGEMM_KSPLIT", ks)
    A = oracle.uniform_f32(m * k, 31, 1)
    B = oracle.uniform_f32(k * n, 31, 2)
    C = oracle.uniform_f32(m * n, 31, 3)
    bias = oracle.uniform_f32(n, 31, 5)
    h = b2blas.Handle(0)
    try:
        cfg = b2blas.GemmConfig(m, n, k, 1.5, beta)
        a, b = h.upload(A), h.upload(B)
        outs = []
        for _ in range(2):
            c = h.upload(C)
            h.sgemm(cfg, a, b, c)
            h.synchronize()
            outs.append(h.download(c))
        assert np.array_equal(outs[0], outs[1])
        ref = oracle.sgemm_f64(m, n, k, 1.5, A, B, beta, C)
        assert oracle.rel_err(outs[0], ref) <= oracle.tol_normwise(k, "f32")
        c, bd = h.upload(C), h.upload(bias)
        h.sgemm_bias(cfg, a, b, c, bias=bd, relu=True)
        h.synchronize()
        fused = h.download(c)
        expect = np.maximum(outs[0].reshape(m, n) + bias[None, :], np.float32(0)).ravel()
        assert np.array_equal(fused, expect.astype(np.float32))
    finally:
        h.close()


def test_sgemm_split_k_simple_matches_device_bits(oracle):
    # 4096^3 splits in two (512 tiles are 3.46 waves on 148 SMs).  The
    # pipelined host-slice call computes 512 x 2048 tiles, each far under a
    # wave; it forces the whole GEMM's split on every tile, so every output
    # sums the same k ranges in the same order: the device call's bits.
    import b2blas

    m = n = k = 4096
    A = oracle.uniform_f32(m * k, 32, 1)
    B = oracle.uniform_f32(k * n, 32, 2)
    C = oracle.uniform_f32(m * n, 32, 3)
    h = b2blas.Handle(0)
    try:
        cfg = b2blas.GemmConfig(m, n, k, 1.25, -0.5)
        host = C.copy()
        h.sgemm_simple(cfg, A, B, host)
        a, b, c = h.upload(A), h.upload(B), h.upload(C)
        h.sgemm(cfg, a, b, c)
        h.synchronize()
        dev = h.download(c)
        assert np.array_equal(dev, host)
        for r in (0, 2049, m - 1):
            ref = oracle.sgemm_f64(m, n, k, 1.25, A, B, -0.5, C, row0=r, nrows=1)
            assert oracle.rel_err(np.ascontiguousarray(host.reshape(m, n)[r]), ref) <= oracle.tol_normwise(k, "f32")
    finally:
        h.close()


def test_sgemm_splits_query_and_row_pieces_reproduce_whole(oracle):
    # b2b_sgemm_splits reports the split the device call takes; fixing the
    # whole GEMM's split with b2b_set_sgemm_splits makes two row halves,
    # computed as separate calls, reproduce the whole call's bits (without
    # it each half, a different shape, may split differently).
    import b2blas

    h = b2blas.Handle(0)
    try:
        assert h.sgemm_splits(1024, 1024, 1024) == 4
        assert h.sgemm_splits(8192, 8192, 8192) == 1
        assert h.sgemm_splits(512, 512, 512) == 2  # 8 tiles on the persistent kernel
        assert h.sgemm_splits(512, 514, 512) == 1  # N % 4 != 0: the cp.async kernel, no split
        m, n, k = 4096, 1024, 4096
        whole = h.sgemm_splits(m, n, k)
        A = oracle.uniform_f32(m * k, 33, 1)
        B = oracle.uniform_f32(k * n, 33, 2)
        a, b, c = h.upload(A), h.upload(B), h.upload(np.zeros(m * n, np.float32))
        h.sgemm(b2blas.GemmConfig(m, n, k, 1.0, 0.0), a, b, c)
        h.synchronize()
        ref = h.download(c)
        half = m // 2
        assert h.sgemm_splits(half, n, k) != whole  # the halves alone would split otherwise
        h.set_sgemm_splits(whole)
        assert h.sgemm_splits(half, n, k) == whole
        outs = []
        for r0 in (0, half):
            ah = b2blas.DeviceBuffer.from_ptr(h, a.ptr + 4 * r0 * k, half * k, np.float32)
            ch = h.upload(np.zeros(half * n, np.float32))
            h.sgemm(b2blas.GemmConfig(half, n, k, 1.0, 0.0), ah, b, ch)
            h.synchronize()
            outs.append(h.download(ch))
        h.set_sgemm_splits(0)
        assert np.array_equal(np.concatenate(outs), ref)
        with pytest.raises(b2blas.CublasError):
            h.set_sgemm_splits(-1)
    finally:
        h.close()


def test_sgemm_split_k_beta_zero_does_not_read_c(oracle):
    # The split-K reduce keeps the rule that beta == 0 leaves C unread: NaN in
    # C does not reach the result, which equals the call on a zeroed C.
    import b2blas

    m = n = k = 1024  # 32 tiles: split in 4
    A = oracle.uniform_f32(m * k, 34, 1)
    B = oracle.uniform_f32(k * n, 34, 2)
    h = b2blas.Handle(0)
    try:
        assert h.sgemm_splits(m, n, k) > 1
        cfg = b2blas.GemmConfig(m, n, k, 0.5, 0.0)
        got = _gemm_dev(h, "sgemm", None, cfg, A, B, np.full(m * n, np.nan, np.float32))
        ref = _gemm_dev(h, "sgemm", None, cfg, A, B, np.zeros(m * n, np.float32))
        assert np.all(np.isfinite(got)) and np.array_equal(got, ref)
    finally:
        h.close()
