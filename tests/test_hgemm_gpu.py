"""HGEMM parity on the GPU (tcgen05 path and the generic path), through the C
ABI, against the CPU oracle.  Tolerance: 2e-2 normwise relative error
against the FP64 evaluation of the exact f16 inputs (FP16 in / FP32
accumulate); the reference's own truncating arithmetic is checked to the
same bound."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _run(handle, m, n, k, alpha, beta, A, B, C):
    import b2blas

    a, b, c = handle.upload(A), handle.upload(B), handle.upload(C)
    handle.hgemm(b2blas.GemmConfig(m, n, k, alpha, beta), a, b, c)
    handle.synchronize()
    return handle.download(c)


def test_known_answer_128(handle):
    import b2blas

    m = n = k = 128
    c = np.zeros(m * n, np.float16)
    handle.hgemm_half(b2blas.GemmConfig(m, n, k, 1.0, 0.0), np.ones(m * k, np.float16), np.ones(k * n, np.float16), c)
    assert np.max(np.abs(c.astype(np.float64) - 128.0) / 128.0) <= 5e-3
    c2 = np.zeros(m * n, np.float16)
    handle.hgemm_tensor_core(b2blas.GemmConfig(m, n, k, 1.0, 0.0), np.ones(m * k, np.float16),
                             np.ones(k * n, np.float16), c2)
    assert np.array_equal(c, c2)


# tcgen05-eligible (K, N multiples of 8) and generic-path shapes
# tcgen05-eligible (K, N multiples of 8; M <= 128 runs the single-CTA kernel,
# M > 128 the CTA-pair kernel) and generic-path shapes
SHAPES = [(128, 256, 64), (256, 512, 192), (128, 256, 8), (200, 264, 72), (1, 8, 8), (130, 300, 1000),
          (512, 512, 512), (1024, 768, 4096), (37, 41, 43), (64, 100, 7), (300, 264, 72), (257, 520, 1000),
          (384, 128, 64), (129, 8, 8), (4096, 4096, 64)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.5, -1.5)])
def test_hgemm_random_parity(handle, oracle, m, n, k, alpha, beta):
    A = oracle.normal_f16(m * k, 42, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 42, 2, 0.0, 0.1)
    C = oracle.normal_f16(m * n, 42, 3, 0.0, 0.1)
    ref = oracle.hgemm_f64(m, n, k, alpha, A, B, beta, C)
    got = _run(handle, m, n, k, alpha, beta, A, B, C)
    err = oracle.rel_err(got, ref)
    assert err <= TOL, err
    # f32 accumulation + one f16 rounding: far inside the bound in practice.
    assert err <= 2e-3, err


def test_hgemm_matches_reference_arithmetic(handle, oracle):
    # Against the reference's own scalar arithmetic (flush + truncation):
    # within the tolerance, and within 1 f16 ulp-ish everywhere.
    m, n, k = 96, 128, 256
    A = oracle.normal_f16(m * k, 3, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 3, 2, 0.0, 0.1)
    C = np.zeros(m * n, np.uint16)
    refc = oracle.hgemm_ref(m, n, k, 1.0, A, B, 0.0, C)
    got = _run(handle, m, n, k, 1.0, 0.0, A, B, C)
    ref64 = refc.view(np.float16).astype(np.float64)
    assert oracle.rel_err(got, ref64) <= TOL


def test_hgemm_8192_full_size_sampled(handle, oracle):
    # The 8192^3 configuration: rows and columns sampled against FP64.
    m = n = k = 8192
    A = oracle.normal_f16(m * k, 42, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 42, 2, 0.0, 0.1)
    got = _run(handle, m, n, k, 1.0, 0.0, A, B, np.zeros(m * n, np.uint16)).reshape(m, n)
    for r in (0, 127, 128, 4000, 8191):
        ref = oracle.hgemm_f64(m, n, k, 1.0, A, B, row0=r, nrows=1)
        assert oracle.rel_err(np.ascontiguousarray(got[r]), ref) <= TOL, r
    A32 = A.view(np.float16).astype(np.float32).reshape(m, k)
    B16 = B.view(np.float16).reshape(k, n)
    for j in (0, 255, 256, 5000, 8191):
        ref = A32.astype(np.float64) @ B16[:, j].astype(np.float64)
        assert oracle.rel_err(np.ascontiguousarray(got[:, j]), ref) <= TOL, j
    # the whole output is finite and not trivially zero
    g = got.view(np.float16)
    assert np.all(np.isfinite(g)) and np.count_nonzero(g) > 0.99 * g.size


def test_hgemm_repeatable_bitwise(handle, oracle):
    m, n, k = 384, 512, 320
    A = oracle.normal_f16(m * k, 8, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 8, 2, 0.0, 0.1)
    C = np.zeros(m * n, np.uint16)
    g1 = _run(handle, m, n, k, 1.0, 0.0, A, B, C)
    g2 = _run(handle, m, n, k, 1.0, 0.0, A, B, C)
    assert np.array_equal(g1, g2)


def test_hgemm_simple_equals_device(handle, oracle):
    import b2blas

    m, n, k = 2048, 1024, 512  # large enough for the pipelined host-slice path
    A = oracle.normal_f16(m * k, 4, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 4, 2, 0.0, 0.1)
    C = oracle.normal_f16(m * n, 4, 3, 0.0, 0.1)
    dev = _run(handle, m, n, k, 1.0, 0.5, A, B, C)
    host = C.copy()
    handle.hgemm_simple(b2blas.GemmConfig(m, n, k, 1.0, 0.5), A, B, host)
    assert np.array_equal(dev, host)


def test_pair_kernel_matches_single_cta_kernel(oracle, monkeypatch):
    # The CTA-pair kernel (M > 128) and the single-CTA kernel (forced with
    # B2B_HGEMM_SINGLE_CTA=1) agree, both within the tolerance of FP64.
    import b2blas

    m, n, k = 1024, 1280, 768
    A = oracle.normal_f16(m * k, 5, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 5, 2, 0.0, 0.1)
    C = oracle.normal_f16(m * n, 5, 3, 0.0, 0.1)
    outs = []
    for single in ("0", "1"):
        monkeypatch.setenv("B2B_HGEMM_SINGLE_CTA", single)
        h = b2blas.Handle(0)
        try:
            outs.append(_run(h, m, n, k, 1.25, 0.5, A, B, C))
        finally:
            h.close()
    ref = oracle.hgemm_f64(m, n, k, 1.25, A, B, 0.5, C)
    for o in outs:
        assert oracle.rel_err(o, ref) <= 2e-3
    diff = np.abs(outs[0].view(np.float16).astype(np.float64) - outs[1].view(np.float16).astype(np.float64))
    assert np.max(diff) <= 2 * np.max(np.abs(ref)) * 2 ** -10


VARIANT_SHAPES = [(1024, 1280, 768), (257, 520, 1000), (300, 264, 72), (256, 512, 64), (129, 1024, 136),
                  (777, 1536, 200), (2048, 2560, 1024)]


@pytest.mark.parametrize("m,n,k", VARIANT_SHAPES)
@pytest.mark.parametrize("beta", [0.0, -0.5])
def test_hgemm_kernel_variants_agree(oracle, monkeypatch, m, n, k, beta):
    # Single-CTA 128x256 (variant 1), pair 256x256 (2), pair 256x512 (3) and
    # pair 256x512 releasing its accumulator in halves (4), forced through
    # B2B_HGEMM_VARIANT, on shapes with ragged M/N/K edges (K from one k-block
    # to more than the stage ring): each within the FP64 bound, all within an
    # f16 ulp or two, and 3 and 4 bit-identical (same MMAs, same k order per
    # column).  beta == 0 takes the pair kernels' TMA-store epilogue, beta != 0
    # the read-modify-write one.
    import b2blas

    A = oracle.normal_f16(m * k, 6, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 6, 2, 0.0, 0.1)
    C = oracle.normal_f16(m * n, 6, 3, 0.0, 0.1)
    ref = oracle.hgemm_f64(m, n, k, 0.75, A, B, beta, C)
    outs = []
    for v in ("1", "2", "3", "4"):
        monkeypatch.setenv("B2B_HGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            outs.append(_run(h, m, n, k, 0.75, beta, A, B, C))
        finally:
            h.close()
    for o in outs:
        assert oracle.rel_err(o, ref) <= 2e-3
    scale = 2 * np.max(np.abs(ref)) * 2 ** -10
    for o in outs[1:]:
        d = np.abs(o.view(np.float16).astype(np.float64) - outs[0].view(np.float16).astype(np.float64))
        assert np.max(d) <= scale
    assert np.array_equal(outs[2], outs[3])


@pytest.mark.parametrize("m,n,k,beta,off", [(777, 1000, 1001, 0.0, 0), (1024, 1030, 1024, 0.5, 0),
                                            (600, 1024, 1000, -0.5, 1), (300, 1536, 2000, 0.0, 1)])
def test_hgemm_unaligned_large_takes_padded_tensor_path(oracle, monkeypatch, m, n, k, beta, off):
    # Large GEMMs whose K or N is not a multiple of 8, or whose operands are
    # not 16-byte aligned (off = 1: every pointer 2 bytes past an aligned
    # address), run on the tensor cores through zero-padded workspace; the
    # CUDA-core kernel (variant 5) is the comparison.  Both are checked
    # against the FP64 evaluation; the padded call must write C's m x n
    # elements only (the guard elements around C stay as they were).
    import b2blas

    A = oracle.normal_f16(m * k, 9, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 9, 2, 0.0, 0.1)
    C = oracle.normal_f16(m * n, 9, 3, 0.0, 0.1)
    ref = oracle.hgemm_f64(m, n, k, 0.75, A, B, beta, C)
    guard = np.full(8, np.float16(7.0)).view(np.uint16)
    outs = []
    for v in (None, "5"):
        if v is None:
            monkeypatch.delenv("B2B_HGEMM_VARIANT", raising=False)
        else:
            monkeypatch.setenv("B2B_HGEMM_VARIANT", v)
        h = b2blas.Handle(0)
        try:
            bufs = []
            for X in (A, B, C):
                host = np.concatenate([guard[:off], X, guard])
                d = h.upload(host)
                bufs.append((d, b2blas.DeviceBuffer.from_ptr(h, d.ptr + 2 * off, X.size, np.uint16)))
            (a, av), (b, bv), (c, cv) = bufs
            h.hgemm(b2blas.GemmConfig(m, n, k, 0.75, beta), av, bv, cv)
            h.synchronize()
            full = h.download(c)
            assert np.array_equal(full[:off], guard[:off]) and np.array_equal(full[off + m * n:], guard)
            outs.append(full[off:off + m * n].copy())
        finally:
            h.close()
    for o in outs:
        assert oracle.rel_err(o, ref) <= 2e-3
