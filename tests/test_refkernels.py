"""The reference's GPU kernels restated in CUDA C (baseline/refkernels.cu).

They are a reported baseline (bench.py's "reference_kernels"), not product
code, so they are checked like the product is: against the FP64 oracle and
the oracle's restatement of the reference's own f16/f32 arithmetic on
seeded inputs.  The last tests run the library and the restated reference
kernels on the same full-size inputs and require the two results to agree
within the tolerances both are held to.
"""
import ctypes

import numpy as np
import pytest

from conftest import ROOT


def test_refkernels_library_exports_every_symbol():
    import os

    from baseline import refkernels

    path = os.path.join(ROOT, "baseline", "librefkernels.so")
    if not os.path.exists(path):
        refkernels.build()
    lib = ctypes.CDLL(path)
    for name in refkernels.SYMBOLS:
        assert hasattr(lib, name), name


def _dev(arr):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
    return t, t.data_ptr()


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [0, 1, 2, 3])
@pytest.mark.parametrize("prec", ["s", "d"])
@pytest.mark.parametrize("m,n,k", [(67, 45, 83), (128, 96, 64), (33, 200, 17)])
def test_ref_gemm_variants(oracle, variant, prec, m, n, k):
    import torch

    from baseline import refkernels as R

    if prec == "s":
        A, B, C = (oracle.uniform_f32(s, 7, i) for i, s in ((1, m * k), (2, k * n), (3, m * n)))
        fn, ref, tol = R.sgemm, oracle.sgemm_f64, oracle.tol_normwise(k, "f32")
    else:
        A, B, C = (oracle.uniform_f64(s, 7, i) for i, s in ((1, m * k), (2, k * n), (3, m * n)))
        fn, ref, tol = R.dgemm, oracle.dgemm_f64, oracle.tol_normwise(k, "f64")
    (ta, pa), (tb, pb), (tc, pc) = _dev(A), _dev(B), _dev(C)
    fn(variant, m, n, k, 1.5, pa, pb, 0.5, pc, _stream())
    torch.cuda.synchronize()
    assert oracle.rel_err(tc.cpu().numpy(), ref(m, n, k, 1.5, A, B, 0.5, C)) <= tol


def _f16_ulps(a, b):
    """Distance in f16 ulps between two arrays of finite f16 bit patterns."""
    def key(u):
        u = u.astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u)

    return np.abs(key(a) - key(b))


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(64, 48, 80), (37, 130, 29)])
def test_ref_hgemm_half_matches_reference_arithmetic(oracle, m, n, k):
    import torch

    from baseline import refkernels as R

    A = oracle.normal_f16(m * k, 9, 1, 0.0, 0.5)
    B = oracle.normal_f16(k * n, 9, 2, 0.0, 0.5)
    C = oracle.normal_f16(m * n, 9, 3, 0.0, 0.5)
    (ta, pa), (tb, pb), (tc, pc) = _dev(A.view(np.int16)), _dev(B.view(np.int16)), _dev(C.view(np.int16))
    R.hgemm_half(m, n, k, 1.25, pa, pb, 0.5, pc, _stream())
    torch.cuda.synchronize()
    got = tc.cpu().numpy().view(np.uint16)
    want = oracle.hgemm_ref(m, n, k, 1.25, A, B, 0.5, C)
    # The GPU sum contracts a*b + s into an fma, the oracle's does not: a
    # last-bit f32 difference can move the truncated f16 by one ulp.
    d = _f16_ulps(got, want)
    assert d.max() <= 1 and np.mean(d == 0) >= 0.95


@pytest.mark.gpu
def test_ref_strided_batched(oracle):
    import torch

    from baseline import refkernels as R

    batch, m, n, k = 5, 40, 36, 50
    sa, sb, sc = m * k + 8, k * n + 4, m * n + 12
    A = oracle.uniform_f32(batch * sa, 11, 1)
    B = oracle.uniform_f32(batch * sb, 11, 2)
    C = oracle.uniform_f32(batch * sc, 11, 3)
    (ta, pa), (tb, pb), (tc, pc) = _dev(A), _dev(B), _dev(C)
    R.sgemm_strided_batched(m, n, k, 1.5, pa, sa, pb, sb, 0.5, pc, sc, batch, _stream())
    torch.cuda.synchronize()
    want = oracle.sgemm_strided_batched_f64(m, n, k, 1.5, A, sa, B, sb, 0.5, C, sc, batch)
    got = tc.cpu().numpy()
    for b in range(batch):  # the oracle returns the batches packed, m*n apart
        assert oracle.rel_err(got[b * sc:b * sc + m * n], want[b * m * n:(b + 1) * m * n]) <= \
            oracle.tol_normwise(k, "f32"), b
        assert np.array_equal(got[b * sc + m * n:(b + 1) * sc], C[b * sc + m * n:(b + 1) * sc])  # gaps untouched


@pytest.mark.gpu
@pytest.mark.parametrize("trans", [0, 1])
def test_ref_gemvs(oracle, trans):
    import torch

    from baseline import refkernels as R

    m, n = 300, 77
    xl, yl = (m, n) if trans else (n, m)
    A, x, y = oracle.uniform_f32(m * n, 5, 1), oracle.uniform_f32(xl, 5, 2), oracle.uniform_f32(yl, 5, 3)
    want = oracle.sgemv_f64(trans, m, n, 1.5, A, x, 0.5, y)
    for variant in (0, 1):
        (ta, pa), (tx, px), (ty, py) = _dev(A), _dev(x), _dev(y)
        R.sgemv(variant, trans, m, n, 1.5, pa, px, 0.5, py, _stream())
        torch.cuda.synchronize()
        assert oracle.rel_err(ty.cpu().numpy(), want) <= oracle.tol_normwise(xl, "f32"), variant
    Ad, xd, yd = (v.astype(np.float64) for v in (A, x, y))
    (ta, pa), (tx, px), (ty, py) = _dev(Ad), _dev(xd), _dev(yd)
    R.dgemv(trans, m, n, 1.5, pa, px, 0.5, py, _stream())
    torch.cuda.synchronize()
    assert oracle.rel_err(ty.cpu().numpy(), oracle.dgemv_f64(trans, m, n, 1.5, Ad, xd, 0.5, yd)) <= \
        oracle.tol_normwise(xl, "f64")
    Ah = oracle.normal_f16(m * n, 5, 4, 0.0, 0.5)
    xh = oracle.normal_f16(xl, 5, 5, 0.0, 0.5)
    yh = oracle.normal_f16(yl, 5, 6, 0.0, 0.5)
    (ta, pa), (tx, px), (ty, py) = _dev(Ah.view(np.int16)), _dev(xh.view(np.int16)), _dev(yh.view(np.int16))
    R.hgemv(trans, m, n, 1.25, pa, px, 0.5, py, _stream())
    torch.cuda.synchronize()
    d = _f16_ulps(ty.cpu().numpy().view(np.uint16), oracle.hgemv_ref(trans, m, n, 1.25, Ah, xh, 0.5, yh))
    assert d.max() <= 1 and np.mean(d == 0) >= 0.95


@pytest.mark.gpu
def test_ref_level1(oracle):
    import torch

    from baseline import refkernels as R

    n = 100003
    x, y = oracle.uniform_f32(n, 3, 1), oracle.uniform_f32(n, 3, 2)
    (tx, px), (ty, py) = _dev(x), _dev(y)
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    eps = np.finfo(np.float32).eps
    for op, want in (("dot", oracle.sdot_f64(n, x, y)), ("nrm2", oracle.snrm2_f64(n, x) ** 2),
                     ("asum", oracle.sasum_f64(n, x))):
        R.sreduce(op, n, px, py, out.data_ptr(), _stream())
        torch.cuda.synchronize()
        scale = np.sum(np.abs(x.astype(np.float64) * (y if op == "dot" else x)))
        assert abs(float(out.item()) - want) <= 4 * n / 32 * eps * scale + 1e-30, op
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    R.sreduce("iamax", n, px, 0, idx.data_ptr(), _stream())
    torch.cuda.synchronize()
    assert int(idx.item()) == oracle.isamax_ref(n, x)
    R.saxpy(n, 2.5, px, py, _stream())
    torch.cuda.synchronize()
    assert np.allclose(ty.cpu().numpy(), 2.5 * x.astype(np.float64) + y, rtol=0, atol=4 * eps * 3.5)


@pytest.mark.gpu
def test_library_agrees_with_ref_kernels_sgemm_8192(oracle):
    # Same seeded inputs, the library's SGEMM and the reference's tiled
    # kernel: both are within 4*K*eps of the FP64 result, so within twice
    # that of each other.
    import torch

    import b2blas
    from baseline import refkernels as R

    m = n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(42)
    A = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
    B = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
    C0 = torch.rand(m, n, device="cuda", generator=g) * 2 - 1
    C1, C2 = C0.clone(), C0.clone()
    h = b2blas.Handle(0)
    try:
        h.set_stream(torch.cuda.current_stream().cuda_stream)
        a, b, c = (b2blas.DeviceBuffer.from_ptr(h, t.data_ptr(), t.numel(), "float32", owner=t) for t in (A, B, C1))
        h.sgemm(b2blas.GemmConfig(m, n, k, 1.5, 0.5), a, b, c)
        R.sgemm(1, m, n, k, 1.5, A.data_ptr(), B.data_ptr(), 0.5, C2.data_ptr(), _stream())
        torch.cuda.synchronize()
        d = ((C1.double() - C2.double()).norm() / C2.double().norm()).item()
        assert d <= 2 * oracle.tol_normwise(k, "f32"), d
    finally:
        h.set_stream(None)
        h.close()


@pytest.mark.gpu
def test_library_agrees_with_ref_kernels_hgemm_8192(oracle):
    # HGEMM 8192^3, N(0, 0.1) inputs: the tcgen05 kernel (round-to-nearest
    # f16 output) against the reference's hgemm_half (flushing decode,
    # truncating encode): within the 2e-2 relative bound of each other.
    import torch

    import b2blas
    from baseline import refkernels as R

    m = n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(42)
    A = (torch.randn(m, k, device="cuda", generator=g) * 0.1).half()
    B = (torch.randn(k, n, device="cuda", generator=g) * 0.1).half()
    C1 = torch.zeros(m, n, device="cuda", dtype=torch.float16)
    C2 = torch.zeros_like(C1)
    h = b2blas.Handle(0)
    try:
        h.set_stream(torch.cuda.current_stream().cuda_stream)
        a, b, c = (b2blas.DeviceBuffer.from_ptr(h, t.data_ptr(), t.numel(), np.uint16, owner=t) for t in (A, B, C1))
        h.hgemm(b2blas.GemmConfig(m, n, k, 1.0, 0.0), a, b, c)
        R.hgemm_half(m, n, k, 1.0, A.data_ptr(), B.data_ptr(), 0.0, C2.data_ptr(), _stream())
        torch.cuda.synchronize()
        d = ((C1.double() - C2.double()).norm() / C2.double().norm()).item()
        assert d <= 2e-2, d
    finally:
        h.set_stream(None)
        h.close()
