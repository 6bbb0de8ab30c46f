"""Error behaviour on the GPU: the reference's panics on host-slice length
mismatches become DimensionMismatch errors; bad arguments are
InvalidArgument; a bounded device wait that gives up is reported on the host
and leaves the handle usable (no fault, no hang)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_simple_length_mismatch_is_dimension_error(handle):
    import b2blas

    cfg = b2blas.GemmConfig(4, 4, 4, 1.0, 0.0)
    z16, z15 = np.zeros(16, np.float32), np.zeros(15, np.float32)
    for bad in ((z15, z16, z16), (z16, z15, z16), (z16, z16, z15)):
        with pytest.raises(b2blas.CublasError) as ei:
            handle.sgemm_tiled_simple(cfg, *[x.copy() for x in bad])
        assert ei.value.kind == "DimensionMismatch"
    # length checks come before the empty-dimension early return
    with pytest.raises(b2blas.CublasError):
        handle.sgemm_simple(b2blas.GemmConfig(4, 4, 0, 1.0, 0.0), np.zeros(1, np.float32), np.zeros(0, np.float32),
                            np.zeros(16, np.float32))


def test_strided_simple_too_short_is_dimension_error(handle):
    import b2blas

    cfg = b2blas.GemmConfig(2, 2, 2, 1.0, 0.0)
    with pytest.raises(b2blas.CublasError) as ei:
        handle.strided_batched_sgemm_simple(cfg, 3, np.zeros(11, np.float32), 4, np.zeros(12, np.float32), 4,
                                            np.zeros(12, np.float32), 4)
    assert ei.value.kind == "DimensionMismatch"


def test_sgemv_simple_short_x_is_dimension_error(handle):
    import b2blas

    with pytest.raises(b2blas.CublasError) as ei:
        handle.sgemv_simple(0, 4, 6, 1.0, np.zeros(24, np.float32), np.zeros(5, np.float32), 0.0,
                            np.zeros(4, np.float32))
    assert ei.value.kind == "DimensionMismatch"


def test_device_buffer_too_small_is_dimension_error(handle):
    import b2blas

    a = handle.zeroed(15)
    b = handle.zeroed(16)
    c = handle.zeroed(16)
    with pytest.raises(b2blas.CublasError) as ei:
        handle.sgemm(b2blas.GemmConfig(4, 4, 4, 1.0, 0.0), a, b, c)
    assert ei.value.kind == "DimensionMismatch"


def test_bad_algo_and_trans_are_invalid_argument(handle):
    import b2blas

    lib = b2blas.load_library()
    z = handle.zeroed(16)
    import ctypes

    p = ctypes.c_void_p(z.ptr)
    assert lib.b2b_sgemm(handle._h, 99, 4, 4, 4, 1.0, p, p, 0.0, p) == 3
    assert lib.b2b_sgemv(handle._h, 0, 7, 4, 4, 1.0, p, p, 0.0, p) == 3
    assert lib.b2b_sgemm(handle._h, 0, 4, 4, 4, 1.0, None, p, 0.0, p) == 3


def test_bounded_wait_timeout_reported_and_handle_usable(handle, oracle):
    import b2blas

    handle.selftest_bounded_wait(2_000_000)  # 2 ms
    with pytest.raises(b2blas.CublasError) as ei:
        handle.synchronize()
    assert ei.value.status == 4
    # The status was cleared and the context is intact: a GEMM still works.
    handle.synchronize()
    m = n = k = 128
    A = oracle.normal_f16(m * k, 1, 1, 0.0, 0.1)
    B = oracle.normal_f16(k * n, 1, 2, 0.0, 0.1)
    c = np.zeros(m * n, np.uint16)
    handle.hgemm_simple(b2blas.GemmConfig(m, n, k, 1.0, 0.0), A, B, c)
    assert oracle.rel_err(c, oracle.hgemm_f64(m, n, k, 1.0, A, B)) <= 2e-2


def test_set_stream_roundtrip(handle):
    import torch

    own = handle.stream()
    s = torch.cuda.Stream()
    handle.set_stream(s.cuda_stream)
    assert handle.stream() == s.cuda_stream
    handle.set_stream(None)
    assert handle.stream() == own
    handle.set_stream(0)  # torch's default stream -> the legacy default stream
    assert handle.stream() == 1
    handle.set_stream(None)


def test_stream_switch_orders_workspace_users(oracle):
    # SGEMV-T keeps its split-row partials in the handle's workspace.  A call
    # queued on stream 1 and one queued right after switching to stream 2
    # (which does not wait for stream 1 on its own) must not share the
    # partials: the switch orders stream 2 behind stream 1.
    import torch

    import b2blas

    h = b2blas.Handle(0)
    try:
        m, n = 8192, 4096
        outs, refs = [], []
        streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        bufs = []
        for i in range(2):
            A = oracle.uniform_f32(m * n, 60 + i, 1)
            x = oracle.uniform_f32(m, 60 + i, 2)
            refs.append(oracle.sgemv_f64(1, m, n, 1.0, A, x, 0.0, np.zeros(n, np.float32)))
            bufs.append((h.upload(A), h.upload(x), h.zeroed(n)))
        h.synchronize()
        for i in range(2):
            h.set_stream(streams[i].cuda_stream)
            a, x, y = bufs[i]
            for _ in range(20):
                h.sgemv(1, m, n, 1.0, a, x, 0.0, y)
        torch.cuda.synchronize()
        h.set_stream(None)
        for i in range(2):
            got = h.download(bufs[i][2])
            assert oracle.rel_err(got, refs[i]) <= oracle.tol_normwise(m, "f32")
    finally:
        h.close()


def test_device_info(handle):
    info = handle.device_info()
    assert info["sm_count"] >= 100 and info["device"] == 0
