"""The bench crate's helpers (benches/src/validator.rs, timer.rs, gemm.rs,
hgemm.rs, batched_gemm.rs, vector_ops.rs) as b2blas.benches provides them.
The validators are host-only; the timer and bench functions need a GPU."""
import numpy as np
import pytest


def test_validate_gemm_accepts_and_rejects():
    from b2blas import benches

    rng = np.random.default_rng(3)
    m, n, k = 7, 9, 5
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    c0 = rng.standard_normal(m * n).astype(np.float32)
    good = (1.5 * a.reshape(m, k).astype(np.float64) @ b.reshape(k, n) + 0.5 * c0.reshape(m, n)).astype(np.float32)
    benches.validate_gemm(m, n, k, 1.5, a, b, 0.5, c0, good.ravel(), 1e-5)
    bad = good.ravel().copy()
    bad[13] += 0.01
    with pytest.raises(benches.ValidationError, match=r"C\[1\]\[4\]"):
        benches.validate_gemm(m, n, k, 1.5, a, b, 0.5, c0, bad, 1e-3)
    # beta == 0 ignores C's old contents, NaN included
    zero_beta = (a.reshape(m, k).astype(np.float64) @ b.reshape(k, n)).astype(np.float32).ravel()
    benches.validate_gemm(m, n, k, 1.0, a, b, 0.0, np.full(m * n, np.nan, np.float32), zero_beta, 1e-5)
    nan = zero_beta.copy()
    nan[0] = np.nan
    with pytest.raises(benches.ValidationError, match="NaN"):
        benches.validate_gemm(m, n, k, 1.0, a, b, 0.0, c0, nan, 1e9)
    with pytest.raises(benches.ValidationError, match="elements"):
        benches.validate_gemm(m, n, k, 1.0, a[:-1], b, 0.0, c0, zero_beta, 1.0)


def test_validate_vector():
    from b2blas import benches

    x = np.arange(10, dtype=np.float32)
    benches.validate_vector(x, x + 1e-4, 1e-3)
    with pytest.raises(benches.ValidationError, match=r"\[3\]"):
        y = x.copy()
        y[3] += 1.0
        benches.validate_vector(x, y, 0.5)
    with pytest.raises(benches.ValidationError, match="length"):
        benches.validate_vector(x, x[:-1], 1.0)
    benches.validate_vector([], [], 0.0)


@pytest.mark.gpu
def test_gpu_timer_matches_torch_events(handle):
    import torch

    from b2blas import benches

    s = torch.cuda.Stream()
    handle.set_stream(s.cuda_stream)
    try:
        with torch.cuda.stream(s):
            a = torch.randn(4096, 4096, device="cuda")
            torch.mm(a, a)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t = benches.GpuTimer.start(handle)
            e0.record(s)
            for _ in range(5):
                torch.mm(a, a)
            e1.record(s)
            ms = t.stop()
            torch.cuda.synchronize()
        ref = e0.elapsed_time(e1)
        assert ms > 0 and abs(ms - ref) <= 0.05 * ref + 0.05
        with pytest.raises(RuntimeError):
            t.stop()
    finally:
        handle.set_stream(None)


@pytest.mark.gpu
def test_bench_functions_run(handle, capsys):
    from b2blas import benches

    rows = benches.bench_sgemm(512, 512, 512, reps=2, warmup=1, handle=handle)
    assert [r["variant"] for r in rows][-1] == "cuBLAS sgemm" and all(r["rate"] > 0 for r in rows)
    assert len(rows) == 6
    for fn in (benches.bench_dgemm, benches.bench_hgemm):
        rows = fn(256, 384, 128, reps=2, warmup=1, handle=handle)
        assert all(r["rate"] > 0 for r in rows)
    rows = benches.bench_batched_sgemm(64, 64, 64, 16, reps=2, warmup=1, handle=handle)
    assert len(rows) == 2
    for fn in (benches.bench_saxpy, benches.bench_dot, benches.bench_nrm2):
        rows = fn(1 << 20, reps=2, warmup=1, handle=handle)
        assert all(r["rate"] > 0 for r in rows)
    out = capsys.readouterr().out
    assert "SGEMM 512x512x512" in out and "vs cuBLAS" in out
