// sgemm_example.cpp -- the reference's example known-answer checks, written
// against the C++ Handle mirror (cublas_rs.hpp).
//
// Same checks as examples/sgemm/src/main.rs (SGEMM 512^3 in four variants,
// DGEMM naive/tiled, strided and list-batched 8 x 64^3, HGEMM 128^3), the
// gemm_bench verification (examples/gemm_bench/src/main.rs:147-153, device
// buffers, sizes 256/512/1024) and the sgemv smoke check
// (examples/saxpy/src/main.rs:88-124), then the saxpy example's reduction
// and hgemv checks and the bench crate's timer and validators.  GEMM/GEMV
// inputs are all ones, so every output equals the inner dimension.  Exits 1 on the first failure, like the
// reference's examples.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "cublas_rs.hpp"

using namespace cublas_rs;

static void fail(const char *what) {
    std::fprintf(stderr, "FAIL: %s\n", what);
    std::exit(1);
}

template <typename T>
static size_t bad_count(const std::vector<T> &c, double expect, double tol) {
    size_t bad = 0;
    for (const T &v : c)
        if (std::fabs(double(v) - expect) > tol) ++bad;
    return bad;
}

int main() {
    try {
        Handle h = Handle::create();
        const size_t M = 512, N = 512, K = 512;
        {
            GemmConfig<float> cfg{M, N, K, 1.0f, 0.0f};
            std::vector<float> a(M * K, 1.0f), b(K * N, 1.0f);
            using Fn = void (Handle::*)(const GemmConfig<float> &, const std::vector<float> &,
                                        const std::vector<float> &, std::vector<float> &) const;
            const std::pair<const char *, Fn> variants[] = {{"naive", &Handle::sgemm_naive_simple},
                                                            {"tiled", &Handle::sgemm_tiled_simple},
                                                            {"vector", &Handle::sgemm_vectorized_simple},
                                                            {"dblbuf", &Handle::sgemm_double_buf_simple}};
            for (auto &v : variants) {
                std::vector<float> c(M * N, 0.0f);
                (h.*v.second)(cfg, a, b, c);  // warmup, as the reference does
                auto t0 = std::chrono::steady_clock::now();
                (h.*v.second)(cfg, a, b, c);
                double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
                if (bad_count(c, double(K), 1e-3)) fail(v.first);
                std::printf("  SGEMM %6s: %.3f ms OK\n", v.first, ms);
            }
        }
        {
            GemmConfig<double> cfg{M, N, K, 1.0, 0.0};
            std::vector<double> a(M * K, 1.0), b(K * N, 1.0);
            std::vector<double> c(M * N, 0.0);
            h.dgemm_naive_simple(cfg, a, b, c);
            if (bad_count(c, double(K), 1e-3)) fail("dgemm naive");
            std::fill(c.begin(), c.end(), 0.0);
            h.dgemm_tiled_simple(cfg, a, b, c);
            if (bad_count(c, double(K), 1e-3)) fail("dgemm tiled");
            std::printf("  DGEMM naive/tiled OK\n");
        }
        {
            const size_t B = 8, m = 64;
            GemmConfig<float> cfg{m, m, m, 1.0f, 0.0f};
            std::vector<float> a(B * m * m, 1.0f), b(B * m * m, 1.0f), c(B * m * m, 0.0f);
            h.strided_batched_sgemm_simple(cfg, B, a, m * m, b, m * m, c, m * m);
            if (bad_count(c, 64.0, 1e-3)) fail("strided batched");
            std::vector<std::vector<float>> as(B, std::vector<float>(m * m, 1.0f)), bs = as,
                                            cs(B, std::vector<float>(m * m, 0.0f));
            std::vector<const float *> ap, bp;
            std::vector<float *> cp;
            std::vector<size_t> lens(B, m * m);
            for (size_t i = 0; i < B; ++i) {
                ap.push_back(as[i].data());
                bp.push_back(bs[i].data());
                cp.push_back(cs[i].data());
            }
            h.batched_sgemm(cfg, B, ap, lens, bp, lens, cp, lens);
            for (auto &x : cs)
                if (bad_count(x, 64.0, 1e-3)) fail("batched (slices)");
            std::printf("  strided + list batched 8 x 64^3 OK\n");
        }
        {
            const size_t m = 128;
            GemmConfig<f16> cfg{m, m, m, f16::from_f32(1.0f), f16::from_f32(0.0f)};
            std::vector<f16> a(m * m, f16::from_f32(1.0f)), b = a, c(m * m, f16::from_f32(0.0f));
            h.hgemm_half(cfg, a, b, c);
            for (const f16 &v : c)
                if (std::fabs(v.to_f32() - 128.0f) / 128.0f > 5e-3f) fail("hgemm");
            std::printf("  HGEMM 128^3 OK\n");
        }
        for (size_t size : {256, 512, 1024}) {  // gemm_bench: device buffers
            GemmConfig<float> cfg{size, size, size, 1.0f, 0.0f};
            auto a = h.upload(std::vector<float>(size * size, 1.0f));
            auto b = h.upload(std::vector<float>(size * size, 1.0f));
            auto c = h.zeroed<float>(size * size);
            for (int i = 0; i < 3; ++i) h.sgemm_tiled(cfg, a, b, c);
            h.synchronize();
            if (bad_count(h.download(c), double(size), 1e-3)) fail("gemm_bench sgemm");
            GemmConfig<double> dcfg{size, size, size, 1.0, 0.0};
            auto da = h.upload(std::vector<double>(size * size, 1.0));
            auto db = h.upload(std::vector<double>(size * size, 1.0));
            auto dc = h.zeroed<double>(size * size);
            h.dgemm_vectorized(dcfg, da, db, dc);
            h.synchronize();
            if (bad_count(h.download(dc), double(size), 1e-3)) fail("gemm_bench dgemm");
        }
        std::printf("  gemm_bench 256/512/1024 OK\n");
        {
            const size_t m = 16, n = 24;
            std::vector<float> a(m * n, 1.0f), x(n, 1.0f), y(m, 0.0f);
            h.sgemv_simple(Transpose::NoTrans, m, n, 1.0f, a, x, 0.0f, y);
            if (bad_count(y, double(n), 1e-3)) fail("sgemv N");
            std::vector<float> xt(m, 1.0f), yt(n, 0.0f);
            h.sgemv_tiled_simple(Transpose::Trans, m, n, 1.0f, a, xt, 0.0f, yt);
            if (bad_count(yt, double(m), 1e-3)) fail("sgemv T");
            std::printf("  sgemv N/T OK\n");
        }
        {
            // The saxpy example's reduction and hgemv checks
            // (examples/saxpy/src/main.rs:38-63, 132-172).
            const size_t n = 1024;
            std::vector<float> x(n);
            for (size_t i = 0; i < n; ++i) x[i] = float(i);
            const double sumsq = 357389824.0, asum = 523776.0;  // closed forms of sum i^2, sum i
            const auto rel = [](double got, double want) { return std::fabs(got - want) / want; };
            if (rel(h.sdot_simple(n, x, x), sumsq) > 1e-3) fail("sdot");
            if (rel(h.snrm2_simple(n, x), std::sqrt(sumsq)) > 1e-3) fail("snrm2");
            if (rel(h.sasum_simple(n, x), asum) > 1e-3) fail("sasum");
            if (h.isamax_simple(n, x) != n - 1) fail("isamax");
            auto xd = h.upload(x);
            if (rel(h.sdot(n, xd, xd), sumsq) > 1e-3 || h.isamax(n, xd) != n - 1) fail("device reductions");
            const size_t m = 16, k = 24;
            std::vector<f16> a16(m * k), x16(k), y16(m, f16::from_f32(0.0f));
            for (size_t i = 0; i < m * k; ++i) a16[i] = f16::from_f32(float(i) * 0.01f);
            for (size_t j = 0; j < k; ++j) x16[j] = f16::from_f32(float(j) * 0.1f);
            h.hgemv(Transpose::NoTrans, m, k, f16::from_f32(1.0f), a16, x16, f16::from_f32(0.0f), y16);
            for (size_t i = 0; i < m; ++i) {
                float want = 0.0f;
                for (size_t j = 0; j < k; ++j) want += a16[i * k + j].to_f32() * x16[j].to_f32();
                if (std::fabs(y16[i].to_f32() - want) / std::max(std::fabs(want), 1e-6f) > 5e-3f) fail("hgemv");
            }
            std::vector<double> ad(m * k, 1.0), xdv(k, 1.0), ydv(m, 0.0);
            h.dgemv_simple(Transpose::NoTrans, m, k, 1.0, ad, xdv, 0.0, ydv);
            if (bad_count(ydv, double(k), 1e-9)) fail("dgemv");
            std::printf("  reductions, hgemv, dgemv OK\n");
        }
        {
            // GpuTimer and the validators (benches/src/timer.rs, validator.rs)
            const size_t s = 256;
            GemmConfig<float> cfg{s, s, s, 1.0f, 0.0f};
            std::vector<float> a(s * s), b(s * s), c0(s * s, 0.0f);
            for (size_t i = 0; i < s * s; ++i) {
                a[i] = float(int(i % 7) - 3);
                b[i] = float(int(i % 5) - 2) * 0.5f;
            }
            auto da = h.upload(a), db = h.upload(b);
            auto dc = h.zeroed<float>(s * s);
            GpuTimer t = GpuTimer::start(h);
            h.sgemm(cfg, da, db, dc);
            const double ms = t.stop();
            if (!(ms > 0.0)) fail("GpuTimer");
            const std::vector<float> c = h.download(dc);
            if (!validate_gemm(s, s, s, 1.0f, a, b, 0.0f, c0, c, 1e-3f).ok()) fail("validate_gemm on a good C");
            std::vector<float> bad = c;
            bad[77] += 1.0f;
            if (validate_gemm(s, s, s, 1.0f, a, b, 0.0f, c0, bad, 1e-3f).ok()) fail("validate_gemm on a bad C");
            if (!validate_vector(c, c, 0.0f).ok() || validate_vector(c, bad, 0.5f).ok()) fail("validate_vector");
            std::printf("  GpuTimer %.4f ms, validate_gemm/validate_vector OK\n", ms);
        }
        {
            // A short A slice is a DimensionMismatch (the reference panics).
            bool threw = false;
            try {
                std::vector<float> a(15), b(16), c(16);
                h.sgemm_tiled_simple(GemmConfig<float>{4, 4, 4, 1.0f, 0.0f}, a, b, c);
            } catch (const CublasError &e) {
                threw = e.kind() == CublasError::Kind::DimensionMismatch;
            }
            if (!threw) fail("length check");
            std::printf("  length check OK\n");
        }
    } catch (const CublasError &e) {
        std::fprintf(stderr, "CublasError: %s\n", e.what());
        return 1;
    }
    std::printf("all OK\n");
    return 0;
}
