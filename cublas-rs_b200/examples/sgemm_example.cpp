// sgemm_example.cpp -- the reference's example known-answer checks, written
// against the C++ Handle mirror (cublas_rs.hpp).
//
// Same checks as examples/sgemm/src/main.rs (SGEMM 512^3 in four variants,
// DGEMM naive/tiled, strided and list-batched 8 x 64^3, HGEMM 128^3), the
// gemm_bench verification (examples/gemm_bench/src/main.rs:147-153, device
// buffers, sizes 256/512/1024) and the sgemv smoke check
// (examples/saxpy/src/main.rs:88-124).  All-ones inputs, so every output
// equals the inner dimension.  Exits 1 on the first failure, like the
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
