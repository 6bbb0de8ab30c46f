// cublas_rs.hpp -- header-only C++ mirror of cublas-rs's Handle API
// (crates/cublas-rs/src/lib.rs:42-716) over the b2blas C ABI.
//
// Same method names, argument order, row-major layout and alpha/beta
// semantics.  Rust's Result<()> becomes a thrown CublasError whose kind()
// names the cublas_core::CublasError variant (crates/cublas-core/src/
// error.rs:7-24); where the reference panics on a host-slice length mismatch
// (crates/cublas-l3/src/sgemm.rs:469-471) the C ABI reports
// DimensionMismatch and this header throws it.  `Handle::new()` is spelled
// `Handle::create()` (new is a C++ keyword).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "b2blas.h"

namespace cublas_rs {

// cublas_core::Transpose (crates/cublas-core/src/config.rs:20-23)
enum class Transpose { NoTrans = 0, Trans = 1 };

// cublas_core::GemmConfig<T> (crates/cublas-core/src/config.rs:3-9)
template <typename T>
struct GemmConfig {
    size_t m, n, k;
    T alpha, beta;
};

// half::f16 stand-in: IEEE binary16 bits; from_f32 rounds to nearest even.
struct f16 {
    uint16_t bits = 0;
    static f16 from_bits(uint16_t b) {
        f16 h;
        h.bits = b;
        return h;
    }
    static f16 from_f32(float f) {
        uint32_t x;
        std::memcpy(&x, &f, 4);
        const uint32_t sign = (x >> 16) & 0x8000u;
        const uint32_t ax = x & 0x7fffffffu;
        if (ax >= 0x7f800000u) return from_bits(uint16_t(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u)));
        if (ax >= 0x477ff000u) return from_bits(uint16_t(sign | 0x7c00u));  // rounds to inf
        if (ax < 0x38800000u) {                                            // f16 subnormal or zero
            if (ax < 0x33000000u) return from_bits(uint16_t(sign));        // < 2^-25 rounds to 0
            const uint32_t e = ax >> 23, mant = (ax & 0x7fffffu) | 0x800000u;
            const uint32_t shift = 126u - e;                               // 14..24
            uint32_t q = mant >> shift;
            const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
            if (rem > half || (rem == half && (q & 1u))) ++q;
            return from_bits(uint16_t(sign | q));
        }
        uint32_t r = ax - 0x38000000u;  // rebias 127 -> 15 in place
        const uint32_t rem = r & 0x1fffu;
        r >>= 13;
        if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
        return from_bits(uint16_t(sign | r));
    }
    float to_f32() const {
        const uint32_t sign = uint32_t(bits & 0x8000u) << 16;
        uint32_t e = (bits >> 10) & 0x1fu, m = bits & 0x3ffu, x;
        if (e == 0) {
            if (m == 0) {
                x = sign;
            } else {  // subnormal: normalise
                e = 113;
                while (!(m & 0x400u)) {
                    m <<= 1;
                    --e;
                }
                x = sign | (e << 23) | ((m & 0x3ffu) << 13);
            }
        } else if (e == 31) {
            x = sign | 0x7f800000u | (m << 13);
        } else {
            x = sign | ((e + 112u) << 23) | (m << 13);
        }
        float f;
        std::memcpy(&f, &x, 4);
        return f;
    }
};

class CublasError : public std::runtime_error {
   public:
    enum class Kind { Driver, EmbeddedModule, DimensionMismatch, InvalidArgument };
    CublasError(int status, const std::string &msg)
        : std::runtime_error(msg), status_(status), kind_(kind_of(status)) {}
    int status() const { return status_; }
    Kind kind() const { return kind_; }

   private:
    static Kind kind_of(int s) {
        switch (s) {
            case B2B_ERR_DIMENSION: return Kind::DimensionMismatch;
            case B2B_ERR_INVALID_ARG:
            case B2B_ERR_NOT_SUPPORTED: return Kind::InvalidArgument;
            default: return Kind::Driver;
        }
    }
    int status_;
    Kind kind_;
};

inline void check(int rc) {
    if (rc != B2B_OK) throw CublasError(rc, std::string(b2b_status_string(rc)) + ": " + b2b_last_error());
}

class Handle;

// cuda_core::DeviceBuffer<T> stand-in (re-exported as cublas_rs::DeviceBuf).
template <typename T>
class DeviceBuffer {
   public:
    DeviceBuffer() = default;
    DeviceBuffer(b2b_handle *h, size_t n) : h_(h), n_(n) { check(b2b_malloc(h_, n * sizeof(T), &p_)); }
    ~DeviceBuffer() { reset(); }
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    DeviceBuffer(DeviceBuffer &&o) noexcept { *this = std::move(o); }
    DeviceBuffer &operator=(DeviceBuffer &&o) noexcept {
        if (this != &o) {
            reset();
            h_ = o.h_;
            p_ = o.p_;
            n_ = o.n_;
            o.p_ = nullptr;
            o.n_ = 0;
        }
        return *this;
    }
    size_t len() const { return n_; }
    T *ptr() const { return static_cast<T *>(p_); }
    std::vector<T> to_host_vec() const {
        std::vector<T> v(n_);
        check(b2b_memcpy_d2h(h_, v.data(), p_, n_ * sizeof(T)));
        return v;
    }

   private:
    void reset() {
        if (p_) b2b_free(h_, p_);
        p_ = nullptr;
    }
    b2b_handle *h_ = nullptr;
    void *p_ = nullptr;
    size_t n_ = 0;
};

template <typename T>
using DeviceBuf = DeviceBuffer<T>;

class Handle {
   public:
    static Handle create() { return Handle(0); }
    static Handle with_device(size_t device_idx) { return Handle(static_cast<int>(device_idx)); }
    explicit Handle(int device = 0) { check(b2b_create(device, &h_)); }
    ~Handle() {
        if (h_) b2b_destroy(h_);
    }
    Handle(const Handle &) = delete;
    Handle &operator=(const Handle &) = delete;
    Handle(Handle &&o) noexcept : h_(o.h_) { o.h_ = nullptr; }

    b2b_handle *raw() const { return h_; }
    void *stream() const {
        void *s = nullptr;
        check(b2b_get_stream(h_, &s));
        return s;
    }
    void synchronize() const { check(b2b_synchronize(h_)); }

    template <typename T>
    DeviceBuffer<T> upload(const std::vector<T> &host) const {
        DeviceBuffer<T> d(h_, host.size());
        check(b2b_memcpy_h2d(h_, d.ptr(), host.data(), host.size() * sizeof(T)));
        return d;
    }
    template <typename T>
    std::vector<T> download(const DeviceBuffer<T> &d) const {
        return d.to_host_vec();
    }
    template <typename T>
    DeviceBuffer<T> zeroed(size_t n) const {
        DeviceBuffer<T> d(h_, n);
        check(b2b_memset(h_, d.ptr(), 0, n * sizeof(T)));
        return d;
    }

    // ---- Level 1 (lib.rs:110-129)
    void saxpy(size_t n, float alpha, const DeviceBuffer<float> &x, DeviceBuffer<float> &y) const {
        need(x, n, "x");
        need(y, n, "y");
        check(b2b_saxpy(h_, n, alpha, x.ptr(), y.ptr()));
    }
    void saxpy_simple(size_t n, float alpha, const std::vector<float> &x, std::vector<float> &y) const {
        check(b2b_saxpy_simple(h_, n, alpha, x.data(), x.size(), y.data(), y.size()));
    }

    // ---- Level 2 (lib.rs:230-309)
    void sgemv(Transpose t, size_t m, size_t n, float alpha, const DeviceBuffer<float> &a, const DeviceBuffer<float> &x,
               float beta, DeviceBuffer<float> &y, int algo = B2B_ALGO_DEFAULT) const {
        const size_t xl = t == Transpose::NoTrans ? n : m, yl = t == Transpose::NoTrans ? m : n;
        if (m && n) {
            need(a, m * n, "A");
            need(x, xl, "x");
            need(y, yl, "y");
        }
        check(b2b_sgemv(h_, algo, int(t), m, n, alpha, a.ptr(), x.ptr(), beta, y.ptr()));
    }
    void sgemv_simple(Transpose t, size_t m, size_t n, float alpha, const std::vector<float> &a,
                      const std::vector<float> &x, float beta, std::vector<float> &y,
                      int algo = B2B_ALGO_DEFAULT) const {
        check(b2b_sgemv_simple(h_, algo, int(t), m, n, alpha, a.data(), a.size(), x.data(), x.size(), beta, y.data(),
                               y.size()));
    }
    void sgemv_tiled(Transpose t, size_t m, size_t n, float alpha, const DeviceBuffer<float> &a,
                     const DeviceBuffer<float> &x, float beta, DeviceBuffer<float> &y) const {
        sgemv(t, m, n, alpha, a, x, beta, y, B2B_ALGO_TILED);
    }
    void sgemv_tiled_simple(Transpose t, size_t m, size_t n, float alpha, const std::vector<float> &a,
                            const std::vector<float> &x, float beta, std::vector<float> &y) const {
        sgemv_simple(t, m, n, alpha, a, x, beta, y, B2B_ALGO_TILED);
    }

    void dgemv(Transpose t, size_t m, size_t n, double alpha, const DeviceBuffer<double> &a,
               const DeviceBuffer<double> &x, double beta, DeviceBuffer<double> &y) const {
        const size_t xl = t == Transpose::NoTrans ? n : m, yl = t == Transpose::NoTrans ? m : n;
        if (m && n) {
            need(a, m * n, "A");
            need(x, xl, "x");
            need(y, yl, "y");
        }
        check(b2b_dgemv(h_, int(t), m, n, alpha, a.ptr(), x.ptr(), beta, y.ptr()));
    }
    void dgemv_simple(Transpose t, size_t m, size_t n, double alpha, const std::vector<double> &a,
                      const std::vector<double> &x, double beta, std::vector<double> &y) const {
        check(b2b_dgemv_simple(h_, int(t), m, n, alpha, a.data(), a.size(), x.data(), x.size(), beta, y.data(),
                               y.size()));
    }
    // Handle::hgemv (lib.rs:344-366): host slices only, alpha/beta as f16.
    void hgemv(Transpose t, size_t m, size_t n, f16 alpha, const std::vector<f16> &a, const std::vector<f16> &x,
               f16 beta, std::vector<f16> &y) const {
        check(b2b_hgemv_simple(h_, int(t), m, n, alpha.to_f32(), reinterpret_cast<const uint16_t *>(a.data()),
                               a.size(), reinterpret_cast<const uint16_t *>(x.data()), x.size(), beta.to_f32(),
                               reinterpret_cast<uint16_t *>(y.data()), y.size()));
    }

    // ---- Level 1 reductions (lib.rs:157-195); each returns the value
    float sdot(size_t n, const DeviceBuffer<float> &x, const DeviceBuffer<float> &y) const {
        if (n) {
            need(x, n, "x");
            need(y, n, "y");
        }
        float r = 0.0f;
        check(b2b_sdot(h_, n, x.ptr(), y.ptr(), &r));
        return r;
    }
    float sdot_simple(size_t n, const std::vector<float> &x, const std::vector<float> &y) const {
        float r = 0.0f;
        check(b2b_sdot_simple(h_, n, x.data(), x.size(), y.data(), y.size(), &r));
        return r;
    }
#define CUBLAS_RS_REDUCE(NAME)                                                      \
    float NAME(size_t n, const DeviceBuffer<float> &x) const {                      \
        if (n) need(x, n, "x");                                                     \
        float r = 0.0f;                                                             \
        check(b2b_##NAME(h_, n, x.ptr(), &r));                                      \
        return r;                                                                   \
    }                                                                               \
    float NAME##_simple(size_t n, const std::vector<float> &x) const {              \
        float r = 0.0f;                                                             \
        check(b2b_##NAME##_simple(h_, n, x.data(), x.size(), &r));                  \
        return r;                                                                   \
    }
    CUBLAS_RS_REDUCE(snrm2)
    CUBLAS_RS_REDUCE(sasum)
#undef CUBLAS_RS_REDUCE
    size_t isamax(size_t n, const DeviceBuffer<float> &x) const {
        if (n) need(x, n, "x");
        size_t r = 0;
        check(b2b_isamax(h_, n, x.ptr(), &r));
        return r;
    }
    size_t isamax_simple(size_t n, const std::vector<float> &x) const {
        size_t r = 0;
        check(b2b_isamax_simple(h_, n, x.data(), x.size(), &r));
        return r;
    }

    // ---- Level 3: SGEMM (lib.rs:439-524)
#define CUBLAS_RS_SGEMM_VARIANT(NAME, ALGO)                                                                    \
    void NAME(const GemmConfig<float> &c, const DeviceBuffer<float> &a, const DeviceBuffer<float> &b,        \
              DeviceBuffer<float> &cc) const {                                                               \
        gemm_dev(c, a, b, cc);                                                                               \
        check(b2b_sgemm(h_, ALGO, c.m, c.n, c.k, c.alpha, a.ptr(), b.ptr(), c.beta, cc.ptr()));              \
    }                                                                                                        \
    void NAME##_simple(const GemmConfig<float> &c, const std::vector<float> &a, const std::vector<float> &b, \
                       std::vector<float> &cc) const {                                                       \
        check(b2b_sgemm_simple(h_, ALGO, c.m, c.n, c.k, c.alpha, a.data(), a.size(), b.data(), b.size(),     \
                               c.beta, cc.data(), cc.size()));                                               \
    }
    CUBLAS_RS_SGEMM_VARIANT(sgemm, B2B_ALGO_DEFAULT)
    CUBLAS_RS_SGEMM_VARIANT(sgemm_naive, B2B_ALGO_NAIVE)
    CUBLAS_RS_SGEMM_VARIANT(sgemm_tiled, B2B_ALGO_TILED)
    CUBLAS_RS_SGEMM_VARIANT(sgemm_vectorized, B2B_ALGO_VECTORIZED)
    CUBLAS_RS_SGEMM_VARIANT(sgemm_double_buf, B2B_ALGO_DOUBLE_BUF)
#undef CUBLAS_RS_SGEMM_VARIANT

    // ---- Level 3: DGEMM (lib.rs:527-612)
#define CUBLAS_RS_DGEMM_VARIANT(NAME, ALGO)                                                                       \
    void NAME(const GemmConfig<double> &c, const DeviceBuffer<double> &a, const DeviceBuffer<double> &b,        \
              DeviceBuffer<double> &cc) const {                                                                 \
        gemm_dev(c, a, b, cc);                                                                                  \
        check(b2b_dgemm(h_, ALGO, c.m, c.n, c.k, c.alpha, a.ptr(), b.ptr(), c.beta, cc.ptr()));                 \
    }                                                                                                           \
    void NAME##_simple(const GemmConfig<double> &c, const std::vector<double> &a, const std::vector<double> &b, \
                       std::vector<double> &cc) const {                                                         \
        check(b2b_dgemm_simple(h_, ALGO, c.m, c.n, c.k, c.alpha, a.data(), a.size(), b.data(), b.size(),        \
                               c.beta, cc.data(), cc.size()));                                                  \
    }
    CUBLAS_RS_DGEMM_VARIANT(dgemm, B2B_ALGO_DEFAULT)
    CUBLAS_RS_DGEMM_VARIANT(dgemm_naive, B2B_ALGO_NAIVE)
    CUBLAS_RS_DGEMM_VARIANT(dgemm_tiled, B2B_ALGO_TILED)
    CUBLAS_RS_DGEMM_VARIANT(dgemm_vectorized, B2B_ALGO_VECTORIZED)
    CUBLAS_RS_DGEMM_VARIANT(dgemm_double_buf, B2B_ALGO_DOUBLE_BUF)
#undef CUBLAS_RS_DGEMM_VARIANT

    // ---- Level 3: HGEMM (lib.rs:616-635); host slices only, like the reference
    void hgemm_half(const GemmConfig<f16> &c, const std::vector<f16> &a, const std::vector<f16> &b,
                    std::vector<f16> &cc) const {
        static_assert(sizeof(f16) == 2, "f16 is two bytes");
        check(b2b_hgemm_simple(h_, c.m, c.n, c.k, c.alpha.to_f32(), reinterpret_cast<const uint16_t *>(a.data()),
                               a.size(), reinterpret_cast<const uint16_t *>(b.data()), b.size(), c.beta.to_f32(),
                               reinterpret_cast<uint16_t *>(cc.data()), cc.size()));
    }
    void hgemm_tensor_core(const GemmConfig<f16> &c, const std::vector<f16> &a, const std::vector<f16> &b,
                           std::vector<f16> &cc) const {
        hgemm_half(c, a, b, cc);
    }

    // ---- batched (lib.rs:639-709)
    void batched_sgemm(const GemmConfig<float> &c, size_t batch_count, const std::vector<const float *> &a,
                       const std::vector<size_t> &a_lens, const std::vector<const float *> &b,
                       const std::vector<size_t> &b_lens, std::vector<float *> &cc,
                       const std::vector<size_t> &c_lens) const {
        if (a.size() != batch_count || b.size() != batch_count || cc.size() != batch_count)
            throw CublasError(B2B_ERR_DIMENSION, "slice counts must equal batch_count");
        check(b2b_sgemm_batched_simple(h_, c.m, c.n, c.k, c.alpha, a.data(), a_lens.data(), b.data(), b_lens.data(),
                                       c.beta, cc.data(), c_lens.data(), batch_count));
    }
    void strided_batched_sgemm(const GemmConfig<float> &c, size_t batch_count, const DeviceBuffer<float> &a,
                               size_t stride_a, const DeviceBuffer<float> &b, size_t stride_b, DeviceBuffer<float> &cc,
                               size_t stride_c) const {
        if (c.m && c.n && c.k && batch_count) {
            need(a, (batch_count - 1) * stride_a + c.m * c.k, "A");
            need(b, (batch_count - 1) * stride_b + c.k * c.n, "B");
            need(cc, (batch_count - 1) * stride_c + c.m * c.n, "C");
        }
        check(b2b_sgemm_strided_batched(h_, c.m, c.n, c.k, c.alpha, a.ptr(), stride_a, b.ptr(), stride_b, c.beta,
                                        cc.ptr(), stride_c, batch_count));
    }
    void strided_batched_sgemm_simple(const GemmConfig<float> &c, size_t batch_count, const std::vector<float> &a,
                                      size_t stride_a, const std::vector<float> &b, size_t stride_b,
                                      std::vector<float> &cc, size_t stride_c) const {
        check(b2b_sgemm_strided_batched_simple(h_, c.m, c.n, c.k, c.alpha, a.data(), a.size(), stride_a, b.data(),
                                               b.size(), stride_b, c.beta, cc.data(), cc.size(), stride_c,
                                               batch_count));
    }

   private:
    template <typename T>
    static void need(const DeviceBuffer<T> &d, size_t n, const char *what) {
        if (d.len() < n)
            throw CublasError(B2B_ERR_DIMENSION, std::string("dimension mismatch in ") + what + ": expected " +
                                                     std::to_string(n) + ", got " + std::to_string(d.len()));
    }
    template <typename T>
    static void gemm_dev(const GemmConfig<T> &c, const DeviceBuffer<T> &a, const DeviceBuffer<T> &b,
                         const DeviceBuffer<T> &cc) {
        if (c.m && c.n && c.k) {
            need(a, c.m * c.k, "A");
            need(b, c.k * c.n, "B");
            need(cc, c.m * c.n, "C");
        }
    }
    b2b_handle *h_ = nullptr;
};

// GpuTimer (benches/src/timer.rs:6-19): start() records a CUDA event on the
// handle's stream; stop() records the end event, waits for it and returns
// the elapsed milliseconds.  Move-only; a timer dropped without stop() is
// released.
class GpuTimer {
   public:
    static GpuTimer start(const Handle &h) {
        b2b_gpu_timer *t = nullptr;
        check(b2b_gpu_timer_start(h.raw(), &t));
        return GpuTimer(t);
    }
    double stop() {
        if (!t_) throw CublasError(B2B_ERR_INVALID_ARG, "GpuTimer::stop called twice");
        double ms = 0.0;
        b2b_gpu_timer *t = t_;
        t_ = nullptr;
        check(b2b_gpu_timer_stop(t, &ms));
        return ms;
    }
    ~GpuTimer() {
        if (t_) b2b_gpu_timer_stop(t_, nullptr);
    }
    GpuTimer(const GpuTimer &) = delete;
    GpuTimer &operator=(const GpuTimer &) = delete;
    GpuTimer(GpuTimer &&o) noexcept : t_(o.t_) { o.t_ = nullptr; }

   private:
    explicit GpuTimer(b2b_gpu_timer *t) : t_(t) {}
    b2b_gpu_timer *t_ = nullptr;
};

// Result of validate_gemm / validate_vector (validator.rs:6-25), where the
// reference returns Result<(), String>: ok() or the error message.
struct Validation {
    std::string error;
    bool ok() const { return error.empty(); }
};

// validate_gemm (validator.rs:6-20): recompute alpha*A*B + beta*C on the
// host in double, C being `expected` (C before the call), and check
// max |actual - reference| <= tolerance.  Row-major A m x k, B k x n.
inline Validation validate_gemm(size_t m, size_t n, size_t k, float alpha, const std::vector<float> &a,
                                const std::vector<float> &b, float beta, const std::vector<float> &expected,
                                const std::vector<float> &actual, float tolerance) {
    if (a.size() != m * k || b.size() != k * n || expected.size() != m * n || actual.size() != m * n)
        return {"slice lengths do not match m, n, k"};
    std::vector<double> row(n);
    double worst = 0.0;
    size_t wi = 0;
    for (size_t i = 0; i < m; ++i) {
        std::fill(row.begin(), row.end(), 0.0);
        for (size_t p = 0; p < k; ++p) {
            const double av = a[i * k + p];
            for (size_t j = 0; j < n; ++j) row[j] += av * double(b[p * n + j]);
        }
        for (size_t j = 0; j < n; ++j) {
            double ref = double(alpha) * row[j];
            if (beta != 0.0f) ref += double(beta) * double(expected[i * n + j]);
            const double got = actual[i * n + j];
            const double err = got != got ? HUGE_VAL : (got > ref ? got - ref : ref - got);
            if (err > worst) {
                worst = err;
                wi = i * n + j;
            }
        }
    }
    if (worst > double(tolerance))
        return {"max abs error " + std::to_string(worst) + " at C[" + std::to_string(wi / n) + "][" +
                std::to_string(wi % n) + "] exceeds tolerance " + std::to_string(tolerance)};
    return {};
}

// validate_vector (validator.rs:22-25): equal lengths, element-wise
// max |actual - expected| <= tolerance.
inline Validation validate_vector(const std::vector<float> &expected, const std::vector<float> &actual,
                                  float tolerance) {
    if (expected.size() != actual.size()) return {"length mismatch"};
    for (size_t i = 0; i < expected.size(); ++i) {
        const double d = double(actual[i]) - double(expected[i]);
        if (!(d <= double(tolerance) && -d <= double(tolerance)))
            return {"element " + std::to_string(i) + " differs by " + std::to_string(d) + " (tolerance " +
                    std::to_string(tolerance) + ")"};
    }
    return {};
}

}  // namespace cublas_rs
