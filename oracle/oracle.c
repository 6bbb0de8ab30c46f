/*
 * oracle.c -- CPU restatement of cublas-rs's Level-3 / Level-2 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: the parity tests, the
 * smoke check and the CPU-baseline leg of the bench call it; the product
 * library (libb2blas) never links or calls it, and there is no CPU fallback
 * anywhere in the product path.
 *
 * What is restated, and from where (paths inside the cublas-rs project):
 *   - GEMM  C <- alpha*A*B + beta*C, row-major A[MxK], B[KxN], C[MxN],
 *     sum over k then alpha*sum + beta*C:
 *       crates/cublas-l3/src/sgemm.rs:50-56 (naive), :121-127 (tiled epilogue)
 *       crates/cublas-l3/src/dgemm.rs:44-50 (f64)
 *   - HGEMM f16 in, f32 accumulate, f16 out, with the reference's own
 *     software conversions (subnormal flush on decode, truncation on encode):
 *       crates/cublas-l3/src/hgemm.rs:20-32 (f16_to_f32), :34-51 (f32_to_f16),
 *       :116-124 (epilogue)
 *   - strided batched: base offsets batch*stride, crates/cublas-l3/src/batched.rs:55-58,95-100
 *   - GEMV N / T index formulas, crates/cublas-l2/src/gemv.rs:28-81
 *   - SAXPY y = alpha*x + y, crates/cublas-l1/src/saxpy.rs:14-19
 *
 * The reference's device arithmetic is produced by cuda-oxide (git rev
 * 396c76aaca11de3a49c982afd94069dbbc1cb8ef, Cargo.lock:161-183), which is not
 * vendored, so whether `sum += a*b` is contracted to an FMA is not pinned.
 * The parity bar is therefore a normwise bound against an FP64 evaluation
 * (oracle_*_f64 below) plus the reference's all-ones known answers.
 *
 * Inputs for tests come from PCG32 (O'Neill, XSH-RR 64->32), seed and stream
 * chosen per tensor; uniform[lo,hi) = lo + (hi-lo) * (u>>8) * 2^-24; normal
 * by Box-Muller in FP64.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ PCG32 */

typedef struct {
    uint64_t state;
    uint64_t inc;
} pcg32_t;

static uint32_t pcg32_next(pcg32_t *r) {
    uint64_t old = r->state;
    r->state = old * 6364136223846793005ULL + r->inc;
    uint32_t xorshifted = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    uint32_t rot = (uint32_t)(old >> 59u);
    return (xorshifted >> rot) | (xorshifted << ((32u - rot) & 31u));
}

static void pcg32_seed(pcg32_t *r, uint64_t seed, uint64_t stream) {
    r->state = 0u;
    r->inc = (stream << 1u) | 1u;
    pcg32_next(r);
    r->state += seed;
    pcg32_next(r);
}

uint32_t oracle_pcg32_first(uint64_t seed, uint64_t stream, uint32_t *out, size_t n) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = pcg32_next(&r);
    return n ? out[0] : 0u;
}

/* u in [0,1) with 24 random bits */
static double u24(pcg32_t *r) { return (double)(pcg32_next(r) >> 8) * (1.0 / 16777216.0); }

void oracle_fill_uniform_f32(float *out, size_t n, uint64_t seed, uint64_t stream, double lo, double hi) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = (float)(lo + (hi - lo) * u24(&r));
}

void oracle_fill_uniform_f64(double *out, size_t n, uint64_t seed, uint64_t stream, double lo, double hi) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = lo + (hi - lo) * u24(&r);
}

static double normal01(pcg32_t *r, int *have_spare, double *spare) {
    if (*have_spare) {
        *have_spare = 0;
        return *spare;
    }
    double u1 = ((double)(pcg32_next(r) >> 8) + 1.0) * (1.0 / 16777216.0); /* (0,1] */
    double u2 = u24(r);
    double rad = sqrt(-2.0 * log(u1));
    double th = 2.0 * 3.14159265358979323846 * u2;
    *spare = rad * sin(th);
    *have_spare = 1;
    return rad * cos(th);
}

void oracle_fill_normal_f32(float *out, size_t n, uint64_t seed, uint64_t stream, double mean, double std) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    int hs = 0;
    double sp = 0.0;
    for (size_t i = 0; i < n; ++i) out[i] = (float)(mean + std * normal01(&r, &hs, &sp));
}

/* ------------------------------------------------------------ f16 helpers */

/* Reference decode, crates/cublas-l3/src/hgemm.rs:20-32: subnormals flush to
 * a signed zero, exp==31 keeps inf/nan, otherwise rebias 15 -> 127. */
float oracle_ref_f16_to_f32(uint16_t h16) {
    uint32_t h = h16;
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) bits = sign;
    else if (exp == 31) bits = sign | (0xffu << 23) | (mant << 13);
    else bits = sign | ((exp + 112u) << 23) | (mant << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Reference encode, crates/cublas-l3/src/hgemm.rs:34-51: truncates the
 * mantissa, flushes results below the f16 normal range to a signed zero,
 * saturates overflow to inf, maps nan to a quiet nan with payload 1. */
uint16_t oracle_ref_f32_to_f16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exp = (int32_t)((bits >> 23) & 0xffu);
    uint32_t mant = bits & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant != 0 ? 1u : 0u));
    int32_t ne = exp - 127 + 15;
    if (ne >= 31) return (uint16_t)(sign | 0x7c00u);
    if (ne <= 0) return sign;
    return (uint16_t)(sign | ((uint32_t)ne << 10) | (mant >> 13));
}

/* Exact widening of an IEEE binary16 value (subnormals kept). */
double oracle_f16_to_f64(uint16_t h) {
    int sign = (h >> 15) & 1;
    int exp = (h >> 10) & 0x1f;
    int mant = h & 0x3ff;
    double v;
    if (exp == 0) v = ldexp((double)mant, -24);
    else if (exp == 31) v = mant ? NAN : INFINITY;
    else v = ldexp((double)(mant | 0x400), exp - 25);
    return sign ? -v : v;
}

/* IEEE round-to-nearest-even binary64 -> binary16 (what the half crate's
 * f16::from_f64/from_f32 and the GPU's cvt.rn.f16 produce). */
uint16_t oracle_f64_to_f16_rne(double x) {
    uint16_t sign = 0;
    if (signbit(x)) {
        sign = 0x8000u;
        x = -x;
    }
    if (isnan(x)) return (uint16_t)(sign | 0x7e00u);
    if (x >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (x < ldexp(1.0, -25)) {
        /* exactly 2^-25 rounds to even (0); anything above rounds up */
        return sign;
    }
    int e;
    double m = frexp(x, &e); /* x = m * 2^e, m in [0.5,1) */
    int exp16 = e - 1 + 15;  /* biased exponent if normal */
    if (exp16 <= 0) {
        /* subnormal: value = q * 2^-24 */
        double q = x * 16777216.0;
        double fl = floor(q);
        double diff = q - fl;
        uint32_t qi = (uint32_t)fl;
        if (diff > 0.5 || (diff == 0.5 && (qi & 1u))) qi++;
        return (uint16_t)(sign | qi); /* qi==0x400 carries into the first normal */
    }
    /* normal: mantissa with 10 fraction bits */
    double scaled = ldexp(m, 11); /* in [1024, 2048) */
    double fl = floor(scaled);
    double diff = scaled - fl;
    uint32_t mi = (uint32_t)fl;
    if (diff > 0.5 || (diff == 0.5 && (mi & 1u))) mi++;
    if (mi == 2048u) {
        mi = 1024u;
        exp16++;
    }
    if (exp16 >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exp16 << 10) | (mi & 0x3ffu));
}

void oracle_fill_normal_f16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream, double mean, double std) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    int hs = 0;
    double sp = 0.0;
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f64_to_f16_rne(mean + std * normal01(&r, &hs, &sp));
}

void oracle_fill_uniform_f16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream, double lo, double hi) {
    pcg32_t r;
    pcg32_seed(&r, seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f64_to_f16_rne(lo + (hi - lo) * u24(&r));
}

/* --------------------------------------------------- FP64 GEMM evaluation */

/* Rows [row0, row0+nrows) of alpha*A*B + beta*C, evaluated in FP64, written
 * to out[(i-row0)*n + j].  Element accessors widen the stored values
 * exactly.  C may be NULL (treated as zero).  i-k-j order: the j loop is
 * contiguous in B and out. */
#define GEMM_F64_BODY(LOADA, LOADB, LOADC)                                            \
    _Pragma("omp parallel for schedule(dynamic, 1)") for (long ii = 0; ii < (long)nrows; \
                                                          ++ii) {                       \
        size_t i = row0 + (size_t)ii;                                                   \
        double *o = out + (size_t)ii * n;                                               \
        for (size_t j = 0; j < n; ++j) o[j] = 0.0;                                      \
        for (size_t p = 0; p < k; ++p) {                                                \
            double a = LOADA(i * k + p);                                                \
            const size_t brow = p * n;                                                  \
            for (size_t j = 0; j < n; ++j) o[j] += a * LOADB(brow + j);                 \
        }                                                                               \
        for (size_t j = 0; j < n; ++j) {                                                \
            double c = C ? LOADC(i * n + j) : 0.0;                                      \
            o[j] = alpha * o[j] + (beta != 0.0 ? beta * c : 0.0);                       \
        }                                                                               \
    }

#define LD_F32A(idx) ((double)A[(idx)])
#define LD_F32B(idx) ((double)B[(idx)])
#define LD_F32C(idx) ((double)C[(idx)])
void oracle_sgemm_rows_f64(size_t m, size_t n, size_t k, size_t row0, size_t nrows, double alpha,
                           const float *A, const float *B, double beta, const float *C, double *out) {
    (void)m;
    GEMM_F64_BODY(LD_F32A, LD_F32B, LD_F32C)
}

#define LD_F64A(idx) (A[(idx)])
#define LD_F64B(idx) (B[(idx)])
#define LD_F64C(idx) (C[(idx)])
void oracle_dgemm_rows_f64(size_t m, size_t n, size_t k, size_t row0, size_t nrows, double alpha,
                           const double *A, const double *B, double beta, const double *C, double *out) {
    (void)m;
    GEMM_F64_BODY(LD_F64A, LD_F64B, LD_F64C)
}

#define LD_F16A(idx) (oracle_f16_to_f64(A[(idx)]))
#define LD_F16B(idx) (oracle_f16_to_f64(B[(idx)]))
#define LD_F16C(idx) (oracle_f16_to_f64(C[(idx)]))
void oracle_hgemm_rows_f64(size_t m, size_t n, size_t k, size_t row0, size_t nrows, double alpha,
                           const uint16_t *A, const uint16_t *B, double beta, const uint16_t *C,
                           double *out) {
    (void)m;
    GEMM_F64_BODY(LD_F16A, LD_F16B, LD_F16C)
}

/* strided batched: batch b uses A + b*sa, B + b*sb, C + b*sc
 * (crates/cublas-l3/src/batched.rs:55-58). out is batch-major [batch][m][n]. */
void oracle_sgemm_strided_batched_f64(size_t m, size_t n, size_t k, double alpha, const float *A, size_t sa,
                                      const float *B, size_t sb, double beta, const float *C, size_t sc,
                                      size_t batch, double *out) {
    for (size_t b = 0; b < batch; ++b)
        oracle_sgemm_rows_f64(m, n, k, 0, m, alpha, A + b * sa, B + b * sb, beta, C ? C + b * sc : NULL,
                              out + b * m * n);
}

/* GEMV, crates/cublas-l2/src/gemv.rs:28-81.  A is m x n row-major.
 * trans==0: y[i] = alpha*sum_j A[i,j] x[j] + beta*y[i]  (len m)
 * trans==1: y[j] = alpha*sum_i A[i,j] x[i] + beta*y[j]  (len n) */
void oracle_sgemv_f64(int trans, size_t m, size_t n, double alpha, const float *A, const float *x,
                      double beta, const float *y, double *out) {
    if (!trans) {
#pragma omp parallel for schedule(static)
        for (long ii = 0; ii < (long)m; ++ii) {
            size_t i = (size_t)ii;
            double s = 0.0;
            for (size_t j = 0; j < n; ++j) s += (double)A[i * n + j] * (double)x[j];
            out[i] = alpha * s + (beta != 0.0 ? beta * (double)y[i] : 0.0);
        }
    } else {
        for (size_t j = 0; j < n; ++j) out[j] = 0.0;
        for (size_t i = 0; i < m; ++i) {
            double xi = x[i];
            for (size_t j = 0; j < n; ++j) out[j] += (double)A[i * n + j] * xi;
        }
        for (size_t j = 0; j < n; ++j) out[j] = alpha * out[j] + (beta != 0.0 ? beta * (double)y[j] : 0.0);
    }
}

/* SAXPY, crates/cublas-l1/src/saxpy.rs:14-19 */
void oracle_saxpy_f64(size_t n, double alpha, const float *x, const float *y, double *out) {
    for (size_t i = 0; i < n; ++i) out[i] = alpha * (double)x[i] + (double)y[i];
}

/* ------------------------------------- reference-arithmetic restatements */

/* The reference's f32 kernel arithmetic: per output, sum += a*b in k order in
 * f32 (unfused multiply-add), then alpha*sum + beta*c  (sgemm.rs:50-56). */
void oracle_sgemm_ref_f32(size_t m, size_t n, size_t k, float alpha, const float *A, const float *B, float beta,
                          float *C) {
#pragma omp parallel for schedule(static)
    for (long ii = 0; ii < (long)m; ++ii) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; ++j) {
            volatile float sum = 0.0f;
            for (size_t p = 0; p < k; ++p) {
                volatile float prod = A[i * k + p] * B[p * n + j];
                sum = sum + prod;
            }
            C[i * n + j] = alpha * sum + beta * C[i * n + j];
        }
    }
}

/* The reference's HGEMM arithmetic (hgemm.rs:104-124): decode with the
 * flushing f16_to_f32, f32 accumulate in k order, epilogue
 * f32_to_f16(alpha*sum + beta*f16_to_f32(c)) with the truncating encode. */
void oracle_hgemm_ref(size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B, float beta,
                      uint16_t *C) {
#pragma omp parallel for schedule(static)
    for (long ii = 0; ii < (long)m; ++ii) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (size_t p = 0; p < k; ++p)
                sum += oracle_ref_f16_to_f32(A[i * k + p]) * oracle_ref_f16_to_f32(B[p * n + j]);
            float cur = oracle_ref_f16_to_f32(C[i * n + j]);
            C[i * n + j] = oracle_ref_f32_to_f16(alpha * sum + beta * cur);
        }
    }
}

/* ------------------------------------------------------------ error norms */

double oracle_rel_fro_err_f32(const float *got, const double *ref, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        double d = (double)got[i] - ref[i];
        num += d * d;
        den += ref[i] * ref[i];
    }
    if (den == 0.0) return sqrt(num);
    return sqrt(num / den);
}

double oracle_rel_fro_err_f64(const double *got, const double *ref, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        double d = got[i] - ref[i];
        num += d * d;
        den += ref[i] * ref[i];
    }
    if (den == 0.0) return sqrt(num);
    return sqrt(num / den);
}

double oracle_rel_fro_err_f16(const uint16_t *got, const double *ref, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        double d = oracle_f16_to_f64(got[i]) - ref[i];
        num += d * d;
        den += ref[i] * ref[i];
    }
    if (den == 0.0) return sqrt(num);
    return sqrt(num / den);
}

/* ----------------------------------------------- timed CPU baseline loops */

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int t) {
#ifdef _OPENMP
    if (t > 0) omp_set_num_threads(t);
#else
    (void)t;
#endif
}

/* Host triple loop in i-k-j order with the reference's f32 accumulate, over
 * the first `rows` rows of C (the timed sample). */
void oracle_cpu_sgemm_ikj(size_t rows, size_t n, size_t k, float alpha, const float *A, const float *B, float beta,
                          float *C, float *rowacc) {
#pragma omp parallel for schedule(dynamic, 1)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        float *o = rowacc + i * n;
        for (size_t j = 0; j < n; ++j) o[j] = 0.0f;
        for (size_t p = 0; p < k; ++p) {
            float a = A[i * k + p];
            const float *b = B + p * n;
            for (size_t j = 0; j < n; ++j) o[j] += a * b[j];
        }
        for (size_t j = 0; j < n; ++j) C[i * n + j] = alpha * o[j] + beta * C[i * n + j];
    }
}

void oracle_cpu_dgemm_ikj(size_t rows, size_t n, size_t k, double alpha, const double *A, const double *B,
                          double beta, double *C, double *rowacc) {
#pragma omp parallel for schedule(dynamic, 1)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        double *o = rowacc + i * n;
        for (size_t j = 0; j < n; ++j) o[j] = 0.0;
        for (size_t p = 0; p < k; ++p) {
            double a = A[i * k + p];
            const double *b = B + p * n;
            for (size_t j = 0; j < n; ++j) o[j] += a * b[j];
        }
        for (size_t j = 0; j < n; ++j) C[i * n + j] = alpha * o[j] + beta * C[i * n + j];
    }
}

/* HGEMM host loop: B is decoded to f32 once per call (the reference decodes
 * in its kernel), rows of A decoded on the fly, f32 accumulate, truncating
 * encode of the result.  `Bf` is caller scratch of k*n floats. */
void oracle_cpu_hgemm_ikj(size_t rows, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                          float beta, uint16_t *C, float *Bf, float *rowacc) {
#pragma omp parallel for schedule(static)
    for (long q = 0; q < (long)(k * n); ++q) Bf[q] = oracle_ref_f16_to_f32(B[q]);
#pragma omp parallel for schedule(dynamic, 1)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        float *o = rowacc + i * n;
        for (size_t j = 0; j < n; ++j) o[j] = 0.0f;
        for (size_t p = 0; p < k; ++p) {
            float a = oracle_ref_f16_to_f32(A[i * k + p]);
            const float *b = Bf + p * n;
            for (size_t j = 0; j < n; ++j) o[j] += a * b[j];
        }
        for (size_t j = 0; j < n; ++j)
            C[i * n + j] = oracle_ref_f32_to_f16(alpha * o[j] + beta * oracle_ref_f16_to_f32(C[i * n + j]));
    }
}

void oracle_cpu_sgemv_n(size_t rows, size_t n, float alpha, const float *A, const float *x, float beta, float *y) {
#pragma omp parallel for schedule(static)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        float s = 0.0f;
        for (size_t j = 0; j < n; ++j) s += A[i * n + j] * x[j];
        y[i] = alpha * s + beta * y[i];
    }
}
