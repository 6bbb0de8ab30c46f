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
 *   - DGEMV (f64) and HGEMV (f16 in/out, f32 accumulate, the same
 *     conversions as HGEMM), crates/cublas-l2/src/gemv.rs:386-437, :553-606
 *   - SAXPY y = alpha*x + y, crates/cublas-l1/src/saxpy.rs:14-19
 *   - SDOT / SNRM2 / SASUM / ISAMAX, crates/cublas-l1/src/dot.rs:21-53,
 *     nrm2.rs:16-48, asum.rs:15-47, iamax.rs:16-61
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

/* DGEMV, crates/cublas-l2/src/gemv.rs:386-437 (same shapes as SGEMV), with
 * each dot product evaluated by Ogita-Rump-Oishi Dot2 (error-free
 * TwoProduct through fma plus TwoSum; "Accurate sum and dot product", SIAM J.
 * Sci. Comput. 26(6), 2005), so the oracle's own rounding error is about
 * eps_f64 * |y| + eps_f64^2 * sum |a x| and the parity bound measures the
 * kernel alone.  beta == 0 ignores y. */
static void dot2_acc(double *s, double *c, double a, double b) {
    double p = a * b;
    double pe = fma(a, b, -p);
    double t = *s + p;
    double z = t - *s;
    double se = (*s - (t - z)) + (p - z);
    *s = t;
    *c += pe + se;
}

void oracle_dgemv_f64(int trans, size_t m, size_t n, double alpha, const double *A, const double *x, double beta,
                      const double *y, double *out) {
    if (!trans) {
#pragma omp parallel for schedule(static)
        for (long ii = 0; ii < (long)m; ++ii) {
            size_t i = (size_t)ii;
            double s = 0.0, c = 0.0;
            for (size_t j = 0; j < n; ++j) dot2_acc(&s, &c, A[i * n + j], x[j]);
            out[i] = alpha * (s + c) + (beta != 0.0 ? beta * y[i] : 0.0);
        }
    } else {
#pragma omp parallel for schedule(static)
        for (long jj = 0; jj < (long)n; ++jj) {
            size_t j = (size_t)jj;
            double s = 0.0, c = 0.0;
            for (size_t i = 0; i < m; ++i) dot2_acc(&s, &c, A[i * n + j], x[i]);
            out[j] = alpha * (s + c) + (beta != 0.0 ? beta * y[j] : 0.0);
        }
    }
}

/* HGEMV in f64 from the exact f16 inputs (gemv.rs:553-606 shapes):
 * out = alpha*op(A)x + beta*y, unrounded. */
void oracle_hgemv_f64(int trans, size_t m, size_t n, double alpha, const uint16_t *A, const uint16_t *x,
                      double beta, const uint16_t *y, double *out) {
    size_t len = trans ? n : m;
#pragma omp parallel for schedule(static)
    for (long oo = 0; oo < (long)len; ++oo) {
        size_t o = (size_t)oo;
        double s = 0.0, c = 0.0;
        if (!trans)
            for (size_t j = 0; j < n; ++j) dot2_acc(&s, &c, oracle_f16_to_f64(A[o * n + j]), oracle_f16_to_f64(x[j]));
        else
            for (size_t i = 0; i < m; ++i) dot2_acc(&s, &c, oracle_f16_to_f64(A[i * n + o]), oracle_f16_to_f64(x[i]));
        out[o] = alpha * (s + c) + (beta != 0.0 ? beta * oracle_f16_to_f64(y[o]) : 0.0);
    }
}

/* Level-1 reductions in f64 (crates/cublas-l1/src/dot.rs:21-53,
 * nrm2.rs:16-48, asum.rs:15-47), each sum Dot2-compensated so the oracle is
 * accurate to about eps_f64 of the result. */
double oracle_sdot_f64(size_t n, const float *x, const float *y) {
    double s = 0.0, c = 0.0;
    for (size_t i = 0; i < n; ++i) dot2_acc(&s, &c, x[i], y[i]);
    return s + c;
}

double oracle_snrm2_f64(size_t n, const float *x) {
    double s = 0.0, c = 0.0;
    for (size_t i = 0; i < n; ++i) dot2_acc(&s, &c, x[i], x[i]);
    return sqrt(s + c);
}

double oracle_sasum_f64(size_t n, const float *x) {
    double s = 0.0, c = 0.0;
    for (size_t i = 0; i < n; ++i) dot2_acc(&s, &c, fabs((double)x[i]), 1.0);
    return s + c;
}

/* ISAMAX as the BLAS defines it: the smallest index of the largest |x[i]|.
 * NaN never compares greater (as in iamax.rs:26-31); all-NaN or n == 0 -> 0. */
size_t oracle_isamax(size_t n, const float *x) {
    float best = -1.0f;
    size_t idx = 0;
    for (size_t i = 0; i < n; ++i) {
        float a = fabsf(x[i]);
        if (a > best) {
            best = a;
            idx = i;
        }
    }
    return idx;
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

/* The reference's HGEMV arithmetic (gemv.rs:553-606): flushing decode, f32
 * accumulate in index order, f32_to_f16(alpha*sum + beta*f16_to_f32(y)) with
 * the truncating encode.  y is updated in place. */
void oracle_hgemv_ref(int trans, size_t m, size_t n, float alpha, const uint16_t *A, const uint16_t *x, float beta,
                      uint16_t *y) {
    size_t len = trans ? n : m;
    for (size_t o = 0; o < len; ++o) {
        float sum = 0.0f;
        if (!trans)
            for (size_t j = 0; j < n; ++j) sum += oracle_ref_f16_to_f32(A[o * n + j]) * oracle_ref_f16_to_f32(x[j]);
        else
            for (size_t i = 0; i < m; ++i) sum += oracle_ref_f16_to_f32(A[i * n + o]) * oracle_ref_f16_to_f32(x[i]);
        float cur = oracle_ref_f16_to_f32(y[o]);
        y[o] = oracle_ref_f32_to_f16(alpha * sum + beta * cur);
    }
}

/* The reference's reduction arithmetic: 32 lanes, lane t visits i = t,
 * t+32, ... accumulating in f32, then the shared-memory tree for stride 16,
 * 8, 4, 2, 1 adds slot t+stride into slot t (dot.rs:24-45; nrm2.rs and
 * asum.rs likewise; nrm2's sqrt is taken on the host in f32, nrm2.rs:69-70).
 * op: 0 dot, 1 sum of squares then sqrt, 2 sum of |x|. */
float oracle_sreduce_ref(int op, size_t n, const float *x, const float *y) {
    float lane[32];
    for (size_t t = 0; t < 32; ++t) {
        float acc = 0.0f;
        for (size_t i = t; i < n; i += 32) {
            float v = x[i];
            float term = op == 0 ? v * y[i] : op == 1 ? v * v : (v < 0.0f ? -v : v);
            acc += term;
        }
        lane[t] = acc;
    }
    for (size_t stride = 16; stride > 0; stride /= 2)
        for (size_t t = 0; t < stride; ++t) lane[t] += lane[t + stride];
    return op == 1 ? sqrtf(lane[0]) : lane[0];
}

/* The reference's ISAMAX (iamax.rs:16-61): per lane the first index of its
 * largest |x| (strict >, start value -1, index 0), then the tree keeps the
 * higher slot only when strictly greater.  With ties across lanes the
 * winner is decided by lane position, not by index. */
size_t oracle_isamax_ref(size_t n, const float *x) {
    float val[32];
    uint32_t idx[32];
    for (size_t t = 0; t < 32; ++t) {
        float bv = -1.0f;
        uint32_t bi = 0;
        for (size_t i = t; i < n; i += 32) {
            float v = x[i];
            float av = v < 0.0f ? -v : v;
            if (av > bv) {
                bv = av;
                bi = (uint32_t)i;
            }
        }
        val[t] = bv;
        idx[t] = bi;
    }
    for (size_t stride = 16; stride > 0; stride /= 2)
        for (size_t t = 0; t < stride; ++t)
            if (val[t + stride] > val[t]) {
                val[t] = val[t + stride];
                idx[t] = idx[t + stride];
            }
    return idx[0];
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

/* DGEMV N rows, the reference's f64 loop (gemv.rs:386-410), one row per
 * iteration across threads. */
void oracle_cpu_dgemv_n(size_t rows, size_t n, double alpha, const double *A, const double *x, double beta,
                        double *y) {
#pragma omp parallel for schedule(static)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        double s = 0.0;
        for (size_t j = 0; j < n; ++j) s += A[i * n + j] * x[j];
        y[i] = alpha * s + beta * y[i];
    }
}

/* HGEMV N rows with the reference's arithmetic (gemv.rs:553-577): x is
 * decoded once into xf (n floats), A row by row. */
void oracle_cpu_hgemv_n(size_t rows, size_t n, float alpha, const uint16_t *A, const uint16_t *x, float beta,
                        uint16_t *y, float *xf) {
    for (size_t j = 0; j < n; ++j) xf[j] = oracle_ref_f16_to_f32(x[j]);
#pragma omp parallel for schedule(static)
    for (long ii = 0; ii < (long)rows; ++ii) {
        size_t i = (size_t)ii;
        float s = 0.0f;
        for (size_t j = 0; j < n; ++j) s += oracle_ref_f16_to_f32(A[i * n + j]) * xf[j];
        y[i] = oracle_ref_f32_to_f16(alpha * s + beta * oracle_ref_f16_to_f32(y[i]));
    }
}

/* SDOT over all threads: per-thread f32 partial sums (the reference's
 * per-lane f32 accumulation, dot.rs:27-31), added at the end. */
float oracle_cpu_sdot(size_t n, const float *x, const float *y) {
    float acc = 0.0f;
#pragma omp parallel for schedule(static) reduction(+ : acc)
    for (long i = 0; i < (long)n; ++i) acc += x[i] * y[i];
    return acc;
}
