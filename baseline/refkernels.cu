// refkernels.cu -- the reference's own GPU kernels, restated in CUDA C so that
// they can run on the same B200 as a reported baseline (the reference is Rust
// compiled by cuda-oxide, whose toolchain is not available here).
//
// This is NOT part of the library: nothing in cublas-rs_b200 links or calls
// it.  bench.py times it beside the product kernels on the same resident
// buffers, and tests/test_refkernels.py checks it against the FP64
// oracle, so the numbers it gives are those of a working restatement.
//
// Each kernel keeps the reference's algorithm, launch geometry and summation
// order (one thread per output, `sum += a * b` over k in order):
//   sgemm/dgemm naive        crates/cublas-l3/src/sgemm.rs:31-57,  dgemm.rs:26-54
//   sgemm/dgemm tiled (16x16 shared tiles)
//                            crates/cublas-l3/src/sgemm.rs:62-127, dgemm.rs:56-125
//   sgemm/dgemm vectorized (32x32 block, 4 rows per thread, k-tile 16)
//                            crates/cublas-l3/src/sgemm.rs:135-235, dgemm.rs:127-234
//   sgemm/dgemm double_buf (two 16x16 buffers, one barrier per tile)
//                            crates/cublas-l3/src/sgemm.rs:243-340, dgemm.rs:236-334
//   hgemm_half (16x16 tiles of raw f16 bits, decoded at use; the reference's
//   flush-subnormals decode and truncating encode)
//                            crates/cublas-l3/src/hgemm.rs:20-125
//   strided_batched_sgemm (tiled, batch on grid z)
//                            crates/cublas-l3/src/batched.rs:25-102
//   sgemv naive (a thread per output) and tiled (a 32-thread block per output,
//   x staged in shared memory, shared-memory tree reduction)
//                            crates/cublas-l2/src/gemv.rs:29-223
//   dgemv / hgemv (naive; hgemv with the f16 conversions above)
//                            crates/cublas-l2/src/gemv.rs:387-440, 553-606
//   saxpy                    crates/cublas-l1/src/saxpy.rs:13-20
//   sdot / snrm2 (sum of squares; the host takes the root) / sasum / isamax:
//   one block of 32 threads, strided loop, shared-memory tree
//                            crates/cublas-l1/src/dot.rs:21-53, nrm2.rs:16-47,
//                            asum.rs:15-46, iamax.rs:16-60
// Differences, all in the restatement's favour or neutral: Rust's slice bounds
// checks are not repeated (every access the guards allow is in bounds), and
// indices are 64-bit.  `sum += a * b` is contracted to an fma by nvcc; whether
// cuda-oxide contracts it is not pinned by the reference.  The block size of
// cuda-oxide's LaunchConfig::for_num_elems (naive GEMV, saxpy) is not in the
// reference's sources: 256 is used.
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kTile = 16;
constexpr int kVecM = 32, kVecN = 32, kVecK = 16, kVecRows = 4;

template <typename T>
__global__ void gemm_naive(int m, int n, int k, T alpha, const T *__restrict__ a, const T *__restrict__ b, T beta,
                           T *__restrict__ c) {
    const size_t row = static_cast<size_t>(blockIdx.y) * blockDim.y + threadIdx.y;
    const size_t col = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (row >= static_cast<size_t>(m) || col >= static_cast<size_t>(n)) return;
    T sum = T(0);
    for (int i = 0; i < k; ++i) sum += a[row * k + i] * b[static_cast<size_t>(i) * n + col];
    c[row * n + col] = alpha * sum + beta * c[row * n + col];
}

template <typename T>
__global__ void gemm_tiled(int m, int n, int k, T alpha, const T *__restrict__ a, const T *__restrict__ b, T beta,
                           T *__restrict__ c) {
    __shared__ T ta[kTile * kTile], tb[kTile * kTile];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const size_t row = static_cast<size_t>(blockIdx.y) * kTile + ty;
    const size_t col = static_cast<size_t>(blockIdx.x) * kTile + tx;
    const int tiles = (k + kTile - 1) / kTile;
    T sum = T(0);
    for (int t = 0; t < tiles; ++t) {
        const int k0 = t * kTile;
        ta[ty * kTile + tx] = (row < static_cast<size_t>(m) && k0 + tx < k) ? a[row * k + k0 + tx] : T(0);
        tb[ty * kTile + tx] =
            (k0 + ty < k && col < static_cast<size_t>(n)) ? b[static_cast<size_t>(k0 + ty) * n + col] : T(0);
        __syncthreads();
        for (int i = 0; i < kTile; ++i) sum += ta[ty * kTile + i] * tb[i * kTile + tx];
        __syncthreads();
    }
    if (row < static_cast<size_t>(m) && col < static_cast<size_t>(n))
        c[row * n + col] = alpha * sum + beta * c[row * n + col];
}

template <typename T>
__global__ void gemm_vectorized(int m, int n, int k, T alpha, const T *__restrict__ a, const T *__restrict__ b,
                                T beta, T *__restrict__ c) {
    __shared__ T ta[kVecM * kVecK], tb[kVecK * kVecN];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const size_t brow = static_cast<size_t>(blockIdx.y) * kVecM, bcol = static_cast<size_t>(blockIdx.x) * kVecN;
    const int tid = ty * kVecN + tx;  // 0..255
    const int tiles = (k + kVecK - 1) / kVecK;
    T acc[kVecRows] = {};
    for (int t = 0; t < tiles; ++t) {
        const int k0 = t * kVecK;
        for (int idx = tid; idx < kVecM * kVecK; idx += 256) {  // A tile: 32 rows x 16 k
            const int r = idx / kVecK, kk = idx % kVecK;
            ta[idx] = (brow + r < static_cast<size_t>(m) && k0 + kk < k) ? a[(brow + r) * k + k0 + kk] : T(0);
        }
        for (int idx = tid; idx < kVecK * kVecN; idx += 256) {  // B tile: 16 k x 32 cols
            const int kk = idx / kVecN, cc = idx % kVecN;
            tb[idx] = (k0 + kk < k && bcol + cc < static_cast<size_t>(n)) ? b[static_cast<size_t>(k0 + kk) * n + bcol + cc]
                                                                         : T(0);
        }
        __syncthreads();
        for (int kk = 0; kk < kVecK; ++kk) {
            const T bv = tb[kk * kVecN + tx];
#pragma unroll
            for (int r = 0; r < kVecRows; ++r) acc[r] += ta[(ty * kVecRows + r) * kVecK + kk] * bv;
        }
        __syncthreads();
    }
    const size_t col = bcol + tx;
#pragma unroll
    for (int r = 0; r < kVecRows; ++r) {
        const size_t row = brow + static_cast<size_t>(ty) * kVecRows + r;
        if (row < static_cast<size_t>(m) && col < static_cast<size_t>(n))
            c[row * n + col] = alpha * acc[r] + beta * c[row * n + col];
    }
}

template <typename T>
__global__ void gemm_double_buf(int m, int n, int k, T alpha, const T *__restrict__ a, const T *__restrict__ b,
                                T beta, T *__restrict__ c) {
    __shared__ T ta[2 * kTile * kTile], tb[2 * kTile * kTile];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const size_t row = static_cast<size_t>(blockIdx.y) * kTile + ty;
    const size_t col = static_cast<size_t>(blockIdx.x) * kTile + tx;
    const int tiles = (k + kTile - 1) / kTile;
    if (tiles == 0) return;
    const int s = ty * kTile + tx;
    auto load = [&](int off, int k0) {
        ta[off + s] = (row < static_cast<size_t>(m) && k0 + tx < k) ? a[row * k + k0 + tx] : T(0);
        tb[off + s] = (k0 + ty < k && col < static_cast<size_t>(n)) ? b[static_cast<size_t>(k0 + ty) * n + col] : T(0);
    };
    load(0, 0);
    __syncthreads();
    T sum = T(0);
    int t = 0;
    for (; t + 1 < tiles; ++t) {
        const int cur = (t & 1) * kTile * kTile, nxt = ((t + 1) & 1) * kTile * kTile;
        load(nxt, (t + 1) * kTile);  // the buffer every thread finished reading before the last barrier
        for (int i = 0; i < kTile; ++i) sum += ta[cur + ty * kTile + i] * tb[cur + i * kTile + tx];
        __syncthreads();
    }
    const int last = (t & 1) * kTile * kTile;
    for (int i = 0; i < kTile; ++i) sum += ta[last + ty * kTile + i] * tb[last + i * kTile + tx];
    if (row < static_cast<size_t>(m) && col < static_cast<size_t>(n))
        c[row * n + col] = alpha * sum + beta * c[row * n + col];
}

// The reference's f16 conversions (hgemm.rs:20-51): subnormals decode to
// signed zero; encoding truncates the mantissa, flushes to signed zero below
// the normal range and saturates to infinity above it.
__device__ __forceinline__ float ref_f16_to_f32(uint16_t h) {
    const uint32_t x = h, sign = (x & 0x8000u) << 16, e = (x >> 10) & 0x1fu, man = x & 0x3ffu;
    if (e == 0) return __uint_as_float(sign);
    if (e == 31) return __uint_as_float(sign | (0xffu << 23) | (man << 13));
    return __uint_as_float(sign | ((e + 112u) << 23) | (man << 13));
}

__device__ __forceinline__ uint16_t ref_f32_to_f16(float f) {
    const uint32_t bits = __float_as_uint(f);
    const uint16_t sign = static_cast<uint16_t>((bits >> 16) & 0x8000u);
    const int e = static_cast<int>((bits >> 23) & 0xffu);
    const uint32_t man = bits & 0x7fffffu;
    if (e == 0xff) return sign | 0x7c00u | (man != 0 ? 1u : 0u);
    const int ne = e - 127 + 15;
    if (ne >= 31) return sign | 0x7c00u;
    if (ne <= 0) return sign;
    return sign | static_cast<uint16_t>(ne << 10) | static_cast<uint16_t>(man >> 13);
}

__global__ void hgemm_half(int m, int n, int k, float alpha, const uint16_t *__restrict__ a,
                           const uint16_t *__restrict__ b, float beta, uint16_t *__restrict__ c) {
    __shared__ uint16_t ta[kTile * kTile], tb[kTile * kTile];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const size_t row = static_cast<size_t>(blockIdx.y) * kTile + ty;
    const size_t col = static_cast<size_t>(blockIdx.x) * kTile + tx;
    const int tiles = (k + kTile - 1) / kTile;
    float sum = 0.0f;
    for (int t = 0; t < tiles; ++t) {
        const int k0 = t * kTile;
        ta[ty * kTile + tx] = (row < static_cast<size_t>(m) && k0 + tx < k) ? a[row * k + k0 + tx] : uint16_t(0);
        tb[ty * kTile + tx] =
            (k0 + ty < k && col < static_cast<size_t>(n)) ? b[static_cast<size_t>(k0 + ty) * n + col] : uint16_t(0);
        __syncthreads();
        for (int i = 0; i < kTile; ++i) sum += ref_f16_to_f32(ta[ty * kTile + i]) * ref_f16_to_f32(tb[i * kTile + tx]);
        __syncthreads();
    }
    if (row < static_cast<size_t>(m) && col < static_cast<size_t>(n)) {
        const float cur = ref_f16_to_f32(c[row * n + col]);
        c[row * n + col] = ref_f32_to_f16(alpha * sum + beta * cur);
    }
}

__global__ void sgemm_strided_batched(int m, int n, int k, float alpha, const float *__restrict__ a, int64_t sa,
                                      const float *__restrict__ b, int64_t sb, float beta, float *__restrict__ c,
                                      int64_t sc) {
    const size_t z = blockIdx.z;  // batch index; the tile loop is gemm_tiled's
    a += z * sa;
    b += z * sb;
    c += z * sc;
    __shared__ float ta[kTile * kTile], tb[kTile * kTile];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const size_t row = static_cast<size_t>(blockIdx.y) * kTile + ty;
    const size_t col = static_cast<size_t>(blockIdx.x) * kTile + tx;
    const int tiles = (k + kTile - 1) / kTile;
    float sum = 0.0f;
    for (int t = 0; t < tiles; ++t) {
        const int k0 = t * kTile;
        ta[ty * kTile + tx] = (row < static_cast<size_t>(m) && k0 + tx < k) ? a[row * k + k0 + tx] : 0.0f;
        tb[ty * kTile + tx] =
            (k0 + ty < k && col < static_cast<size_t>(n)) ? b[static_cast<size_t>(k0 + ty) * n + col] : 0.0f;
        __syncthreads();
        for (int i = 0; i < kTile; ++i) sum += ta[ty * kTile + i] * tb[i * kTile + tx];
        __syncthreads();
    }
    if (row < static_cast<size_t>(m) && col < static_cast<size_t>(n))
        c[row * n + col] = alpha * sum + beta * c[row * n + col];
}

template <typename T>
__global__ void gemv_naive(int trans, int m, int n, T alpha, const T *__restrict__ a, const T *__restrict__ x,
                           T beta, T *__restrict__ y) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    T sum = T(0);
    if (!trans) {  // y[i] = alpha * sum_j A[i][j] x[j] + beta y[i]
        if (i >= static_cast<size_t>(m)) return;
        for (int j = 0; j < n; ++j) sum += a[i * n + j] * x[j];
    } else {  // y[j] = alpha * sum_i A[i][j] x[i] + beta y[j]
        if (i >= static_cast<size_t>(n)) return;
        for (int r = 0; r < m; ++r) sum += a[static_cast<size_t>(r) * n + i] * x[r];
    }
    y[i] = alpha * sum + beta * y[i];
}

__global__ void hgemv_naive(int trans, int m, int n, float alpha, const uint16_t *__restrict__ a,
                            const uint16_t *__restrict__ x, float beta, uint16_t *__restrict__ y) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    float sum = 0.0f;
    if (!trans) {
        if (i >= static_cast<size_t>(m)) return;
        for (int j = 0; j < n; ++j) sum += ref_f16_to_f32(a[i * n + j]) * ref_f16_to_f32(x[j]);
    } else {
        if (i >= static_cast<size_t>(n)) return;
        for (int r = 0; r < m; ++r) sum += ref_f16_to_f32(a[static_cast<size_t>(r) * n + i]) * ref_f16_to_f32(x[r]);
    }
    y[i] = ref_f32_to_f16(alpha * sum + beta * ref_f16_to_f32(y[i]));
}

__global__ void sgemv_tiled(int trans, int m, int n, float alpha, const float *__restrict__ a,
                            const float *__restrict__ x, float beta, float *__restrict__ y) {
    __shared__ float sx[32], red[32];
    const int tid = threadIdx.x;
    const size_t out = blockIdx.x;
    const int len = trans ? m : n;  // length of x
    const int tiles = (len + 31) / 32;
    float acc = 0.0f;
    for (int t = 0; t < tiles; ++t) {
        const int j = t * 32 + tid;
        sx[tid] = j < len ? x[j] : 0.0f;
        __syncthreads();
        if (j < len) acc += (trans ? a[static_cast<size_t>(j) * n + out] : a[out * n + j]) * sx[tid];
        __syncthreads();
    }
    red[tid] = acc;
    __syncthreads();
    for (int s = 16; s > 0; s >>= 1) {
        if (tid < s) red[tid] += red[tid + s];
        __syncthreads();
    }
    if (tid == 0) y[out] = alpha * red[0] + beta * y[out];
}

__global__ void saxpy_kernel(int n, float alpha, const float *__restrict__ x, float *__restrict__ y) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < static_cast<size_t>(n)) y[i] = alpha * x[i] + y[i];
}

// OP 0: sum x*y, 1: sum x*x, 2: sum |x|.  Launched as one block of 32 threads.
template <int OP>
__global__ void sum32(int n, const float *__restrict__ x, const float *__restrict__ y, float *__restrict__ out) {
    __shared__ float sd[32];
    const int tid = threadIdx.x;
    float acc = 0.0f;
    for (size_t i = tid; i < static_cast<size_t>(n); i += 32) {
        const float v = x[i];
        acc += OP == 0 ? v * y[i] : OP == 1 ? v * v : (v < 0.0f ? -v : v);
    }
    sd[tid] = acc;
    __syncthreads();
    for (int s = 16; s > 0; s >>= 1) {
        if (tid < s) sd[tid] += sd[tid + s];
        __syncthreads();
    }
    if (tid == 0) out[0] = sd[0];
}

// First index of the largest |x| per lane, then a tree that takes the other
// half's entry only when strictly larger (0-based, as the kernel returns it).
__global__ void isamax32(int n, const float *__restrict__ x, uint32_t *__restrict__ out) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    const int tid = threadIdx.x;
    float best = -1.0f;
    uint32_t bi = 0;
    for (size_t i = tid; i < static_cast<size_t>(n); i += 32) {
        const float v = x[i];
        const float av = v < 0.0f ? -v : v;
        if (av > best) {
            best = av;
            bi = static_cast<uint32_t>(i);
        }
    }
    sv[tid] = best;
    si[tid] = bi;
    __syncthreads();
    for (int s = 16; s > 0; s >>= 1) {
        if (tid < s && sv[tid + s] > sv[tid]) {
            sv[tid] = sv[tid + s];
            si[tid] = si[tid + s];
        }
        __syncthreads();
    }
    if (tid == 0) out[0] = si[0];
}

template <typename T>
int launch_gemm(int variant, int m, int n, int k, T alpha, const T *a, const T *b, T beta, T *c, cudaStream_t st) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    switch (variant) {
        case 0:
            gemm_naive<T><<<dim3((n + 15) / 16, (m + 15) / 16), dim3(16, 16), 0, st>>>(m, n, k, alpha, a, b, beta, c);
            break;
        case 1:
            gemm_tiled<T><<<dim3((n + 15) / 16, (m + 15) / 16), dim3(16, 16), 0, st>>>(m, n, k, alpha, a, b, beta, c);
            break;
        case 2:
            gemm_vectorized<T><<<dim3((n + kVecN - 1) / kVecN, (m + kVecM - 1) / kVecM), dim3(kVecN, kVecM / kVecRows),
                                 0, st>>>(m, n, k, alpha, a, b, beta, c);
            break;
        case 3:
            gemm_double_buf<T><<<dim3((n + 15) / 16, (m + 15) / 16), dim3(16, 16), 0, st>>>(m, n, k, alpha, a, b, beta,
                                                                                            c);
            break;
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" {

// variant: 0 naive, 1 tiled, 2 vectorized, 3 double_buf.  Returns a cudaError_t.
__attribute__((visibility("default"))) int refk_sgemm(int variant, int m, int n, int k, float alpha, const float *a,
                                                      const float *b, float beta, float *c, void *stream) {
    return launch_gemm<float>(variant, m, n, k, alpha, a, b, beta, c, static_cast<cudaStream_t>(stream));
}

__attribute__((visibility("default"))) int refk_dgemm(int variant, int m, int n, int k, double alpha, const double *a,
                                                      const double *b, double beta, double *c, void *stream) {
    return launch_gemm<double>(variant, m, n, k, alpha, a, b, beta, c, static_cast<cudaStream_t>(stream));
}

__attribute__((visibility("default"))) int refk_hgemm_half(int m, int n, int k, float alpha, const uint16_t *a,
                                                           const uint16_t *b, float beta, uint16_t *c, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    hgemm_half<<<dim3((n + 15) / 16, (m + 15) / 16), dim3(16, 16), 0, static_cast<cudaStream_t>(stream)>>>(
        m, n, k, alpha, a, b, beta, c);
    return static_cast<int>(cudaGetLastError());
}

__attribute__((visibility("default"))) int refk_sgemm_strided_batched(int m, int n, int k, float alpha,
                                                                      const float *a, int64_t sa, const float *b,
                                                                      int64_t sb, float beta, float *c, int64_t sc,
                                                                      int batch, void *stream) {
    if (m <= 0 || n <= 0 || k <= 0 || batch <= 0) return 0;
    if (batch > 65535) return static_cast<int>(cudaErrorInvalidValue);  // grid z, as the reference launches it
    sgemm_strided_batched<<<dim3((n + 15) / 16, (m + 15) / 16, batch), dim3(16, 16), 0,
                            static_cast<cudaStream_t>(stream)>>>(m, n, k, alpha, a, sa, b, sb, beta, c, sc);
    return static_cast<int>(cudaGetLastError());
}

// variant: 0 naive, 1 tiled; trans: 0 y = A x (x has n entries), 1 y = A^T x (x has m).
__attribute__((visibility("default"))) int refk_sgemv(int variant, int trans, int m, int n, float alpha,
                                                      const float *a, const float *x, float beta, float *y,
                                                      void *stream) {
    if (m <= 0 || n <= 0) return 0;
    const int outs = trans ? n : m;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (variant == 0)
        gemv_naive<float><<<(outs + 255) / 256, 256, 0, st>>>(trans, m, n, alpha, a, x, beta, y);
    else if (variant == 1)
        sgemv_tiled<<<outs, 32, 0, st>>>(trans, m, n, alpha, a, x, beta, y);
    else
        return static_cast<int>(cudaErrorInvalidValue);
    return static_cast<int>(cudaGetLastError());
}

__attribute__((visibility("default"))) int refk_dgemv(int trans, int m, int n, double alpha, const double *a,
                                                      const double *x, double beta, double *y, void *stream) {
    if (m <= 0 || n <= 0) return 0;
    const int outs = trans ? n : m;
    gemv_naive<double><<<(outs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(trans, m, n, alpha, a, x,
                                                                                          beta, y);
    return static_cast<int>(cudaGetLastError());
}

__attribute__((visibility("default"))) int refk_hgemv(int trans, int m, int n, float alpha, const uint16_t *a,
                                                      const uint16_t *x, float beta, uint16_t *y, void *stream) {
    if (m <= 0 || n <= 0) return 0;
    const int outs = trans ? n : m;
    hgemv_naive<<<(outs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(trans, m, n, alpha, a, x, beta,
                                                                                   y);
    return static_cast<int>(cudaGetLastError());
}

// op: 0 sdot (float out), 1 snrm2's sum of squares (float out; the host takes
// the square root), 2 sasum (float out), 3 isamax (uint32 out, 0-based).
__attribute__((visibility("default"))) int refk_sreduce(int op, int n, const float *x, const float *y, void *out,
                                                        void *stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n <= 0) return static_cast<int>(cudaMemsetAsync(out, 0, 4, st));
    switch (op) {
        case 0: sum32<0><<<1, 32, 0, st>>>(n, x, y, static_cast<float *>(out)); break;
        case 1: sum32<1><<<1, 32, 0, st>>>(n, x, nullptr, static_cast<float *>(out)); break;
        case 2: sum32<2><<<1, 32, 0, st>>>(n, x, nullptr, static_cast<float *>(out)); break;
        case 3: isamax32<<<1, 32, 0, st>>>(n, x, static_cast<uint32_t *>(out)); break;
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
    return static_cast<int>(cudaGetLastError());
}

__attribute__((visibility("default"))) int refk_saxpy(int n, float alpha, const float *x, float *y, void *stream) {
    if (n <= 0) return 0;
    saxpy_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(n, alpha, x, y);
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
