// gemv.cu -- SGEMV for sm_100a: y <- alpha * op(A) * x + beta * y, A m x n
// row-major, op(A) = A (N) or A^T (T), the operation of cublas-rs's
// sgemv_n / sgemv_t / sgemv_n_tiled / sgemv_t_tiled
// (crates/cublas-l2/src/gemv.rs:29-223).
//
// SGEMV reads every element of A once, so it is bound by HBM bandwidth; the
// kernels are built to keep enough 16-byte loads in flight:
//   * N: S warps per row (S = 1..8, rows cut into ~16 KiB segments); each
//     lane streams 16-byte vectors of its segment with
//     ld.global.nc.L1::no_allocate (A is touched once, keep it out of L1),
//     UNROLL vectors in flight per lane, while x is read through L1 (it is
//     shared by every row); warp-shuffle reduction, the S partials added in
//     segment order through shared memory.
//   * T: the rows are split into S slices; CTA (column block, slice) walks
//     its slice with each lane owning 4 consecutive columns (16-byte loads
//     across the row, coalesced), reduces its 8 warps through shared memory
//     and writes one partial row.  A second kernel sums the S partials in a
//     fixed order (deterministic) and applies alpha/beta.  S is chosen so
//     that about 4 CTAs per SM are in flight.  The partials live in the
//     handle's workspace (S * n floats).
// beta == 0 does not read y.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "internal.h"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float ld_stream1(const float *p) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// N: S warps share a row, warp s summing the s-th of S contiguous column
// segments; the S partials meet in shared memory and are added in segment
// order (deterministic).  Long rows split this way give the grid more,
// shorter work units: a warp streaming one 64-128 KiB row alone holds the
// GPU's last wave open.
template <int UNROLL, bool VEC, int S>
__global__ void __launch_bounds__(kThreads) sgemv_n_kernel(const float *__restrict__ A, const float *__restrict__ x,
                                                           float *__restrict__ y, int64_t m, int64_t n, float alpha,
                                                           float beta) {
    static_assert(kWarps % S == 0, "segments per row divide the CTA's warps");
    __shared__ float part[kWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (kWarps / S) + warp / S;
    const int seg = warp % S;
    float acc = 0.0f;
    if (row < m) {
        if constexpr (VEC) {
            const float4 *a = reinterpret_cast<const float4 *>(A + row * n);
            const float4 *xv = reinterpret_cast<const float4 *>(x);
            const int64_t nv = n >> 2;
            const int64_t seg_len = (nv + S - 1) / S;
            const int64_t v0 = seg * seg_len, v1 = v0 + seg_len < nv ? v0 + seg_len : nv;
            int64_t j = v0 + lane;
            // Full groups: UNROLL independent 16-byte loads per lane in flight.
            for (; j + 32 * (UNROLL - 1) < v1; j += 32 * UNROLL) {
                float4 av[UNROLL], xx[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) av[u] = ld_stream(a + j + 32 * u);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) xx[u] = __ldg(xv + j + 32 * u);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    acc = fmaf(av[u].x, xx[u].x, acc);
                    acc = fmaf(av[u].y, xx[u].y, acc);
                    acc = fmaf(av[u].z, xx[u].z, acc);
                    acc = fmaf(av[u].w, xx[u].w, acc);
                }
            }
            for (; j < v1; j += 32) {
                float4 av = ld_stream(a + j), xx = __ldg(xv + j);
                acc = fmaf(av.x, xx.x, acc);
                acc = fmaf(av.y, xx.y, acc);
                acc = fmaf(av.z, xx.z, acc);
                acc = fmaf(av.w, xx.w, acc);
            }
        } else {
            const float *a = A + row * n;
            const int64_t seg_len = (n + S - 1) / S;
            const int64_t c0 = seg * seg_len, c1 = c0 + seg_len < n ? c0 + seg_len : n;
            for (int64_t j = c0 + lane; j < c1; j += 32) acc = fmaf(ld_stream1(a + j), __ldg(x + j), acc);
        }
        acc = warp_sum(acc);
    }
    if constexpr (S > 1) {
        if (lane == 0) part[warp] = acc;
        __syncthreads();
        if (seg == 0 && lane == 0 && row < m) {
            float t = part[warp];
#pragma unroll
            for (int q = 1; q < S; ++q) t += part[warp + q];
            acc = t;
        }
    }
    if (seg == 0 && lane == 0 && row < m) {
        float v = alpha * acc;
        if (beta != 0.0f) v = fmaf(beta, y[row], v);
        y[row] = v;
    }
}

// Segments per row for the N kernels: rows of `row_bytes` are cut into
// pieces of about `seg_bytes` (a power of two count, at most 8).
inline int gemv_segments(int64_t row_bytes, int64_t seg_bytes) {
    int S = 1;
    while (S < 8 && row_bytes >= 2 * S * seg_bytes) S *= 2;
    return S;
}

template <bool VEC>
cudaError_t launch_sgemv_n_vec(b2b_handle *h, const float *A, const float *x, float *y, int64_t m, int64_t n,
                               float alpha, float beta, int S) {
    const int64_t rows_per_cta = kWarps / S;
    const unsigned blocks = static_cast<unsigned>((m + rows_per_cta - 1) / rows_per_cta);
    switch (S) {
        case 1: sgemv_n_kernel<8, VEC, 1><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        case 2: sgemv_n_kernel<8, VEC, 2><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        case 4: sgemv_n_kernel<8, VEC, 4><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        default: sgemv_n_kernel<8, VEC, 8><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
    }
    return cudaGetLastError();
}

// The N launch shared by b2b_sgemv and b2b_sgemv_noalloc.
int launch_sgemv_n(b2b_handle *h, const float *A, const float *x, float *y, int64_t m, int64_t n, float alpha,
                   float beta) {
    const bool vec = (n % 4 == 0) && b2b::aligned16(A) && b2b::aligned16(x);
    const int S = gemv_segments(n * 4, h->gemv_seg_bytes);
    if ((m + kWarps / S - 1) / (kWarps / S) > 0x7fffffffLL) return b2b::fail(B2B_ERR_INVALID_ARG, "sgemv: m too large");
    const cudaError_t e = vec ? launch_sgemv_n_vec<true>(h, A, x, y, m, n, alpha, beta, S)
                              : launch_sgemv_n_vec<false>(h, A, x, y, m, n, alpha, beta, S);
    return e == cudaSuccess ? B2B_OK : b2b::fail_cuda(e, "sgemv N launch");
}

// T, pass 1: CTA (blockIdx.x = column block of 128, blockIdx.y = row slice).
// Lane l of every warp owns columns cb*128 + 4l .. +3 (VEC) or
// cb*128 + l + 32e, e = 0..3 (scalar).  Warp w takes rows r0+w, r0+w+8, ...
// Writes partial[slice][col] (direct=false) or y (direct=true, one slice).
template <bool VEC, bool DIRECT>
__global__ void __launch_bounds__(kThreads) sgemv_t_partial_kernel(const float *__restrict__ A,
                                                                   const float *__restrict__ x,
                                                                   float *__restrict__ out, int64_t m, int64_t n,
                                                                   int64_t rows_per_slice, float alpha, float beta) {
    __shared__ float red[kWarps][128];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 128;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_slice;
    const int64_t r1 = r0 + rows_per_slice < m ? r0 + rows_per_slice : m;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (VEC) {
        const int64_t c = c0 + lane * 4;
        if (c < n) {  // n % 4 == 0, so the whole vector is in range
            int64_t r = r0 + warp;
            for (; r + 3 * kWarps < r1; r += 4 * kWarps) {
                float4 v[4];
                float xs[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = ld_stream(reinterpret_cast<const float4 *>(A + (r + u * kWarps) * n + c));
#pragma unroll
                for (int u = 0; u < 4; ++u) xs[u] = __ldg(x + r + u * kWarps);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    acc[0] = fmaf(v[u].x, xs[u], acc[0]);
                    acc[1] = fmaf(v[u].y, xs[u], acc[1]);
                    acc[2] = fmaf(v[u].z, xs[u], acc[2]);
                    acc[3] = fmaf(v[u].w, xs[u], acc[3]);
                }
            }
            for (; r < r1; r += kWarps) {
                float4 v = ld_stream(reinterpret_cast<const float4 *>(A + r * n + c));
                float xs = __ldg(x + r);
                acc[0] = fmaf(v.x, xs, acc[0]);
                acc[1] = fmaf(v.y, xs, acc[1]);
                acc[2] = fmaf(v.z, xs, acc[2]);
                acc[3] = fmaf(v.w, xs, acc[3]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][lane * 4 + e] = acc[e];
    } else {
        for (int64_t r = r0 + warp; r < r1; r += kWarps) {
            const float xs = __ldg(x + r);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int64_t c = c0 + lane + 32 * e;
                if (c < n) acc[e] = fmaf(ld_stream1(A + r * n + c), xs, acc[e]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][lane + 32 * e] = acc[e];
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        const int64_t c = c0 + threadIdx.x;
        if (c < n) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += red[w][threadIdx.x];
            if constexpr (DIRECT) {
                float v = alpha * s;
                if (beta != 0.0f) v = fmaf(beta, out[c], v);
                out[c] = v;
            } else {
                out[static_cast<int64_t>(blockIdx.y) * n + c] = s;
            }
        }
    }
}

// T, pass 2: y[j] = alpha * sum_s partial[s][j] + beta * y[j], s in order.
__global__ void sgemv_t_reduce_kernel(const float *__restrict__ partial, float *__restrict__ y, int64_t n,
                                      int slices, float alpha, float beta) {
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float s = 0.0f;
    for (int i = 0; i < slices; ++i) s += partial[static_cast<int64_t>(i) * n + j];
    float v = alpha * s;
    if (beta != 0.0f) v = fmaf(beta, y[j], v);
    y[j] = v;
}

// Split-row plan of the transposed SGEMV, shared by b2b_sgemv and
// b2b_sgemv_noalloc so both give the same bits: enough slices for ~4 CTAs per
// SM, each slice at least 64 rows, at most 65535 slices.
struct TSlicing {
    int64_t col_blocks, slices, rows_per;
};

TSlicing sgemv_t_slicing(int sm_count, int64_t m, int64_t n) {
    TSlicing p;
    p.col_blocks = (n + 127) / 128;
    const int64_t target = 4LL * sm_count;
    int64_t slices = (target + p.col_blocks - 1) / p.col_blocks;
    const int64_t max_slices = (m + 63) / 64;
    if (slices > max_slices) slices = max_slices;
    if (slices > 65535) slices = 65535;
    if (slices < 1) slices = 1;
    p.rows_per = (m + slices - 1) / slices;
    p.slices = (m + p.rows_per - 1) / p.rows_per;
    return p;
}

}  // namespace

namespace b2b {

int launch_sgemv(b2b_handle *h, int trans, size_t m_, size_t n_, float alpha, const float *A, const float *x,
                 float beta, float *y) {
    const int64_t m = static_cast<int64_t>(m_), n = static_cast<int64_t>(n_);
    cudaError_t e;
    if (trans == B2B_OP_N) return launch_sgemv_n(h, A, x, y, m, n, alpha, beta);
    const bool vec_t = (n % 4 == 0) && aligned16(A);
    const TSlicing plan = sgemv_t_slicing(h->sm_count, m, n);
    const int64_t col_blocks = plan.col_blocks, slices = plan.slices, rows_per = plan.rows_per;
    if (col_blocks > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "sgemv: n too large");
    if (slices == 1) {
        dim3 grid((unsigned)col_blocks, 1);
        if (vec_t)
            sgemv_t_partial_kernel<true, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        else
            sgemv_t_partial_kernel<false, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "sgemv T launch");
        return B2B_OK;
    }
    void *ws = nullptr;
    int rc = workspace(h, static_cast<size_t>(slices) * static_cast<size_t>(n) * sizeof(float), &ws);
    if (rc) return rc;
    float *partial = static_cast<float *>(ws);
    dim3 grid((unsigned)col_blocks, (unsigned)slices);
    if (vec_t)
        sgemv_t_partial_kernel<true, false><<<grid, kThreads, 0, h->stream>>>(A, x, partial, m, n, rows_per, alpha, beta);
    else
        sgemv_t_partial_kernel<false, false><<<grid, kThreads, 0, h->stream>>>(A, x, partial, m, n, rows_per, alpha, beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgemv T partial launch");
    const int64_t rblocks = (n + 255) / 256;
    sgemv_t_reduce_kernel<<<(unsigned)rblocks, 256, 0, h->stream>>>(partial, y, n, (int)slices, alpha, beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgemv T reduce launch");
    return B2B_OK;
}

}  // namespace b2b

// ---------------------------------------------------------------------------
// b2b_sgemv_noalloc: SGEMV whose split-row partials live in a fixed device
// array instead of handle workspace, for callers that must not allocate
// device memory (see the declaration in b2blas.h).
//
// The array below is file-scope device memory of kNoAllocScratchFloats
// floats (1 MiB); every GPU that loads this library holds it until the
// process exits.  Every call shares it and it keeps the last call's
// contents.  Nothing in it has to start at zero: pass 1 writes every
// (slice, column) partial before pass 2 reads it.  Calls that overlap on the
// GPU (two streams, or two handles, at once) race on it.
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 18;
static __device__ __align__(256) float g_sgemv_noalloc_scratch[kNoAllocScratchFloats];

// Host code cannot use the array's name as a device address, so the address
// is looked up once per device (with that device current) and cached, keyed
// by the context's unique id as well: after cudaDeviceReset the device gets
// a new context, in which the array may sit elsewhere, and the next call
// looks the address up again instead of using the old one.
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlot {
    unsigned long long ctx_id;
    float *ptr;
};
NoAllocSlot g_noalloc[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

using PfnCtxGetCurrent = CUresult (*)(CUcontext *);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long *);

// The unique id of the current context (cuCtxGetId, never reused within a
// process), through the runtime's driver entry points.
int current_context_id(unsigned long long *id) {
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    if (!get_current || !get_id) {
        void *p1 = nullptr, *p2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p1, 4000, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess ||
            cudaGetDriverEntryPointByVersion("cuCtxGetId", &p2, 12000, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess)
            return b2b::fail(B2B_ERR_CUDA, "b2b_sgemv_noalloc: cuCtxGetCurrent / cuCtxGetId not available");
        get_current = reinterpret_cast<PfnCtxGetCurrent>(p1);
        get_id = reinterpret_cast<PfnCtxGetId>(p2);
    }
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, id) != CUDA_SUCCESS)
        return b2b::fail(B2B_ERR_CUDA, "b2b_sgemv_noalloc: no current CUDA context");
    return B2B_OK;
}

// Call with the handle's device current (DeviceGuard).
int noalloc_scratch(int device, float **out) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return b2b::fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: device ordinal out of range");
    unsigned long long ctx_id = 0;
    if (int rc = current_context_id(&ctx_id)) return rc;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocSlot &slot = g_noalloc[device];
    if (!slot.ptr || slot.ctx_id != ctx_id) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_sgemv_noalloc_scratch);
        if (e != cudaSuccess) return b2b::fail_cuda(e, "b2b_sgemv_noalloc: cudaGetSymbolAddress");
        slot.ptr = static_cast<float *>(p);
        slot.ctx_id = ctx_id;
    }
    *out = slot.ptr;
    return B2B_OK;
}

}  // namespace

extern "C" int b2b_sgemv_noalloc(b2b_handle *h, int trans, size_t m_, size_t n_, float alpha, const float *A,
                                 const float *x, float beta, float *y) {
    using namespace b2b;
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: NULL handle");
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: trans must be B2B_OP_N or B2B_OP_T");
    if (m_ == 0 || n_ == 0) return B2B_OK;
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: NULL operand");
    if (m_ > (size_t(1) << 62) / n_) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: sizes overflow");
    DeviceGuard g(h);
    const int64_t m = static_cast<int64_t>(m_), n = static_cast<int64_t>(n_);
    cudaError_t e;
    if (trans == B2B_OP_N) return launch_sgemv_n(h, A, x, y, m, n, alpha, beta);  // needs no scratch
    // T: the same slicing as b2b_sgemv, so both give the same bits.
    const bool vec_t = (n % 4 == 0) && aligned16(A);
    const TSlicing plan = sgemv_t_slicing(h->sm_count, m, n);
    const int64_t col_blocks = plan.col_blocks, slices = plan.slices, rows_per = plan.rows_per;
    if (col_blocks > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: n too large");
    if (slices == 1) {
        dim3 grid((unsigned)col_blocks, 1);
        if (vec_t)
            sgemv_t_partial_kernel<true, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        else
            sgemv_t_partial_kernel<false, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        e = cudaGetLastError();
        return e == cudaSuccess ? B2B_OK : fail_cuda(e, "b2b_sgemv_noalloc: T launch");
    }
    // The limit is the array's size, or a lower one the handle was created
    // with (B2B_NOALLOC_SCRATCH_FLOATS; lets tests reach this rejection,
    // which no shape reaches on a 148-SM GPU: slices x n stays below
    // 4 * 148 * 128 + n <= 151,424 floats whenever slices > 1).
    const size_t limit = (h->noalloc_limit_floats > 0 && h->noalloc_limit_floats < kNoAllocScratchFloats)
                             ? h->noalloc_limit_floats
                             : kNoAllocScratchFloats;
    if (static_cast<uint64_t>(slices) * static_cast<uint64_t>(n) > limit)
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv_noalloc: this shape needs " + std::to_string(slices) + " x " +
                                             std::to_string(n) + " partial sums, more than the " +
                                             std::to_string(limit) + "-float fixed scratch holds; use b2b_sgemv");
    float *partial = nullptr;
    if (int rc = noalloc_scratch(h->device, &partial)) return rc;
    dim3 grid((unsigned)col_blocks, (unsigned)slices);
    if (vec_t)
        sgemv_t_partial_kernel<true, false><<<grid, kThreads, 0, h->stream>>>(A, x, partial, m, n, rows_per, alpha, beta);
    else
        sgemv_t_partial_kernel<false, false><<<grid, kThreads, 0, h->stream>>>(A, x, partial, m, n, rows_per, alpha, beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "b2b_sgemv_noalloc: T partial launch");
    sgemv_t_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, h->stream>>>(partial, y, n, (int)slices, alpha, beta);
    e = cudaGetLastError();
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "b2b_sgemv_noalloc: T reduce launch");
}
