// level1_reduce.cu -- SDOT, SNRM2, SASUM, ISAMAX over f32 vectors.
//
// The reference runs each of these as one 32-thread block
// (crates/cublas-l1/src/dot.rs:21-53, nrm2.rs:16-48, asum.rs:15-47,
// iamax.rs:16-61), which reads at a few GB/s.  Here one launch streams the
// vector over the whole GPU:
//   * grid = min(ceil(n / 4096), the CTAs resident at once), 256 threads
//     (one wave, no partial second one); each thread
//     grid-strides over 16-byte vectors (ld.global.nc.L1::no_allocate, eight
//     in flight per thread) and keeps its sums in f64 -- a product of two f32
//     values is exact in f64, so the only rounding left that matters is the
//     final f64 -> f32 one;
//   * warp shuffle, then shared memory, reduces the block to one partial,
//     written to the handle workspace;
//   * the last block to finish (a ticket from atomicAdd on a counter in the
//     handle's status block; nothing waits) adds the partials in block order
//     and writes the result.  Every partial covers a fixed set of indices and
//     the final sum has a fixed order, so results are bitwise repeatable for a
//     given n and GPU.
// SNRM2 is sqrt of the f64 sum of squares, so it neither overflows nor
// underflows for any finite f32 input (the reference squares in f32,
// nrm2.rs:24-27).  ISAMAX returns the smallest index of the largest |x|,
// skips NaN as the reference's comparisons do (iamax.rs:26-31), and returns 0
// when no element compares (all NaN).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct Partial {
    double v;   // sum, or the max |x| for ISAMAX (as f64)
    int64_t i;  // ISAMAX index
};

__device__ __forceinline__ float4 ld_stream4(const float *p) {
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

// element contribution for the summing ops
template <int OP>
__device__ __forceinline__ double term(float a, float b) {
    if constexpr (OP == B2B_REDUCE_DOT) return (double)a * (double)b;
    else if constexpr (OP == B2B_REDUCE_NRM2) return (double)a * (double)a;
    else return fabs((double)a);
}

// ISAMAX combine: larger |x| wins, ties go to the smaller index.  NaN never
// wins a comparison, so it is skipped.
__device__ __forceinline__ void amax_take(float &bv, int64_t &bi, float v, int64_t i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

template <int OP>
__device__ __forceinline__ void block_finish(double s, float bv, int64_t bi, Partial *red, Partial *out_slot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if constexpr (OP == B2B_REDUCE_IAMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            amax_take(bv, bi, ov, oi);
        }
        if (lane == 0) red[warp] = Partial{(double)bv, bi};
        __syncthreads();
        if (warp == 0) {
            bv = lane < kWarps ? (float)red[lane].v : -1.0f;
            bi = lane < kWarps ? red[lane].i : INT64_MAX;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                amax_take(bv, bi, ov, oi);
            }
            if (lane == 0) *out_slot = Partial{(double)bv, bi};
        }
    } else {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[warp].v = s;
        __syncthreads();
        if (warp == 0) {
            s = lane < kWarps ? red[lane].v : 0.0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) *out_slot = Partial{s, 0};
        }
    }
}

template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads) sreduce_kernel(const float *__restrict__ x, const float *__restrict__ y,
                                                           int64_t n, Partial *__restrict__ partial,
                                                           unsigned int *__restrict__ counter, void *__restrict__ out) {
    __shared__ Partial red[kWarps];
    __shared__ Partial block_part;
    __shared__ bool is_last;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;

    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    float bv = -1.0f;
    int64_t bi = INT64_MAX;

    if constexpr (VEC) {
        const int64_t n4 = n >> 2;
        int64_t j = tid;
        // eight 16-byte loads in flight per thread (four per operand for DOT)
        constexpr int U = (OP == B2B_REDUCE_DOT) ? 4 : 8;
        for (; j + (U - 1) * stride < n4; j += U * stride) {
            float4 a[U], b[U];
#pragma unroll
            for (int u = 0; u < U; ++u) a[u] = ld_stream4(x + 4 * (j + u * stride));
            if constexpr (OP == B2B_REDUCE_DOT) {
#pragma unroll
                for (int u = 0; u < U; ++u) b[u] = ld_stream4(y + 4 * (j + u * stride));
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if constexpr (OP == B2B_REDUCE_IAMAX) {
                    const int64_t base = 4 * (j + u * stride);
                    amax_take(bv, bi, fabsf(a[u].x), base);
                    amax_take(bv, bi, fabsf(a[u].y), base + 1);
                    amax_take(bv, bi, fabsf(a[u].z), base + 2);
                    amax_take(bv, bi, fabsf(a[u].w), base + 3);
                } else {
                    const float4 bb = (OP == B2B_REDUCE_DOT) ? b[u] : a[u];
                    s0 += term<OP>(a[u].x, bb.x);
                    s1 += term<OP>(a[u].y, bb.y);
                    s2 += term<OP>(a[u].z, bb.z);
                    s3 += term<OP>(a[u].w, bb.w);
                }
            }
        }
        for (; j < n4; j += stride) {
            const float4 a = ld_stream4(x + 4 * j);
            if constexpr (OP == B2B_REDUCE_IAMAX) {
                amax_take(bv, bi, fabsf(a.x), 4 * j);
                amax_take(bv, bi, fabsf(a.y), 4 * j + 1);
                amax_take(bv, bi, fabsf(a.z), 4 * j + 2);
                amax_take(bv, bi, fabsf(a.w), 4 * j + 3);
            } else {
                const float4 b = (OP == B2B_REDUCE_DOT) ? ld_stream4(y + 4 * j) : a;
                s0 += term<OP>(a.x, b.x);
                s1 += term<OP>(a.y, b.y);
                s2 += term<OP>(a.z, b.z);
                s3 += term<OP>(a.w, b.w);
            }
        }
        // the n % 4 tail
        const int64_t t = 4 * n4 + tid;
        if (t < n) {
            const float a = ld_stream1(x + t);
            if constexpr (OP == B2B_REDUCE_IAMAX) amax_take(bv, bi, fabsf(a), t);
            else s0 += term<OP>(a, (OP == B2B_REDUCE_DOT) ? ld_stream1(y + t) : a);
        }
    } else {
        int64_t j = tid;
        for (; j + 3 * stride < n; j += 4 * stride) {
            float a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = ld_stream1(x + j + u * stride);
            if constexpr (OP == B2B_REDUCE_DOT) {
#pragma unroll
                for (int u = 0; u < 4; ++u) b[u] = ld_stream1(y + j + u * stride);
            }
            if constexpr (OP == B2B_REDUCE_IAMAX) {
#pragma unroll
                for (int u = 0; u < 4; ++u) amax_take(bv, bi, fabsf(a[u]), j + u * stride);
            } else {
                s0 += term<OP>(a[0], (OP == B2B_REDUCE_DOT) ? b[0] : a[0]);
                s1 += term<OP>(a[1], (OP == B2B_REDUCE_DOT) ? b[1] : a[1]);
                s2 += term<OP>(a[2], (OP == B2B_REDUCE_DOT) ? b[2] : a[2]);
                s3 += term<OP>(a[3], (OP == B2B_REDUCE_DOT) ? b[3] : a[3]);
            }
        }
        for (; j < n; j += stride) {
            const float a = ld_stream1(x + j);
            if constexpr (OP == B2B_REDUCE_IAMAX) amax_take(bv, bi, fabsf(a), j);
            else s0 += term<OP>(a, (OP == B2B_REDUCE_DOT) ? ld_stream1(y + j) : a);
        }
    }

    block_finish<OP>((s0 + s1) + (s2 + s3), bv, bi, red, &block_part);
    if (threadIdx.x == 0) {
        partial[blockIdx.x] = block_part;
        __threadfence();  // the partial is visible device-wide before the ticket
        const unsigned int ticket = atomicAdd(counter, 1u);
        is_last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last) return;

    // Last block: every other block's partial was published before its
    // ticket.  Add them in block order (fixed, so the result repeats).
    __threadfence();
    s0 = 0.0;
    bv = -1.0f;
    bi = INT64_MAX;
    for (unsigned int b = threadIdx.x; b < gridDim.x; b += kThreads) {
        // .cg loads read L2, where the other blocks' partials landed.
        const double pv = __ldcg(&partial[b].v);
        if constexpr (OP == B2B_REDUCE_IAMAX)
            amax_take(bv, bi, (float)pv, (int64_t)__ldcg(reinterpret_cast<const long long *>(&partial[b].i)));
        else
            s0 += pv;
    }
    block_finish<OP>(s0, bv, bi, red, &block_part);
    if (threadIdx.x == 0) {
        const Partial r = block_part;
        if constexpr (OP == B2B_REDUCE_IAMAX) {
            *static_cast<uint64_t *>(out) = (r.v < 0.0 || r.i == INT64_MAX) ? 0ull : (uint64_t)r.i;
        } else if constexpr (OP == B2B_REDUCE_NRM2) {
            *static_cast<float *>(out) = (float)sqrt(r.v);
        } else {
            *static_cast<float *>(out) = (float)r.v;
        }
        *counter = 0u;  // ready for the next reduction on this handle
    }
}

template <int OP>
int launch_op(b2b_handle *h, int64_t n, const float *x, const float *y, void *out) {
    const bool vec = b2b::aligned16(x) && (OP != B2B_REDUCE_DOT || b2b::aligned16(y));
    // one resident wave: the grid-stride loop covers any n
    const void *kern = vec ? reinterpret_cast<const void *>(sreduce_kernel<OP, true>)
                           : reinterpret_cast<const void *>(sreduce_kernel<OP, false>);
    int64_t blocks = (n + 4095) / 4096;
    const int64_t cap = b2b::resident_ctas(h, kern, kThreads, 0);
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    void *ws = nullptr;
    if (int rc = b2b::workspace(h, static_cast<size_t>(blocks) * sizeof(Partial), &ws)) return rc;
    unsigned int *counter = reinterpret_cast<unsigned int *>(reinterpret_cast<char *>(h->d_status) +
                                                             B2B_STATUS_REDUCE_COUNTER);
    if (vec)
        sreduce_kernel<OP, true><<<(unsigned)blocks, kThreads, 0, h->stream>>>(x, y, n, static_cast<Partial *>(ws),
                                                                              counter, out);
    else
        sreduce_kernel<OP, false><<<(unsigned)blocks, kThreads, 0, h->stream>>>(x, y, n, static_cast<Partial *>(ws),
                                                                               counter, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? B2B_OK : b2b::fail_cuda(e, "reduction launch");
}

}  // namespace

namespace b2b {

int launch_sreduce(b2b_handle *h, int op, size_t n, const float *x, const float *y, void *d_out) {
    switch (op) {
        case B2B_REDUCE_DOT: return launch_op<B2B_REDUCE_DOT>(h, (int64_t)n, x, y, d_out);
        case B2B_REDUCE_NRM2: return launch_op<B2B_REDUCE_NRM2>(h, (int64_t)n, x, y, d_out);
        case B2B_REDUCE_ASUM: return launch_op<B2B_REDUCE_ASUM>(h, (int64_t)n, x, y, d_out);
        case B2B_REDUCE_IAMAX: return launch_op<B2B_REDUCE_IAMAX>(h, (int64_t)n, x, y, d_out);
        default: return fail(B2B_ERR_INVALID_ARG, "reduction: unknown op");
    }
}

}  // namespace b2b
