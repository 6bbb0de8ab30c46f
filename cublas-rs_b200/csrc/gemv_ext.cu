// gemv_ext.cu -- DGEMV and HGEMV: y <- alpha * op(A) * x + beta * y with A
// m x n row-major, the operations of cublas-rs's dgemv_n/t
// (crates/cublas-l2/src/gemv.rs:386-437) and hgemv_n/t (gemv.rs:553-606;
// f16 in/out, f32 accumulate, alpha/beta as f32).
//
// Same streaming structure as SGEMV (gemv.cu), templated on the element type:
//   * N: S warps per row (rows cut into ~16 KiB segments), 16-byte loads of
//     A (2 doubles / 8 halves) with ld.global.nc.L1::no_allocate, x through
//     L1, shuffle reduction, partials added in segment order.
//   * T: split-row partial sums (as many row slices as fill one resident
//     wave of CTAs), four rows' loads in flight per lane, each lane owning one
//     16-byte column group, ordered second-pass reduction; partials in the
//     handle's workspace in the accumulation type.
// Accumulation is in double for DGEMV and float for HGEMV; the f16 result is
// rounded to nearest even (the reference truncates, gemv.rs:534-551).
// beta == 0 does not read y.  Rows or pointers that break 16-byte alignment
// take the scalar path of the same kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// 16-byte loads, kept raw until every load of an unrolled group is issued
// (the asm is volatile, so the loads stay in program order; the unpacking
// that follows is free to wait for them).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 u;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "l"(p));
    return u;
}

__device__ __forceinline__ uint4 ld_cached16(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

template <typename T>
struct GV;
template <>
struct GV<double> {
    using Acc = double;
    static constexpr int W = 2;  // elements per 16-byte vector
    __device__ __forceinline__ static void unpack(const uint4 &u, Acc (&v)[W]) {
        v[0] = __hiloint2double((int)u.y, (int)u.x);
        v[1] = __hiloint2double((int)u.w, (int)u.z);
    }
    __device__ __forceinline__ static Acc get(const double *p) { return *p; }
    __device__ __forceinline__ static Acc get_stream(const double *p) {
        double v;
        asm volatile("ld.global.nc.L1::no_allocate.f64 %0, [%1];" : "=d"(v) : "l"(p));
        return v;
    }
    __device__ __forceinline__ static double put(Acc v) { return v; }
};
template <>
struct GV<uint16_t> {
    using Acc = float;
    static constexpr int W = 8;
    __device__ __forceinline__ static void unpack(const uint4 &u, Acc (&v)[W]) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    __device__ __forceinline__ static Acc get(const uint16_t *p) { return __half2float(__ushort_as_half(*p)); }
    __device__ __forceinline__ static Acc get_stream(const uint16_t *p) {
        unsigned short v;
        asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
        return __half2float(__ushort_as_half(v));
    }
    __device__ __forceinline__ static uint16_t put(Acc v) { return __half_as_ushort(__float2half_rn(v)); }
};

template <typename Acc>
__device__ __forceinline__ Acc warp_sum(Acc v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// N: S warps per row, warp s summing the s-th of S contiguous column
// segments; partials added in segment order through shared memory.
template <typename T, bool VEC, int S>
__global__ void __launch_bounds__(kThreads) gemvx_n_kernel(const T *__restrict__ A, const T *__restrict__ x,
                                                           T *__restrict__ y, int64_t m, int64_t n,
                                                           typename GV<T>::Acc alpha, typename GV<T>::Acc beta) {
    using Acc = typename GV<T>::Acc;
    constexpr int W = GV<T>::W;
    constexpr int UNROLL = 4;
    static_assert(kWarps % S == 0, "segments per row divide the CTA's warps");
    if constexpr (S == 1) {
        // One warp per row: no shared memory, finished warps leave early.
        const int lane = threadIdx.x & 31;
        const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
        if (row >= m) return;
        const T *a = A + row * n;
        Acc acc = Acc(0);
        if constexpr (VEC) {
            const int64_t nv = n / W;
            int64_t j = lane;
            for (; j + 32 * (UNROLL - 1) < nv; j += 32 * UNROLL) {
                uint4 ar[UNROLL], xr[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) ar[u] = ld_stream16(a + (j + 32 * u) * W);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) xr[u] = ld_cached16(x + (j + 32 * u) * W);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    Acc av[W], xv[W];
                    GV<T>::unpack(ar[u], av);
                    GV<T>::unpack(xr[u], xv);
#pragma unroll
                    for (int e = 0; e < W; ++e) acc = fma(av[e], xv[e], acc);
                }
            }
            for (; j < nv; j += 32) {
                Acc av[W], xv[W];
                GV<T>::unpack(ld_stream16(a + j * W), av);
                GV<T>::unpack(ld_cached16(x + j * W), xv);
#pragma unroll
                for (int e = 0; e < W; ++e) acc = fma(av[e], xv[e], acc);
            }
        } else {
            for (int64_t j = lane; j < n; j += 32) acc = fma(GV<T>::get_stream(a + j), GV<T>::get(x + j), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            Acc v = alpha * acc;
            if (beta != Acc(0)) v = fma(beta, GV<T>::get(y + row), v);
            y[row] = GV<T>::put(v);
        }
        return;
    }
    __shared__ Acc part[kWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (kWarps / S) + warp / S;
    const int seg = warp % S;
    Acc acc = Acc(0);
    if (row < m) {
        const T *a = A + row * n;
        if constexpr (VEC) {
            const int64_t nv = n / W;
            const int64_t seg_len = (nv + S - 1) / S;
            const int64_t v0 = seg * seg_len, v1 = v0 + seg_len < nv ? v0 + seg_len : nv;
            int64_t j = v0 + lane;
            for (; j + 32 * (UNROLL - 1) < v1; j += 32 * UNROLL) {
                uint4 ar[UNROLL], xr[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) ar[u] = ld_stream16(a + (j + 32 * u) * W);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) xr[u] = ld_cached16(x + (j + 32 * u) * W);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    Acc av[W], xv[W];
                    GV<T>::unpack(ar[u], av);
                    GV<T>::unpack(xr[u], xv);
#pragma unroll
                    for (int e = 0; e < W; ++e) acc = fma(av[e], xv[e], acc);
                }
            }
            for (; j < v1; j += 32) {
                Acc av[W], xv[W];
                GV<T>::unpack(ld_stream16(a + j * W), av);
                GV<T>::unpack(ld_cached16(x + j * W), xv);
#pragma unroll
                for (int e = 0; e < W; ++e) acc = fma(av[e], xv[e], acc);
            }
        } else {
            const int64_t seg_len = (n + S - 1) / S;
            const int64_t c0 = seg * seg_len, c1 = c0 + seg_len < n ? c0 + seg_len : n;
            for (int64_t j = c0 + lane; j < c1; j += 32) acc = fma(GV<T>::get_stream(a + j), GV<T>::get(x + j), acc);
        }
        acc = warp_sum(acc);
    }
    if constexpr (S > 1) {
        if (lane == 0) part[warp] = acc;
        __syncthreads();
        if (seg == 0 && lane == 0 && row < m) {
            Acc t = part[warp];
#pragma unroll
            for (int q = 1; q < S; ++q) t += part[warp + q];
            acc = t;
        }
    }
    if (seg == 0 && lane == 0 && row < m) {
        Acc v = alpha * acc;
        if (beta != Acc(0)) v = fma(beta, GV<T>::get(y + row), v);
        y[row] = GV<T>::put(v);
    }
}

template <typename T, bool VEC>
cudaError_t launch_gemvx_n(b2b_handle *h, const T *A, const T *x, T *y, int64_t m, int64_t n,
                           typename GV<T>::Acc alpha, typename GV<T>::Acc beta, int S) {
    const int64_t rows_per_cta = kWarps / S;
    const unsigned blocks = static_cast<unsigned>((m + rows_per_cta - 1) / rows_per_cta);
    switch (S) {
        case 1: gemvx_n_kernel<T, VEC, 1><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        case 2: gemvx_n_kernel<T, VEC, 2><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        case 4: gemvx_n_kernel<T, VEC, 4><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
        default: gemvx_n_kernel<T, VEC, 8><<<blocks, kThreads, 0, h->stream>>>(A, x, y, m, n, alpha, beta); break;
    }
    return cudaGetLastError();
}

// T, pass 1: CTA (column block of 32*W columns, row slice); lane l owns
// columns c0 + l*W .. +W-1 (VEC) or c0 + l + 32e (scalar).
template <typename T, bool VEC, bool DIRECT>
__global__ void __launch_bounds__(kThreads) gemvx_t_partial_kernel(const T *__restrict__ A, const T *__restrict__ x,
                                                                   void *__restrict__ out, int64_t m, int64_t n,
                                                                   int64_t rows_per_slice,
                                                                   typename GV<T>::Acc alpha,
                                                                   typename GV<T>::Acc beta) {
    using Acc = typename GV<T>::Acc;
    constexpr int W = GV<T>::W;
    constexpr int CB = 32 * W;
    __shared__ Acc red[kWarps][CB];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * CB;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_slice;
    const int64_t r1 = r0 + rows_per_slice < m ? r0 + rows_per_slice : m;
    Acc acc[W];
#pragma unroll
    for (int e = 0; e < W; ++e) acc[e] = Acc(0);
    if constexpr (VEC) {
        const int64_t c = c0 + lane * W;
        if (c < n) {  // n % W == 0: the vector is all in range
            int64_t r = r0 + warp;
            // four rows' 16-byte loads in flight per lane
            for (; r + 3 * kWarps < r1; r += 4 * kWarps) {
                uint4 raw[4];
                Acc xs[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) raw[u] = ld_stream16(A + (r + u * kWarps) * n + c);
#pragma unroll
                for (int u = 0; u < 4; ++u) xs[u] = GV<T>::get(x + r + u * kWarps);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    Acc v[W];
                    GV<T>::unpack(raw[u], v);
#pragma unroll
                    for (int e = 0; e < W; ++e) acc[e] = fma(v[e], xs[u], acc[e]);
                }
            }
            for (; r < r1; r += kWarps) {
                Acc v[W];
                GV<T>::unpack(ld_stream16(A + r * n + c), v);
                const Acc xs = GV<T>::get(x + r);
#pragma unroll
                for (int e = 0; e < W; ++e) acc[e] = fma(v[e], xs, acc[e]);
            }
        }
#pragma unroll
        for (int e = 0; e < W; ++e) red[warp][lane * W + e] = acc[e];
    } else {
        for (int64_t r = r0 + warp; r < r1; r += kWarps) {
            const Acc xs = GV<T>::get(x + r);
#pragma unroll
            for (int e = 0; e < W; ++e) {
                const int64_t c = c0 + lane + 32 * e;
                if (c < n) acc[e] = fma(GV<T>::get_stream(A + r * n + c), xs, acc[e]);
            }
        }
#pragma unroll
        for (int e = 0; e < W; ++e) red[warp][lane + 32 * e] = acc[e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < CB; i += kThreads) {
        const int64_t c = c0 + i;
        if (c >= n) continue;
        Acc s = Acc(0);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w][i];
        if constexpr (DIRECT) {
            T *y = static_cast<T *>(out);
            Acc v = alpha * s;
            if (beta != Acc(0)) v = fma(beta, GV<T>::get(y + c), v);
            y[c] = GV<T>::put(v);
        } else {
            static_cast<Acc *>(out)[static_cast<int64_t>(blockIdx.y) * n + c] = s;
        }
    }
}

template <typename T>
__global__ void gemvx_t_reduce_kernel(const typename GV<T>::Acc *__restrict__ partial, T *__restrict__ y, int64_t n,
                                      int slices, typename GV<T>::Acc alpha, typename GV<T>::Acc beta) {
    using Acc = typename GV<T>::Acc;
    const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= n) return;
    Acc s = Acc(0);
    for (int i = 0; i < slices; ++i) s += partial[static_cast<int64_t>(i) * n + j];
    Acc v = alpha * s;
    if (beta != Acc(0)) v = fma(beta, GV<T>::get(y + j), v);
    y[j] = GV<T>::put(v);
}

template <typename T>
int run_gemvx(b2b_handle *h, int trans, int64_t m, int64_t n, typename GV<T>::Acc alpha,
              typename GV<T>::Acc beta, const T *A, const T *x, T *y) {
    using Acc = typename GV<T>::Acc;
    constexpr int W = GV<T>::W;
    cudaError_t e;
    if (trans == B2B_OP_N) {
        const bool vec = (n % W == 0) && b2b::aligned16(A) && b2b::aligned16(x);
        // Row segments of about gemv_seg_bytes (twice that for f16, whose
        // unpacking makes short segments slower: HGEMV 16384^2 takes 79 us
        // with whole 32 KiB rows per warp, 91 us with 16 KiB segments; DGEMV
        // 16384^2 325 us whole, 301 us in 16 KiB segments).
        const int64_t seg_bytes = h->gemv_seg_bytes * (sizeof(T) == 2 ? 2 : 1);
        int S = 1;
        while (S < 8 && n * static_cast<int64_t>(sizeof(T)) >= 2 * S * seg_bytes) S *= 2;
        if ((m + kWarps / S - 1) / (kWarps / S) > 0x7fffffffLL) return b2b::fail(B2B_ERR_INVALID_ARG, "gemv: m too large");
        e = vec ? launch_gemvx_n<T, true>(h, A, x, y, m, n, alpha, beta, S)
                : launch_gemvx_n<T, false>(h, A, x, y, m, n, alpha, beta, S);
        return e == cudaSuccess ? B2B_OK : b2b::fail_cuda(e, "gemv N launch");
    }
    const bool vec = (n % W == 0) && b2b::aligned16(A);
    const int64_t cb = (n + 32 * W - 1) / (32 * W);
    if (cb > 0x7fffffffLL) return b2b::fail(B2B_ERR_INVALID_ARG, "gemv: n too large");
    // Row slices so that every CTA of the grid is resident at once: a grid a
    // little over one wave would leave a short second wave running alone.
    const int64_t slots = b2b::resident_ctas(
        h, vec ? reinterpret_cast<const void *>(gemvx_t_partial_kernel<T, true, false>)
               : reinterpret_cast<const void *>(gemvx_t_partial_kernel<T, false, false>),
        kThreads, 0);
    int64_t slices = cb >= slots ? 1 : slots / cb;
    const int64_t max_slices = (m + 63) / 64;
    if (slices > max_slices) slices = max_slices;
    if (slices > 65535) slices = 65535;
    if (slices < 1) slices = 1;
    const int64_t rows_per = (m + slices - 1) / slices;
    slices = (m + rows_per - 1) / rows_per;
    if (slices == 1) {
        dim3 grid((unsigned)cb, 1);
        if (vec)
            gemvx_t_partial_kernel<T, true, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        else
            gemvx_t_partial_kernel<T, false, true><<<grid, kThreads, 0, h->stream>>>(A, x, y, m, n, rows_per, alpha, beta);
        e = cudaGetLastError();
        return e == cudaSuccess ? B2B_OK : b2b::fail_cuda(e, "gemv T launch");
    }
    void *ws = nullptr;
    if (int rc = b2b::workspace(h, static_cast<size_t>(slices) * static_cast<size_t>(n) * sizeof(Acc), &ws)) return rc;
    dim3 grid((unsigned)cb, (unsigned)slices);
    if (vec)
        gemvx_t_partial_kernel<T, true, false><<<grid, kThreads, 0, h->stream>>>(A, x, ws, m, n, rows_per, alpha, beta);
    else
        gemvx_t_partial_kernel<T, false, false><<<grid, kThreads, 0, h->stream>>>(A, x, ws, m, n, rows_per, alpha, beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return b2b::fail_cuda(e, "gemv T partial launch");
    gemvx_t_reduce_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, h->stream>>>(static_cast<const Acc *>(ws), y, n,
                                                                                 (int)slices, alpha, beta);
    e = cudaGetLastError();
    return e == cudaSuccess ? B2B_OK : b2b::fail_cuda(e, "gemv T reduce launch");
}

}  // namespace

namespace b2b {

int launch_dgemv(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A, const double *x,
                 double beta, double *y) {
    return run_gemvx<double>(h, trans, (int64_t)m, (int64_t)n, alpha, beta, A, x, y);
}

int launch_hgemv(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A, const uint16_t *x,
                 float beta, uint16_t *y) {
    return run_gemvx<uint16_t>(h, trans, (int64_t)m, (int64_t)n, alpha, beta, A, x, y);
}

}  // namespace b2b
