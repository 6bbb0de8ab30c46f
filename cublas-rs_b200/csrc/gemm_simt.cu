// gemm_simt.cu -- register-blocked FFMA / DFMA GEMM for sm_100a: SGEMM,
// DGEMM and strided-batched SGEMM.
//
// Computes, per batch b, C_b <- alpha * A_b * B_b + beta * C_b with row-major
// A_b[M x K], B_b[K x N], C_b[M x N] and X_b = X + b * stride_X, the operation
// of cublas-rs's sgemm_* / dgemm_* / strided_batched_sgemm kernels
// (crates/cublas-l3/src/sgemm.rs:31-360, dgemm.rs:25-334, batched.rs:25-102).
// Unlike those (one 16x16 or 32x32 shared tile per CTA, one or four outputs
// per thread), every CTA here owns a BM x BN tile and every thread a TM x TN
// register block, so each shared-memory value feeds TM (or TN) FMAs:
//
//   * 256 threads = 8 warps laid out WARPS_M x WARPS_N; a warp is 4 x 8
//     threads; a thread's rows are ty*4+{0..3} (+16 when TM=8) and its
//     columns tx*4+{0..3} (+32 when TN=8) inside the warp tile, so fragment
//     loads are 16-byte shared loads with no bank conflicts (A values are
//     broadcast to the 8 threads of a row group, B values are 8 distinct
//     16-byte chunks).
//   * A is stored transposed in shared memory (As[k][m], padded by 4) so
//     that fragments along M are contiguous; B is stored as-is (Bs[k][n]).
//   * Two kernels share that layout:
//       - gemm_async_kernel (the default where the 16-byte path applies):
//         a STAGES-deep cp.async ring (4 stages of k-tile 8 for SGEMM), A
//         transposed on the way in with 4-byte copies, B as 16-byte copies,
//         fragments double-buffered in registers, copy addresses derived from
//         two base pointers so the FMA loop keeps its registers;
//       - gemm_simt_kernel (any shape or alignment): two shared stages, the
//         next k-tile fetched from global memory into registers while the
//         current one is multiplied, then stored to the other stage -- one
//         __syncthreads per k-tile.
//     Single large SGEMMs and batched SGEMMs normally take the TMA-fed
//     kernels of sgemm_tma.cu instead, with the same per-element arithmetic.
//   * The epilogue skips reading C when beta == 0.
//   * The batch and tile indices come from one flattened grid index, so there
//     is no 65535 limit on the batch count (the reference puts the batch in
//     gridDim.z, batched.rs:128-137).
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace {

constexpr int kThreads = 256;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
    __device__ __forceinline__ static void load(const float *p, float (&v)[4]) {
        float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x;
        v[1] = t.y;
        v[2] = t.z;
        v[3] = t.w;
    }
    __device__ __forceinline__ static void store(float *p, const float (&v)[4]) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <>
struct Vec4<double> {
    __device__ __forceinline__ static void load(const double *p, double (&v)[4]) {
        double2 a = reinterpret_cast<const double2 *>(p)[0];
        double2 b = reinterpret_cast<const double2 *>(p)[1];
        v[0] = a.x;
        v[1] = a.y;
        v[2] = b.x;
        v[3] = b.y;
    }
    __device__ __forceinline__ static void store(double *p, const double (&v)[4]) {
        reinterpret_cast<double2 *>(p)[0] = make_double2(v[0], v[1]);
        reinterpret_cast<double2 *>(p)[1] = make_double2(v[2], v[3]);
    }
};

// 16-byte global vector of T (4 floats or 2 doubles).
template <typename T>
struct GVec;
template <>
struct GVec<float> {
    static constexpr int W = 4;
    using V = float4;
    __device__ __forceinline__ static void get(const V &v, float (&o)[4]) {
        o[0] = v.x;
        o[1] = v.y;
        o[2] = v.z;
        o[3] = v.w;
    }
};
template <>
struct GVec<double> {
    static constexpr int W = 2;
    using V = double2;
    __device__ __forceinline__ static void get(const V &v, double (&o)[2]) {
        o[0] = v.x;
        o[1] = v.y;
    }
};

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK>
struct Cfg {
    static constexpr int BM = WARPS_M * (TM / 4) * 16;
    static constexpr int BN = WARPS_N * (TN / 4) * 32;
    static constexpr int W = GVec<T>::W;
    static constexpr int PADA = 4;
    static constexpr int LDA_S = BM + PADA;  // As[k][m]
    static constexpr int LDB_S = BN;         // Bs[k][n]
    static constexpr int A_VECS = BM * BK / W / kThreads;
    static constexpr int B_VECS = BK * BN / W / kThreads;
    static constexpr int A_ELEMS = BM * BK / kThreads;  // scalar path
    static constexpr int B_ELEMS = BK * BN / kThreads;
    static constexpr int SMEM = 2 * BK * (LDA_S + LDB_S) * (int)sizeof(T);
    static_assert(WARPS_M * WARPS_N * 32 == kThreads, "256 threads");
    static_assert(A_VECS * W * kThreads == BM * BK, "A tile divides");
    static_assert(B_VECS * W * kThreads == BK * BN, "B tile divides");
};

struct TileMap {
    int64_t tiles_m, tiles_n, tiles_per_batch;
};

// Optional epilogue additions: C = act(alpha*A*B + beta*C + bias[col]) with
// act = ReLU when relu != 0 (bias == nullptr: no bias).
template <typename T>
struct EpiArgs {
    const T *bias;
    int relu;
};

template <typename T>
__device__ __forceinline__ T epi_apply(T v, const EpiArgs<T> &epi, int64_t col) {
    if (epi.bias) v += epi.bias[col];
    if (epi.relu) v = v > T(0) ? v : T(0);
    return v;
}

// Grouped raster: GROUP consecutive M tiles sweep the N tiles together, so
// the A and B panels of the CTAs resident at one time stay in L2.
__device__ __forceinline__ void map_tile(int64_t t, const TileMap &tm, int64_t &batch, int64_t &bm, int64_t &bn) {
    constexpr int64_t GROUP = 8;
    batch = t / tm.tiles_per_batch;
    int64_t r = t - batch * tm.tiles_per_batch;
    int64_t group_span = GROUP * tm.tiles_n;
    int64_t g = r / group_span;
    int64_t first_m = g * GROUP;
    int64_t gm = tm.tiles_m - first_m < GROUP ? tm.tiles_m - first_m : GROUP;
    int64_t rr = r - g * group_span;
    bm = first_m + rr % gm;
    bn = rr / gm;
}

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK, bool VEC, int MINB>
__global__ void __launch_bounds__(kThreads, MINB)
    gemm_simt_kernel(const T *__restrict__ A, const T *__restrict__ B, T *__restrict__ C, int64_t M, int64_t N,
                     int64_t K, T alpha, T beta, int64_t sA, int64_t sB, int64_t sC, TileMap tmap,
                     EpiArgs<T> epi) {
    using Cf = Cfg<T, TM, TN, WARPS_M, WARPS_N, BK>;
    constexpr int BM = Cf::BM, BN = Cf::BN, W = Cf::W;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);         // [2][BK][LDA_S]
    T *Bs = As + 2 * BK * Cf::LDA_S;                  // [2][BK][LDB_S]

    int64_t batch, bm, bn;
    map_tile(blockIdx.x, tmap, batch, bm, bn);
    A += batch * sA;
    B += batch * sB;
    C += batch * sC;
    const int64_t m0 = bm * BM, n0 = bn * BN;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int wm = warp / WARPS_N, wn = warp % WARPS_N;
    const int ty = lane >> 3, tx = lane & 7;
    const int row_base = wm * (TM / 4) * 16 + ty * 4;  // + g*16
    const int col_base = wn * (TN / 4) * 32 + tx * 4;  // + g*32

    T acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = T(0);

    // Registers holding the next k-tile on its way to shared memory.
    T ra[VEC ? Cf::A_VECS * W : Cf::A_ELEMS];
    T rb[VEC ? Cf::B_VECS * W : Cf::B_ELEMS];

    // Per-thread source pointers, advanced by one k-tile per fetch; the row
    // (A) and column (B) bounds are fixed per thread, only k varies.
    constexpr int AV = VEC ? Cf::A_VECS : Cf::A_ELEMS;
    constexpr int BV = VEC ? Cf::B_VECS : Cf::B_ELEMS;
    constexpr int AW = VEC ? W : 1;
    const T *pa[AV];
    const T *pb[BV];
    int ka[AV], kb[BV];  // k offset of each load inside the tile
    bool oka[AV], okb[BV];
#pragma unroll
    for (int v = 0; v < AV; ++v) {
        const int idx = tid + v * kThreads;
        const int r = idx / (BK / AW), kc = (idx % (BK / AW)) * AW;
        oka[v] = m0 + r < M;
        pa[v] = A + (oka[v] ? (m0 + r) * K : 0) + kc;
        ka[v] = kc;
    }
#pragma unroll
    for (int v = 0; v < BV; ++v) {
        const int idx = tid + v * kThreads;
        const int kr = idx / (BN / AW), c = (idx % (BN / AW)) * AW;
        okb[v] = n0 + c < N;
        pb[v] = B + static_cast<int64_t>(kr) * N + (okb[v] ? n0 + c : 0);
        kb[v] = kr;
    }
    const int64_t b_step = static_cast<int64_t>(BK) * N;

    auto fetch = [&](int64_t k0) {
#pragma unroll
        for (int v = 0; v < AV; ++v) {
            if constexpr (VEC) {
                T tmp[W];
                if (oka[v] && k0 + ka[v] < K) {
                    GVec<T>::get(*reinterpret_cast<const typename GVec<T>::V *>(pa[v]), tmp);
                } else {
#pragma unroll
                    for (int e = 0; e < W; ++e) tmp[e] = T(0);
                }
#pragma unroll
                for (int e = 0; e < W; ++e) ra[v * W + e] = tmp[e];
            } else {
                ra[v] = (oka[v] && k0 + ka[v] < K) ? *pa[v] : T(0);
            }
            pa[v] += BK;
        }
#pragma unroll
        for (int v = 0; v < BV; ++v) {
            if constexpr (VEC) {
                T tmp[W];
                if (okb[v] && k0 + kb[v] < K) {
                    GVec<T>::get(*reinterpret_cast<const typename GVec<T>::V *>(pb[v]), tmp);
                } else {
#pragma unroll
                    for (int e = 0; e < W; ++e) tmp[e] = T(0);
                }
#pragma unroll
                for (int e = 0; e < W; ++e) rb[v * W + e] = tmp[e];
            } else {
                rb[v] = (okb[v] && k0 + kb[v] < K) ? *pb[v] : T(0);
            }
            pb[v] += b_step;
        }
    };

    auto stash = [&](int stage) {
        T *as = As + stage * BK * Cf::LDA_S;
        T *bs = Bs + stage * BK * Cf::LDB_S;
        if constexpr (VEC) {
#pragma unroll
            for (int v = 0; v < Cf::A_VECS; ++v) {
                int idx = tid + v * kThreads;
                int r = idx / (BK / W), kc = (idx % (BK / W)) * W;
#pragma unroll
                for (int e = 0; e < W; ++e) as[(kc + e) * Cf::LDA_S + r] = ra[v * W + e];
            }
#pragma unroll
            for (int v = 0; v < Cf::B_VECS; ++v) {
                int idx = tid + v * kThreads;
                int kr = idx / (BN / W), c = (idx % (BN / W)) * W;
                if constexpr (W == 4) {
                    *reinterpret_cast<float4 *>(&bs[kr * Cf::LDB_S + c]) =
                        make_float4(rb[v * 4 + 0], rb[v * 4 + 1], rb[v * 4 + 2], rb[v * 4 + 3]);
                } else {
                    *reinterpret_cast<double2 *>(&bs[kr * Cf::LDB_S + c]) = make_double2(rb[v * 2 + 0], rb[v * 2 + 1]);
                }
            }
        } else {
#pragma unroll
            for (int v = 0; v < Cf::A_ELEMS; ++v) {
                int idx = tid + v * kThreads;
                int r = idx / BK, kc = idx % BK;
                as[kc * Cf::LDA_S + r] = ra[v];
            }
#pragma unroll
            for (int v = 0; v < Cf::B_ELEMS; ++v) {
                int idx = tid + v * kThreads;
                int kr = idx / BN, c = idx % BN;
                bs[kr * Cf::LDB_S + c] = rb[v];
            }
        }
    };

    const int64_t ktiles = (K + BK - 1) / BK;
    fetch(0);
    stash(0);
    __syncthreads();

    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int cur = static_cast<int>(kt & 1);
        const bool more = kt + 1 < ktiles;
        if (more) fetch((kt + 1) * BK);
        const T *as = As + cur * BK * Cf::LDA_S;
        const T *bs = Bs + cur * BK * Cf::LDB_S;
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            T af[TM], bf[TN];
#pragma unroll
            for (int g = 0; g < TM / 4; ++g) {
                T t[4];
                Vec4<T>::load(as + kk * Cf::LDA_S + row_base + g * 16, t);
#pragma unroll
                for (int e = 0; e < 4; ++e) af[g * 4 + e] = t[e];
            }
#pragma unroll
            for (int g = 0; g < TN / 4; ++g) {
                T t[4];
                Vec4<T>::load(bs + kk * Cf::LDB_S + col_base + g * 32, t);
#pragma unroll
                for (int e = 0; e < 4; ++e) bf[g * 4 + e] = t[e];
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fma(af[i], bf[j], acc[i][j]);
        }
        if (more) stash(cur ^ 1);
        __syncthreads();
    }

    // Epilogue: C = alpha*acc (+ beta*C).
    const bool read_c = beta != T(0);
#pragma unroll
    for (int gi = 0; gi < TM / 4; ++gi) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t r = m0 + row_base + gi * 16 + i;
            if (r >= M) continue;
            T *crow = C + r * N;
#pragma unroll
            for (int gj = 0; gj < TN / 4; ++gj) {
                const int64_t c = n0 + col_base + gj * 32;
                T out[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) out[e] = alpha * acc[gi * 4 + i][gj * 4 + e];
                if (VEC && c + 4 <= N) {
                    if (read_c) {
                        T old[4];
                        Vec4<T>::load(crow + c, old);
#pragma unroll
                        for (int e = 0; e < 4; ++e) out[e] = fma(beta, old[e], out[e]);
                    }
                    if (epi.bias || epi.relu) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) out[e] = epi_apply(out[e], epi, c + e);
                    }
                    Vec4<T>::store(crow + c, out);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (c + e < N) {
                            T v = out[e];
                            if (read_c) v = fma(beta, crow[c + e], v);
                            crow[c + e] = epi_apply(v, epi, c + e);
                        }
                    }
                }
            }
        }
    }
}

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK, int MINB>
int run_simt(b2b_handle *h, int64_t M, int64_t N, int64_t K, T alpha, T beta, const T *A, int64_t sA, const T *B,
             int64_t sB, T *C, int64_t sC, int64_t batch, EpiArgs<T> epi = EpiArgs<T>{nullptr, 0}) {
    using Cf = Cfg<T, TM, TN, WARPS_M, WARPS_N, BK>;
    TileMap tm;
    tm.tiles_m = (M + Cf::BM - 1) / Cf::BM;
    tm.tiles_n = (N + Cf::BN - 1) / Cf::BN;
    tm.tiles_per_batch = tm.tiles_m * tm.tiles_n;
    const int64_t blocks = tm.tiles_per_batch * batch;
    if (blocks > 0x7fffffffLL) return b2b::fail(B2B_ERR_INVALID_ARG, "GEMM grid exceeds 2^31-1 tiles");
    // 16-byte vector path: every row start and the base pointers aligned.
    constexpr int W = Cf::W;
    const bool vec = (K % W == 0) && (N % W == 0) && (sA % W == 0) && (sB % W == 0) && (sC % W == 0) &&
                     b2b::aligned16(A) && b2b::aligned16(B) && b2b::aligned16(C);
    cudaError_t e;
    if (vec) {
        auto kern = gemm_simt_kernel<T, TM, TN, WARPS_M, WARPS_N, BK, true, MINB>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM);
        if (e == cudaSuccess) {
            kern<<<static_cast<unsigned>(blocks), kThreads, Cf::SMEM, h->stream>>>(A, B, C, M, N, K, alpha, beta,
                                                                                   sA, sB, sC, tm, epi);
            e = cudaGetLastError();
        }
    } else {
        auto kern = gemm_simt_kernel<T, TM, TN, WARPS_M, WARPS_N, BK, false, MINB>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM);
        if (e == cudaSuccess) {
            kern<<<static_cast<unsigned>(blocks), kThreads, Cf::SMEM, h->stream>>>(A, B, C, M, N, K, alpha, beta,
                                                                                   sA, sB, sC, tm, epi);
            e = cudaGetLastError();
        }
    }
    if (e != cudaSuccess) return b2b::fail_cuda(e, "GEMM launch");
    return B2B_OK;
}

// ---------------------------------------------------------------------------
// FP32 GEMM with a multi-stage cp.async pipeline (16-byte vector path only:
// K, N and the strides multiples of 4, operands 16-byte aligned).
//
// Same thread layout and register blocking as gemm_simt_kernel, but global
// -> shared copies are asynchronous (cp.async), STAGES k-tiles deep, so no
// registers hold tiles in transit and the copies of k-tiles kt+1..kt+S-1
// overlap the FMAs of k-tile kt.  A is transposed on the way in with 4-byte
// copies (As[k][m], padded); B is copied as 16-byte vectors (Bs[k][n]).
// Out-of-range elements are zero-filled by the copy (src-size 0).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(ok ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK, int STAGES>
struct AsyncCfg {
    static constexpr int NT = WARPS_M * WARPS_N * 32;
    static constexpr int BM = WARPS_M * (TM / 4) * 16;
    static constexpr int BN = WARPS_N * (TN / 4) * 32;
    static constexpr int VW = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte copy
    static constexpr int LDA_S = BM + 4;                          // As[k][m]
    static constexpr int LDB_S = BN;                              // Bs[k][n]
    static constexpr int A_STAGE = BK * LDA_S;
    static constexpr int B_STAGE = BK * LDB_S;
    // A copies: each warp writes 4 rows x 8 consecutive k per instruction
    // (conflict-free in the transposed As[k][m] layout, whose pitch is 4
    // banks off a multiple of 32), repeated over row passes and 8-wide k groups.
    static constexpr int A_ROWS_PER_PASS = NT / 8;        // rows covered by one pass of the CTA
    static constexpr int A_PASSES = BM / A_ROWS_PER_PASS;
    static constexpr int A_KGROUPS = BK / 8;
    static constexpr int A_COPIES = A_PASSES * A_KGROUPS;  // element copies per thread
    static constexpr int B_COPIES = BK * BN / VW / NT;    // 16-byte copies per thread
    static constexpr int B_VECS_PER_ROW = BN / VW;
    static constexpr int B_ROWS_PER_PASS = NT / B_VECS_PER_ROW;
    static constexpr int SMEM = STAGES * (A_STAGE + B_STAGE) * static_cast<int>(sizeof(T));
    static_assert(BK % 8 == 0 && BM % A_ROWS_PER_PASS == 0 && A_COPIES * NT == BM * BK, "A tile divides");
    static_assert(NT % B_VECS_PER_ROW == 0 && B_COPIES * NT * VW == BK * BN, "B tile divides");
};

template <typename T>
struct PairOf;
template <>
struct PairOf<float> {
    using type = float2;
};
template <>
struct PairOf<double> {
    using type = double2;
};
__device__ __forceinline__ float2 pair_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ double2 pair_fma(double2 a, double2 b, double2 c) {
    return make_double2(fma(a.x, b.x, c.x), fma(a.y, b.y, c.y));
}

template <typename T>
__device__ __forceinline__ void cp_async_elem(uint32_t dst, const T *src, bool ok) {
    if constexpr (sizeof(T) == 4)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(ok ? 4 : 0) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(ok ? 8 : 0) : "memory");
}

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK, int STAGES, int MINB>
__global__ void __launch_bounds__(WARPS_M *WARPS_N * 32, MINB)
    gemm_async_kernel(const T *__restrict__ A, const T *__restrict__ B, T *__restrict__ C, int64_t M, int64_t N,
                      int64_t K, T alpha, T beta, int64_t sA, int64_t sB, int64_t sC, TileMap tmap,
                     EpiArgs<T> epi) {
    using Cf = AsyncCfg<T, TM, TN, WARPS_M, WARPS_N, BK, STAGES>;
    constexpr int BM = Cf::BM, BN = Cf::BN, NT = Cf::NT, VW = Cf::VW;
    constexpr int ES = static_cast<int>(sizeof(T));
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);
    T *Bs = As + STAGES * Cf::A_STAGE;

    int64_t batch, bm, bn;
    map_tile(blockIdx.x, tmap, batch, bm, bn);
    A += batch * sA;
    B += batch * sB;
    C += batch * sC;
    const int64_t m0 = bm * BM, n0 = bn * BN;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int wm = warp / WARPS_N, wn = warp % WARPS_N;
    const int ty = lane >> 3, tx = lane & 7;
    const int row_base = wm * (TM / 4) * 16 + ty * 4;
    const int col_base = wn * (TN / 4) * 32 + tx * 4;

    // Copy assignment.  A: this thread copies element (r0 + q*A_ROWS_PER_PASS,
    // ka + 8*g) of the A tile for every row pass q and k group g; B: 16-byte
    // vector (kb0 + p*B_ROWS_PER_PASS, cb) of the B tile.  Only two global
    // base pointers and a few scalars live across the main loop.
    const int ka = tid % 8, r0 = tid / 8;
    const int cb = (tid % Cf::B_VECS_PER_ROW) * VW, kb0 = tid / Cf::B_VECS_PER_ROW;
    const int64_t rows_left = M - m0 - r0;  // copy p is in range iff p*A_ROWS_PER_PASS < rows_left
    const bool col_ok = n0 + cb < N;        // N % VW == 0: a vector is all in or all out
    const T *ga = A + (rows_left > 0 ? (m0 + r0) * K : 0) + ka;
    const T *gb = B + static_cast<int64_t>(kb0) * N + (col_ok ? n0 + cb : 0);
    const uint32_t sa0 = static_cast<uint32_t>(__cvta_generic_to_shared(As)) + (ka * Cf::LDA_S + r0) * ES;
    const uint32_t sb0 = static_cast<uint32_t>(__cvta_generic_to_shared(Bs)) + (kb0 * Cf::LDB_S + cb) * ES;
    const int64_t a_pass = static_cast<int64_t>(Cf::A_ROWS_PER_PASS) * K;
    const int64_t b_pass = static_cast<int64_t>(Cf::B_ROWS_PER_PASS) * N;
    const int64_t ktiles = (K + BK - 1) / BK;

    auto load_stage = [&](int stage, int64_t kt) {
        const int64_t k0 = kt * BK;
        const uint32_t a_st = sa0 + static_cast<uint32_t>(stage * Cf::A_STAGE * ES);
        const uint32_t b_st = sb0 + static_cast<uint32_t>(stage * Cf::B_STAGE * ES);
#pragma unroll
        for (int g = 0; g < Cf::A_KGROUPS; ++g) {
            const bool ka_ok = k0 + ka + 8 * g < K;
            const T *pa = ga + k0 + 8 * g;
#pragma unroll
            for (int q = 0; q < Cf::A_PASSES; ++q) {
                const bool ok = ka_ok && q * Cf::A_ROWS_PER_PASS < rows_left;
                cp_async_elem<T>(a_st + (8 * g * Cf::LDA_S + q * Cf::A_ROWS_PER_PASS) * ES, ok ? pa + q * a_pass : A,
                                 ok);
            }
        }
        const T *pb = gb + k0 * N;
#pragma unroll
        for (int p = 0; p < Cf::B_COPIES; ++p) {
            const bool ok = col_ok && k0 + kb0 + p * Cf::B_ROWS_PER_PASS < K;
            cp_async16(b_st + p * Cf::B_ROWS_PER_PASS * Cf::LDB_S * ES, ok ? pb + p * b_pass : B, ok);
        }
    };

    // Outputs as row pairs: acc2[p][j] = (acc[2p][j], acc[2p+1][j]).  For
    // FP32 one packed FFMA2 (__ffma2_rn, sm_100) updates a pair, halving the
    // issue slots of the FMA loop; each lane is the same single-rounding fma,
    // so the result is that of the scalar loop, bit for bit.
    using P2 = typename PairOf<T>::type;
    P2 acc2[TM / 2][TN];
#pragma unroll
    for (int i = 0; i < TM / 2; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc2[i][j] = P2{T(0), T(0)};
    auto acc_at = [&](int i, int j) -> T & { return (i & 1) ? acc2[i >> 1][j].y : acc2[i >> 1][j].x; };

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < ktiles) load_stage(s, s);
        cp_async_commit();
    }

    auto load_frags = [&](const T *as, const T *bs, int kk, T (&af)[TM], T (&bf)[TN]) {
#pragma unroll
        for (int g = 0; g < TM / 4; ++g) {
            T t[4];
            Vec4<T>::load(as + kk * Cf::LDA_S + row_base + g * 16, t);
#pragma unroll
            for (int e = 0; e < 4; ++e) af[g * 4 + e] = t[e];
        }
#pragma unroll
        for (int g = 0; g < TN / 4; ++g) {
            T t[4];
            Vec4<T>::load(bs + kk * Cf::LDB_S + col_base + g * 32, t);
#pragma unroll
            for (int e = 0; e < 4; ++e) bf[g * 4 + e] = t[e];
        }
    };

    for (int64_t kt = 0; kt < ktiles; ++kt) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        const int64_t pre = kt + STAGES - 1;
        if (pre < ktiles) load_stage(static_cast<int>(pre % STAGES), pre);
        cp_async_commit();
        const int stage = static_cast<int>(kt % STAGES);
        const T *as = As + stage * Cf::A_STAGE;
        const T *bs = Bs + stage * Cf::B_STAGE;
        // Fragments double-buffered in registers: step kk+1's shared loads
        // are issued before step kk's FMAs.
        T af[2][TM], bf[2][TN];
        load_frags(as, bs, 0, af[0], bf[0]);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            if (kk + 1 < BK) load_frags(as, bs, kk + 1, af[(kk + 1) & 1], bf[(kk + 1) & 1]);
            const T *a = af[kk & 1], *b = bf[kk & 1];
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const P2 bb{b[j], b[j]};
#pragma unroll
                for (int p = 0; p < TM / 2; ++p) acc2[p][j] = pair_fma(P2{a[2 * p], a[2 * p + 1]}, bb, acc2[p][j]);
            }
        }
    }
    cp_async_wait<0>();

    const bool read_c = beta != T(0);
#pragma unroll
    for (int gi = 0; gi < TM / 4; ++gi) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t r = m0 + row_base + gi * 16 + i;
            if (r >= M) continue;
            T *crow = C + r * N;
#pragma unroll
            for (int gj = 0; gj < TN / 4; ++gj) {
                const int64_t c = n0 + col_base + gj * 32;
                if (c >= N) continue;  // N % 4 == 0: the 4-vector is all in or all out
                T out[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) out[e] = alpha * acc_at(gi * 4 + i, gj * 4 + e);
                if (read_c) {
                    T old[4];
                    Vec4<T>::load(crow + c, old);
#pragma unroll
                    for (int e = 0; e < 4; ++e) out[e] = fma(beta, old[e], out[e]);
                }
                if (epi.bias || epi.relu) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) out[e] = epi_apply(out[e], epi, c + e);
                }
                Vec4<T>::store(crow + c, out);
            }
        }
    }
}

template <typename T, int TM, int TN, int WARPS_M, int WARPS_N, int BK, int STAGES, int MINB>
int run_async(b2b_handle *h, int64_t M, int64_t N, int64_t K, T alpha, T beta, const T *A, int64_t sA, const T *B,
              int64_t sB, T *C, int64_t sC, int64_t batch, EpiArgs<T> epi = EpiArgs<T>{nullptr, 0}) {
    using Cf = AsyncCfg<T, TM, TN, WARPS_M, WARPS_N, BK, STAGES>;
    TileMap tm;
    tm.tiles_m = (M + Cf::BM - 1) / Cf::BM;
    tm.tiles_n = (N + Cf::BN - 1) / Cf::BN;
    tm.tiles_per_batch = tm.tiles_m * tm.tiles_n;
    const int64_t blocks = tm.tiles_per_batch * batch;
    if (blocks > 0x7fffffffLL) return b2b::fail(B2B_ERR_INVALID_ARG, "GEMM grid exceeds 2^31-1 tiles");
    auto kern = gemm_async_kernel<T, TM, TN, WARPS_M, WARPS_N, BK, STAGES, MINB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM);
    if (e == cudaSuccess) {
        kern<<<static_cast<unsigned>(blocks), Cf::NT, Cf::SMEM, h->stream>>>(A, B, C, M, N, K, alpha, beta, sA, sB, sC,
                                                                           tm, epi);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return b2b::fail_cuda(e, "GEMM launch");
    return B2B_OK;
}


bool vec_ok(int64_t K, int64_t N, int64_t sA, int64_t sB, int64_t sC, const void *A, const void *B, const void *C) {
    return (K % 4 == 0) && (N % 4 == 0) && (sA % 4 == 0) && (sB % 4 == 0) && (sC % 4 == 0) && b2b::aligned16(A) &&
           b2b::aligned16(B) && b2b::aligned16(C);
}

// FP32 GEMM dispatch: kernel `variant` (0 = default choice).
int run_sgemm(b2b_handle *h, int variant, int64_t M, int64_t N, int64_t K, float alpha, float beta, const float *A,
              int64_t sA, const float *B, int64_t sB, float *C, int64_t sC, int64_t batch,
              EpiArgs<float> epi = EpiArgs<float>{nullptr, 0}) {
    // Single GEMMs: the TMA-fed kernels (sgemm_tma.cu; same per-element
    // arithmetic) wherever sgemm_tma_path allows -- by default the persistent
    // row-major-A kernel (N and K multiples of 4, aligned, any size), with
    // split-K for grids that fill the GPU badly; variants 20/21/22 force the
    // transposed-A kernel's scalar / row-pair / column-pair forms and variant
    // 11 the cp.async kernel below.  A forced split-K (the tiles of a split
    // host-slice call) must take the TMA path whatever the tile's size.
    if (batch == 1 && b2b::sgemm_tma_path(variant, M, N, K, A, B, C, h->sgemm_ksplit_forced > 1))
        return b2b::launch_sgemm_tma(h, M, N, K, alpha, beta, A, B, C, epi.bias, epi.relu,
                                     variant == 0 ? 1 : variant - 20);
    // Batched calls (and variants 23-28): the TMA-fed kernels on row-major A
    // (no transpose pass through global memory), batched through 3-D tensor
    // maps; by default the persistent warp-specialised one (sgemm_tma.cu),
    // 58.8 vs 52.6 TFLOP/s for the cp.async kernel on 4096 x 256^3, same bits.
    if (((variant >= 23 && variant <= 28) || (variant == 0 && batch > 1)) &&
        b2b::sgemm_tma_rowa_eligible(M, N, K, sA, sB, sC, batch, A, B, C))
        return b2b::launch_sgemm_tma_rowa(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi.bias, epi.relu);
    if (!vec_ok(K, N, sA, sB, sC, A, B, C) || variant == 1)
        return run_simt<float, 8, 8, 4, 2, 8, 2>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
    switch (variant) {
        case 5: return run_async<float, 8, 8, 4, 2, 16, 2, 2>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 6: return run_async<float, 8, 8, 4, 2, 16, 3, 2>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 7: return run_async<float, 8, 16, 4, 2, 16, 2, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 8: return run_async<float, 16, 8, 2, 4, 16, 3, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 9: return run_async<float, 8, 16, 2, 4, 16, 2, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 10: return run_async<float, 16, 8, 2, 4, 16, 2, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 11: return run_async<float, 16, 8, 2, 4, 8, 4, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 12: return run_async<float, 8, 8, 4, 4, 16, 3, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        case 13: return run_async<float, 16, 8, 2, 4, 16, 4, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
        default: return run_async<float, 16, 8, 2, 4, 8, 4, 1>(h, M, N, K, alpha, beta, A, sA, B, sB, C, sC, batch, epi);
    }
}

// FP64 GEMM dispatch: the FP64 tensor path (dgemm_dmma.cu) by default; the
// CUDA-core DFMA kernels where its alignment rules do not hold (or when a
// variant is forced, for comparisons).
int run_dgemm(b2b_handle *h, int variant, int64_t M, int64_t N, int64_t K, double alpha, double beta,
              const double *A, const double *B, double *C) {
    if ((variant == 0 || variant >= 7) && b2b::dgemm_dmma_eligible(N, K, A, B, C))
        return b2b::launch_dgemm_dmma(h, M, N, K, alpha, beta, A, B, C);
    const bool vec = (K % 4 == 0) && (N % 4 == 0) && b2b::aligned16(A) && b2b::aligned16(B) && b2b::aligned16(C);
    if (!vec || variant == 1)
        return run_simt<double, 4, 4, 4, 2, 16, 2>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
    switch (variant) {
        case 2: return run_async<double, 8, 8, 4, 2, 8, 3, 1>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
        case 3: return run_async<double, 4, 8, 4, 2, 16, 3, 2>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
        case 4: return run_async<double, 8, 4, 4, 2, 16, 3, 2>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
        case 5: return run_async<double, 4, 4, 4, 2, 16, 3, 2>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
        case 6: return run_async<double, 8, 8, 2, 4, 8, 3, 1>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
        default: return run_async<double, 8, 8, 2, 4, 8, 3, 1>(h, M, N, K, alpha, beta, A, 0, B, 0, C, 0, 1);
    }
}

}  // namespace

namespace b2b {

// SGEMM: 128x128 CTA tile, 8x8 per thread, cp.async pipeline.
int launch_sgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                 float beta, float *C) {
    return run_sgemm(h, h->sgemm_variant, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta, A, 0, B, 0, C, 0, 1);
}

int launch_sgemm_bias(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                      float beta, float *C, const float *bias, int relu) {
    return run_sgemm(h, h->sgemm_variant, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta, A, 0, B, 0, C, 0, 1,
                     EpiArgs<float>{bias, relu});
}

int launch_sgemm_strided_batched(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                                 size_t sa, const float *B, size_t sb, float beta, float *C, size_t sc,
                                 size_t batch) {
    return run_sgemm(h, h->sgemm_variant, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta, A, (int64_t)sa, B,
                     (int64_t)sb, C, (int64_t)sc, (int64_t)batch);
}

// DGEMM: the FP64 tensor path (dgemm_dmma.cu) where its alignment rules hold,
// else the CUDA-core DFMA kernels above.
int launch_dgemm(b2b_handle *h, size_t m, size_t n, size_t k, double alpha, const double *A, const double *B,
                 double beta, double *C) {
    return run_dgemm(h, h->dgemm_variant, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta, A, B, C);
}

}  // namespace b2b
