// dgemm_dmma.cu -- DGEMM on the FP64 tensor path (mma.sync m8n8k4 .f64).
//
// C <- alpha * A * B + beta * C, row-major f64 operands, the operation of
// cublas-rs's dgemm_* kernels (crates/cublas-l3/src/dgemm.rs:25-334).
// tcgen05 has no f64 kind, so the FP64 matrix instruction on sm_100 is the
// warp-level mma.sync .f64: one m8n8k4 instruction is 256 double FMAs for a
// warp, fed from registers that each hold one element, so a warp loads 12
// doubles from shared memory for 32 instructions (8192 FMAs) per 4-wide k
// step -- about 20 times fewer operand loads per FMA than a DFMA outer
// product.
//
//   * CTA tile 128 x 128, 8 warps as 2 (M) x 4 (N); each warp owns 64 x 32 =
//     8 x 4 tiles of 8 x 8 accumulators (two doubles per thread per tile).
//   * k-tiles of 32 in a 3-stage cp.async ring: A as As[m][k] (k contiguous,
//     row pitch 36 doubles), B as Bs[k][n] (row pitch 132 doubles); both
//     pitches are 32 bytes mod 128, so the fragment loads (thread t reads row
//     t/4, element t%4 of A; row t%4, column t/4 of B) hit 16 distinct 8-byte
//     bank slots per half-warp -- no conflicts.
//   * Fragments are double-buffered in registers across k steps.
//   * Two kernels share that layout: dgemm_dmma_ws_kernel (the default) is
//     persistent, with a producer warpgroup that fills the ring and signals
//     mbarriers, so the DMMA warps never meet a CTA-wide barrier;
//     dgemm_dmma_kernel (one CTA per tile, all warps copy and meet at a
//     __syncthreads per k-tile) is kept for comparison.
// Fragment layout of m8n8k4 .f64: A (8x4, row): thread t holds A[t/4][t%4];
// B (4x8, col): B[t%4][t/4]; C/D (8x8): C[t/4][2(t%4)], C[t/4][2(t%4)+1].
// Requires K and N even and 16-byte aligned operands (else the CUDA-core
// kernel in gemm_simt.cu runs).
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#include "internal.h"
#include "sm100.cuh"

namespace {

constexpr int kWarpsM = 2, kWarpsN = 4;
constexpr int kThreads = kWarpsM * kWarpsN * 32;
constexpr int kMT = 8, kNT = 4;          // 8x8 tiles per warp along M, N
constexpr int kBM = kWarpsM * kMT * 8;   // 128
constexpr int kBN = kWarpsN * kNT * 8;   // 128
constexpr int kLdB = kBN + 4;            // Bs[k][n]

// k-tile and ring depth.  A rows are padded to kBK + 4 doubles so the pitch
// stays 32 bytes mod 128 (conflict-free fragment loads) for kBK = 16 or 32.
template <int BK_, int STAGES_>
struct DCfg {
    static constexpr int kBK = BK_;
    static constexpr int kStages = STAGES_;
    static constexpr int kLdA = kBK + 4;  // As[m][k]
    static constexpr int kAStage = kBM * kLdA;
    static constexpr int kBStage = kBK * kLdB;
    static constexpr int kSmem = kStages * (kAStage + kBStage) * 8;
    static constexpr int kACopies = kBM * kBK / 2 / kThreads;  // 16-byte copies per thread
    static constexpr int kBCopies = kBK * kBN / 2 / kThreads;
    static_assert(kACopies * kThreads * 2 == kBM * kBK, "A tile divides");
    static_assert(kBCopies * kThreads * 2 == kBK * kBN, "B tile divides");
    static_assert((kLdA * 8) % 128 == 32, "conflict-free A pitch");
};

__device__ __forceinline__ void cp16(uint32_t dst, const void *src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

struct DTileMap {
    int64_t tiles_m, tiles_n;
};

template <int BK_, int STAGES_>
__global__ void __launch_bounds__(kThreads, 1)
    dgemm_dmma_kernel(const double *__restrict__ A, const double *__restrict__ B, double *__restrict__ C, int64_t M,
                      int64_t N, int64_t K, double alpha, double beta, DTileMap tmap) {
    using Cf = DCfg<BK_, STAGES_>;
    constexpr int kBK = Cf::kBK, kStages = Cf::kStages, kLdA = Cf::kLdA, kAStage = Cf::kAStage,
                  kBStage = Cf::kBStage, kACopies = Cf::kACopies, kBCopies = Cf::kBCopies;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *As = reinterpret_cast<double *>(smem_raw);
    double *Bs = As + kStages * kAStage;

    // Grouped raster (8 M tiles sweep the N tiles) for L2 reuse.
    const int64_t t = blockIdx.x;
    const int64_t span = 8 * tmap.tiles_n;
    const int64_t g = t / span;
    const int64_t first = g * 8;
    const int64_t gm = tmap.tiles_m - first < 8 ? tmap.tiles_m - first : 8;
    const int64_t r = t - g * span;
    const int64_t m0 = (first + r % gm) * kBM, n0 = (r / gm) * kBN;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm0 = (warp / kWarpsN) * kMT * 8, wn0 = (warp % kWarpsN) * kNT * 8;
    const int fr = lane >> 2, fc = lane & 3;  // fragment row / column in an 8x4 (A) or 4x8 (B) tile

    // Copy assignment: A vector (ar + p*32, ak) and B vector (bk + p*4, bc).
    const int ak = (tid % (kBK / 2)) * 2, ar = tid / (kBK / 2);           // 8 vectors per A row
    const int bc = (tid % (kBN / 2)) * 2, bk = tid / (kBN / 2);           // 64 vectors per B row
    constexpr int kARowsPerPass = kThreads / (kBK / 2);                   // 32
    constexpr int kBRowsPerPass = kThreads / (kBN / 2);                   // 4
    const int64_t rows_left = M - m0 - ar;
    const bool col_ok = n0 + bc < N;
    const double *ga = A + (rows_left > 0 ? (m0 + ar) * K : 0) + ak;
    const double *gb = B + static_cast<int64_t>(bk) * N + (col_ok ? n0 + bc : 0);
    const uint32_t sa0 = static_cast<uint32_t>(__cvta_generic_to_shared(As)) + (ar * kLdA + ak) * 8;
    const uint32_t sb0 = static_cast<uint32_t>(__cvta_generic_to_shared(Bs)) + (bk * kLdB + bc) * 8;
    const int64_t a_pass = static_cast<int64_t>(kARowsPerPass) * K;
    const int64_t b_pass = static_cast<int64_t>(kBRowsPerPass) * N;
    const int64_t ktiles = (K + kBK - 1) / kBK;

    auto load_stage = [&](int stage, int64_t kt) {
        const int64_t k0 = kt * kBK;
        const uint32_t a_st = sa0 + static_cast<uint32_t>(stage * kAStage * 8);
        const uint32_t b_st = sb0 + static_cast<uint32_t>(stage * kBStage * 8);
        const bool ka_ok = k0 + ak < K;  // K even: the 2-vector is all in or all out
#pragma unroll
        for (int p = 0; p < kACopies; ++p) {
            const bool ok = ka_ok && p * kARowsPerPass < rows_left;
            cp16(a_st + p * kARowsPerPass * kLdA * 8, ok ? ga + k0 + p * a_pass : A, ok);
        }
        const double *pb = gb + k0 * N;
#pragma unroll
        for (int p = 0; p < kBCopies; ++p) {
            const bool ok = col_ok && k0 + bk + p * kBRowsPerPass < K;
            cp16(b_st + p * kBRowsPerPass * kLdB * 8, ok ? pb + p * b_pass : B, ok);
        }
    };

    double acc[kMT][kNT][2];
#pragma unroll
    for (int i = 0; i < kMT; ++i)
#pragma unroll
        for (int j = 0; j < kNT; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < ktiles) load_stage(s, s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }

    for (int64_t kt = 0; kt < ktiles; ++kt) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
        __syncthreads();
        const int64_t pre = kt + kStages - 1;
        if (pre < ktiles) load_stage(static_cast<int>(pre % kStages), pre);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const int stage = static_cast<int>(kt % kStages);
        const double *as = As + stage * kAStage + (wm0 + fr) * kLdA + fc;
        const double *bs = Bs + stage * kBStage + fc * kLdB + wn0 + fr;
        double af[2][kMT], bf[2][kNT];
#pragma unroll
        for (int i = 0; i < kMT; ++i) af[0][i] = as[i * 8 * kLdA];
#pragma unroll
        for (int j = 0; j < kNT; ++j) bf[0][j] = bs[j * 8];
#pragma unroll
        for (int ks = 0; ks < kBK / 4; ++ks) {
            const int cur = ks & 1;
            if (ks + 1 < kBK / 4) {
#pragma unroll
                for (int i = 0; i < kMT; ++i) af[cur ^ 1][i] = as[i * 8 * kLdA + (ks + 1) * 4];
#pragma unroll
                for (int j = 0; j < kNT; ++j) bf[cur ^ 1][j] = bs[(ks + 1) * 4 * kLdB + j * 8];
            }
#pragma unroll
            for (int i = 0; i < kMT; ++i)
#pragma unroll
                for (int j = 0; j < kNT; ++j) dmma_8x8x4(acc[i][j], af[cur][i], bf[cur][j]);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    const bool read_c = beta != 0.0;
#pragma unroll
    for (int i = 0; i < kMT; ++i) {
        const int64_t row = m0 + wm0 + i * 8 + fr;
        if (row >= M) continue;
        double *crow = C + row * N;
#pragma unroll
        for (int j = 0; j < kNT; ++j) {
            const int64_t col = n0 + wn0 + j * 8 + 2 * fc;
            if (col >= N) continue;  // N even: both columns in range
            double2 o = make_double2(alpha * acc[i][j][0], alpha * acc[i][j][1]);
            double2 *dst = reinterpret_cast<double2 *>(crow + col);
            if (read_c) {
                const double2 old = *dst;
                o.x = fma(beta, old.x, o.x);
                o.y = fma(beta, old.y, o.y);
            }
            *dst = o;
        }
    }
}

// Persistent warp-specialised form: 8 DMMA warps (the same 2 x 4 warps of
// 64 x 32 and fragment code as dgemm_dmma_kernel) and a producer warpgroup
// that fills the cp.async ring.  Each producer thread copies its 32 chunks of
// a stage, then cp.async.mbarrier.arrive.noinc makes the stage's "full"
// barrier (count 128) complete once all of its copies have landed; the DMMA
// warps wait on "full", run the stage's k steps and arrive on "empty"
// (count 8), which the producer waits on before refilling the stage.  The
// DMMA loop thus meets no CTA-wide barrier, and the producer loads the next
// tile's first stages while the DMMA warps store the current one.  CTA b takes
// tiles b, b + gridDim.x, ... in the grouped raster order.  Same per-element
// arithmetic (and bits) as dgemm_dmma_kernel.  384 threads launched at 168
// registers (64512 in all); the producer warpgroup keeps 56 and the DMMA
// warps take 224 (128 x 56 + 256 x 224 = 64512).
constexpr int kWsThreads = 384;
constexpr int kWsProducers = 128;

struct DWsArgs {
    int64_t tiles;  // work units of the call: tiles x splits
    int *status;
    uint64_t wait_ns;
    // Split-K: unit u is split u / (tiles / ksplit) of tile u % (tiles /
    // ksplit), k-tiles [s * kt_per_split, ...), whose raw sums go to
    // partial[s][M][N]; dgemm_splitk_reduce_kernel finishes the outputs.
    int ksplit;
    int64_t kt_per_split;
    double *partial;
};


__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sm100::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void dtile_coords(const DTileMap &tmap, int64_t t, int64_t &m0, int64_t &n0) {
    const int64_t span = 8 * tmap.tiles_n;
    const int64_t g = t / span;
    const int64_t first = g * 8;
    const int64_t gm = tmap.tiles_m - first < 8 ? tmap.tiles_m - first : 8;
    const int64_t r = t - g * span;
    m0 = (first + r % gm) * kBM;
    n0 = (r / gm) * kBN;
}

// Work unit u: its tile's first row and column, split and k-tiles [kt0, kt0 + nk).
__device__ __forceinline__ void dgemm_unit(const DTileMap &tmap, const DWsArgs &args, int64_t u, int64_t ktiles,
                                           int64_t &m0, int64_t &n0, int64_t &split, int64_t &kt0, int64_t &nk) {
    split = 0;
    kt0 = 0;
    nk = ktiles;
    if (args.ksplit > 1) {
        const int64_t per_split = args.tiles / args.ksplit;
        split = u / per_split;
        u -= split * per_split;
        kt0 = split * args.kt_per_split;
        nk = ktiles - kt0 < args.kt_per_split ? ktiles - kt0 : args.kt_per_split;
        if (nk < 0) nk = 0;
    }
    dtile_coords(tmap, u, m0, n0);
}

template <int BK_, int STAGES_>
__global__ void __launch_bounds__(kWsThreads, 1)
    dgemm_dmma_ws_kernel(const double *__restrict__ A, const double *__restrict__ B, double *__restrict__ C,
                         int64_t M, int64_t N, int64_t K, double alpha, double beta, DTileMap tmap, DWsArgs args) {
    using namespace sm100;
    using Cf = DCfg<BK_, STAGES_>;
    constexpr int kBK = Cf::kBK, kStages = Cf::kStages, kLdA = Cf::kLdA, kAStage = Cf::kAStage,
                  kBStage = Cf::kBStage;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *As = reinterpret_cast<double *>(smem_raw);
    double *Bs = As + kStages * kAStage;
    uint64_t *full = reinterpret_cast<uint64_t *>(Bs + kStages * kBStage);
    uint64_t *empty = full + kStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStages);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t ktiles = (K + kBK - 1) / kBK;
    const int64_t ntiles = (args.tiles - static_cast<int64_t>(blockIdx.x) + gridDim.x - 1) / gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kWsProducers);
            mbar_init(&empty[s], kThreads / 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp >= kThreads / 32) {
        // ------------------------------------------------ producer warpgroup
        asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
        const int pt = tid - kThreads;
        // Chunk q (0..2047) of a stage: A row q / (kBK / 2), doubles 2 (q % (kBK / 2)) ..;
        // B row q / (kBN / 2), columns 2 (q % (kBN / 2)) ..
        const uint32_t as0 = static_cast<uint32_t>(__cvta_generic_to_shared(As));
        const uint32_t bs0 = static_cast<uint32_t>(__cvta_generic_to_shared(Bs));
        int64_t g = 0;
        bool ok = true;
        for (int64_t ti = 0; ti < ntiles && ok; ++ti) {
            int64_t m0, n0, split, kt0, nk;
            dgemm_unit(tmap, args, static_cast<int64_t>(blockIdx.x) + ti * gridDim.x, ktiles, m0, n0, split, kt0, nk);
            for (int64_t kt = 0; kt < nk; ++kt, ++g) {
                const int s = static_cast<int>(g % kStages);
                if (g >= kStages) {
                    bool w = mbar_wait(&empty[s], static_cast<uint32_t>((g / kStages - 1) & 1), abort_flag,
                                       args.status, B2B_DEVSTAT_TIMEOUT | 0x41, args.wait_ns);
                    if (!__all_sync(0xffffffffu, w)) {
                        ok = false;
                        break;
                    }
                }
                const int64_t k0 = (kt0 + kt) * kBK;
#pragma unroll 4
                for (int q = pt; q < kBM * kBK / 2; q += kWsProducers) {
                    const int r = q / (kBK / 2), c = (q % (kBK / 2)) * 2;
                    const bool in = m0 + r < M && k0 + c < K;  // K even: the pair is all in or all out
                    cp16(as0 + static_cast<uint32_t>((s * kAStage + r * kLdA + c) * 8),
                         in ? A + (m0 + r) * K + k0 + c : A, in);
                }
#pragma unroll 4
                for (int q = pt; q < kBK * kBN / 2; q += kWsProducers) {
                    const int r = q / (kBN / 2), c = (q % (kBN / 2)) * 2;
                    const bool in = k0 + r < K && n0 + c < N;  // N even
                    cp16(bs0 + static_cast<uint32_t>((s * kBStage + r * kLdB + c) * 8),
                         in ? B + (k0 + r) * N + n0 + c : B, in);
                }
                cp_async_arrive_noinc(&full[s]);
            }
        }
        // Copies still in flight land before the CTA's shared memory goes away.
        asm volatile("cp.async.wait_all;" ::: "memory");
        return;
    }

    // ---------------------------------------------------- DMMA warps
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
    const int wm0 = (warp / kWarpsN) * kMT * 8, wn0 = (warp % kWarpsN) * kNT * 8;
    const int fr = lane >> 2, fc = lane & 3;
    int64_t g = 0;
    bool ok = true;
#pragma unroll 1
    for (int64_t ti = 0; ti < ntiles && ok; ++ti) {
        double acc[kMT][kNT][2];
#pragma unroll
        for (int i = 0; i < kMT; ++i)
#pragma unroll
            for (int j = 0; j < kNT; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
        int64_t nk;
        {
            int64_t m_, n_, s_, k_;
            dgemm_unit(tmap, args, static_cast<int64_t>(blockIdx.x) + ti * gridDim.x, ktiles, m_, n_, s_, k_, nk);
        }
        for (int64_t kt = 0; kt < nk; ++kt, ++g) {
            const int stage = static_cast<int>(g % kStages);
            bool w = mbar_wait(&full[stage], static_cast<uint32_t>((g / kStages) & 1), abort_flag, args.status,
                               B2B_DEVSTAT_TIMEOUT | 0x42, args.wait_ns);
            if (!__all_sync(0xffffffffu, w)) {
                ok = false;
                break;
            }
            const double *as = As + stage * kAStage + (wm0 + fr) * kLdA + fc;
            const double *bs = Bs + stage * kBStage + fc * kLdB + wn0 + fr;
            double af[2][kMT], bf[2][kNT];
#pragma unroll
            for (int i = 0; i < kMT; ++i) af[0][i] = as[i * 8 * kLdA];
#pragma unroll
            for (int j = 0; j < kNT; ++j) bf[0][j] = bs[j * 8];
#pragma unroll
            for (int ks = 0; ks < kBK / 4; ++ks) {
                const int cur = ks & 1;
                if (ks + 1 < kBK / 4) {
#pragma unroll
                    for (int i = 0; i < kMT; ++i) af[cur ^ 1][i] = as[i * 8 * kLdA + (ks + 1) * 4];
#pragma unroll
                    for (int j = 0; j < kNT; ++j) bf[cur ^ 1][j] = bs[(ks + 1) * 4 * kLdB + j * 8];
                }
#pragma unroll
                for (int i = 0; i < kMT; ++i)
#pragma unroll
                    for (int j = 0; j < kNT; ++j) dmma_8x8x4(acc[i][j], af[cur][i], bf[cur][j]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }
        if (!ok) break;
        int64_t m0, n0, split, kt0, nk_;
        dgemm_unit(tmap, args, static_cast<int64_t>(blockIdx.x) + ti * gridDim.x, ktiles, m0, n0, split, kt0, nk_);
        if (args.ksplit > 1) {
            // raw sums of this k range; the reduce applies alpha and beta
            double *P = args.partial + split * M * N;
#pragma unroll
            for (int i = 0; i < kMT; ++i) {
                const int64_t row = m0 + wm0 + i * 8 + fr;
                if (row >= M) continue;
#pragma unroll
                for (int j = 0; j < kNT; ++j) {
                    const int64_t col = n0 + wn0 + j * 8 + 2 * fc;
                    if (col >= N) continue;
                    *reinterpret_cast<double2 *>(P + row * N + col) = make_double2(acc[i][j][0], acc[i][j][1]);
                }
            }
            continue;
        }
        const bool read_c = beta != 0.0;
#pragma unroll
        for (int i = 0; i < kMT; ++i) {
            const int64_t row = m0 + wm0 + i * 8 + fr;
            if (row >= M) continue;
            double *crow = C + row * N;
#pragma unroll
            for (int j = 0; j < kNT; ++j) {
                const int64_t col = n0 + wn0 + j * 8 + 2 * fc;
                if (col >= N) continue;  // N even: both columns in range
                double2 o = make_double2(alpha * acc[i][j][0], alpha * acc[i][j][1]);
                double2 *dst = reinterpret_cast<double2 *>(crow + col);
                if (read_c) {
                    const double2 old = *dst;
                    o.x = fma(beta, old.x, o.x);
                    o.y = fma(beta, old.y, o.y);
                }
                *dst = o;
            }
        }
    }
}

// C <- alpha * (P[0] + P[1] + ... + P[S-1]) + beta * C, the partials added in
// split order, alpha and beta applied as the unsplit epilogue does: the same
// bits on every run for a given S.
__global__ void __launch_bounds__(256) dgemm_splitk_reduce_kernel(const double *__restrict__ P, int S, int64_t M,
                                                                  int64_t N, double *__restrict__ C, double alpha,
                                                                  double beta) {
    const int64_t MN = M * N;
    for (int64_t q = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 2; q < MN;
         q += static_cast<int64_t>(gridDim.x) * blockDim.x * 2) {
        double2 s = *reinterpret_cast<const double2 *>(P + q);
        for (int i = 1; i < S; ++i) {
            const double2 v = *reinterpret_cast<const double2 *>(P + i * MN + q);
            s.x += v.x;
            s.y += v.y;
        }
        double2 o = make_double2(alpha * s.x, alpha * s.y);
        if (beta != 0.0) {
            const double2 old = *reinterpret_cast<const double2 *>(C + q);
            o.x = fma(beta, old.x, o.x);
            o.y = fma(beta, old.y, o.y);
        }
        *reinterpret_cast<double2 *>(C + q) = o;
    }
}

}  // namespace

namespace b2b {

// Split-K factor for an M x N x K DGEMM on the persistent DMMA kernel: the S
// in {1, 2, 3, 4, 6, 8} with the least estimated time, where the GEMM costs
// waves x k-tiles per CTA (a 128 x 128 x 32 k-tile takes ~4.7 us at the
// kernel's DMMA rate) and a split adds the reduce (reading S partials and
// writing C, 8 (S + 1) M N bytes at ~6 TB/s: the partials' writes hide under
// the compute-bound GEMM) plus a launch.  Each split keeps at least 8
// k-tiles.  Taken when it saves 5% or more.  Measured: 1024^3 S = 2 24.8 vs
// 13.6 TFLOP/s unsplit, 2048^3 S = 4 30.2 vs 28.0, 4096 x 1024 x 4096 S = 8
// 31.0 vs 28.6; 4096^3 (6.9 waves) stays unsplit.
int dgemm_ksplit(int sm_count, int64_t M, int64_t N, int64_t K) {
    const double tiles = static_cast<double>(((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN));
    const int64_t kt = (K + 31) / 32;
    const double kt_us = 4.7;
    auto est = [&](int S) {
        const double waves = std::ceil(tiles * S / sm_count);
        const double kts = static_cast<double>((kt + S - 1) / S);
        double t = waves * kts * kt_us;
        if (S > 1) t += 8.0 * (S + 1) * static_cast<double>(M) * static_cast<double>(N) / 6e12 * 1e6 + 4.0;
        return t;
    };
    const double t1 = est(1);
    int best = 1;
    double tb = t1;
    for (int S : {2, 3, 4, 6, 8}) {
        if ((kt + S - 1) / S < 8) break;
        const double t = est(S);
        if (t < tb) {
            tb = t;
            best = S;
        }
    }
    return tb <= 0.95 * t1 ? best : 1;
}

bool dgemm_dmma_eligible(int64_t N, int64_t K, const void *A, const void *B, const void *C) {
    return (K % 2 == 0) && (N % 2 == 0) && aligned16(A) && aligned16(B) && aligned16(C);
}

namespace {
template <int BK_, int STAGES_>
int launch_dmma(b2b_handle *h, int64_t M, int64_t N, int64_t K, double alpha, double beta, const double *A,
                const double *B, double *C) {
    using Cf = DCfg<BK_, STAGES_>;
    DTileMap tm{(M + kBM - 1) / kBM, (N + kBN - 1) / kBN};
    const int64_t blocks = tm.tiles_m * tm.tiles_n;
    if (blocks > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "dgemm: grid exceeds 2^31-1 tiles");
    auto kern = dgemm_dmma_kernel<BK_, STAGES_>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmem);
    if (e == cudaSuccess) {
        kern<<<static_cast<unsigned>(blocks), kThreads, Cf::kSmem, h->stream>>>(A, B, C, M, N, K, alpha, beta, tm);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return fail_cuda(e, "dgemm launch");
    return B2B_OK;
}
template <int BK_, int STAGES_>
int launch_dmma_ws(b2b_handle *h, int64_t M, int64_t N, int64_t K, double alpha, double beta, const double *A,
                   const double *B, double *C) {
    using Cf = DCfg<BK_, STAGES_>;
    constexpr int smem = Cf::kSmem + 2 * Cf::kStages * 8 + 16;  // + full/empty barriers, abort flag
    static_assert(smem <= 232448, "shared memory per CTA");
    DTileMap tm{(M + kBM - 1) / kBM, (N + kBN - 1) / kBN};
    const int64_t tiles = tm.tiles_m * tm.tiles_n;
    // The split: forced by the caller (a host-slice call's tiles take the
    // whole GEMM's, so every tile sums the same k ranges), else chosen here.
    const int64_t ktiles = (K + BK_ - 1) / BK_;
    int S = h->dgemm_ksplit_forced > 0 ? h->dgemm_ksplit_forced : dgemm_ksplit(h->sm_count, M, N, K);
    if (S > ktiles) S = static_cast<int>(ktiles);
    if (S < 1) S = 1;
    const int64_t ktps = (ktiles + S - 1) / S;
    double *partial = nullptr;
    if (S > 1) {
        void *ws = nullptr;
        const size_t bytes = static_cast<size_t>(S) * static_cast<size_t>(M) * static_cast<size_t>(N) * 8;
        if (int rc = workspace(h, bytes, &ws)) return rc;
        partial = static_cast<double *>(ws);
    }
    const int64_t units = tiles * S;
    auto kern = dgemm_dmma_ws_kernel<BK_, STAGES_>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) {
        // one CTA per SM: its shared memory allows no second one
        const int64_t grid = units < h->sm_count ? units : h->sm_count;
        kern<<<static_cast<unsigned>(grid), kWsThreads, smem, h->stream>>>(
            A, B, C, M, N, K, alpha, beta, tm, DWsArgs{units, h->d_status, h->wait_limit_ns, S, ktps, partial});
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return fail_cuda(e, "dgemm (persistent) launch");
    if (S > 1) {
        int64_t blocks = (M * N / 2 + 255) / 256;
        const int64_t cap = 8LL * h->sm_count;
        if (blocks > cap) blocks = cap;
        dgemm_splitk_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, h->stream>>>(partial, S, M, N, C, alpha,
                                                                                          beta);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "dgemm split-K reduce launch");
    }
    return B2B_OK;
}
}  // namespace

int launch_dgemm_dmma(b2b_handle *h, int64_t M, int64_t N, int64_t K, double alpha, double beta, const double *A,
                      const double *B, double *C) {
    // The persistent warp-specialised form, k-tile 32, 3 stages: 32.8 TF/s at
    // 4096^3 against 32.1 for dgemm_dmma_kernel<32, 3> (variant 8) and
    // 32.2-32.4 for the persistent form with k-tile 16 and 4-5 stages, same
    // bits.  dgemm_dmma_kernel with k-tile 16 (variant 7): 31.4-31.6.
    if (h->dgemm_variant == 7) return launch_dmma<16, 3>(h, M, N, K, alpha, beta, A, B, C);
    if (h->dgemm_variant == 8) return launch_dmma<32, 3>(h, M, N, K, alpha, beta, A, B, C);
    return launch_dmma_ws<32, 3>(h, M, N, K, alpha, beta, A, B, C);
}

}  // namespace b2b
