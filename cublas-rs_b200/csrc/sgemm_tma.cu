// sgemm_tma.cu -- FP32 SGEMM on the CUDA cores with TMA-fed operands.
//
// The operation of cublas-rs's sgemm_* kernels (crates/cublas-l3/src/
// sgemm.rs:31-360): C <- alpha*A*B + beta*C (+ bias[j], ReLU for the fused
// epilogue), row-major, FP32 FFMA arithmetic, each output summed over k in
// order by one thread -- the same per-element arithmetic as the cp.async
// kernel in gemm_simt.cu, so results are bit-identical to it.
//
// The FFMA loop wants A as As[k][m] (four consecutive rows of one k in a
// 16-byte shared load).  Instead of transposing A tile by tile with 4-byte
// copies in the FFMA warps, A is transposed once into workspace (At, K x M;
// an HBM-bound pass of 8 bytes per element of A, ~0.4% of an 8192^3 GEMM),
// after which both operands are plain row-major tiles that TMA copies into
// shared memory exactly as the FFMA warps read them:
//   * CTA tile 128 x 256, k-block 32, 4-stage ring of 48 KiB (At box 128 x 32,
//     B box 256 x 32, no swizzle: fragment loads are conflict-free as laid out).
//   * 8 FFMA warps (2 x 4, 16 x 8 outputs per thread, the gemm_simt.cu
//     fragment layout) wait on a stage's "full" mbarrier (TMA completion)
//     and release it on its "empty" mbarrier -- no CTA-wide barrier and no
//     copy instructions in the loop.  Lane 0 of warp 0 issues the TMA loads:
//     all stages up front, then, after each k-block, a refill of the stage
//     every warp released one k-block earlier (S - 1 blocks ahead), so it
//     rarely waits for a slower warp.  (A separate producer warp would make
//     the CTA 288 threads, which registers are allocated for as 384, too few
//     registers per thread for the 128 accumulators.)
//   * The 16 x 8 outer product per k runs as 64 packed FFMA2 instructions
//     (__ffma2_rn, sm_100: two FP32 fmas per lane, each rounded once) on row
//     pairs, with b duplicated into a register pair: the FMA pipe stays fed
//     while half the issue slots go free for the shared loads (8192^3: 60.2
//     vs 52.2 TFLOP/s for 128 scalar FFMAs per k, same bits).
//   * Every wait is bounded; a wait that gives up records a status code,
//     raises the abort flag, and warp 0 drains its in-flight loads before the
//     CTA exits.
// That transposed-A kernel (sgemm_tma_kernel) is the one the forced variants
// 20-22 take.  By default single GEMMs with K % 4 == 0 (split or not) and
// strided-batched GEMMs run sgemm_tma_rowa_ws_kernel below instead: the same
// FFMA loop, persistent, with a producer warpgroup (setmaxnreg makes the
// 384-thread CTA affordable) that loads row-major A and B with TMA and
// transposes each A tile in shared memory, so no pass through global memory
// and no workspace precede the GEMM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace {

constexpr int kTM = 16, kTN = 8, kWM = 2, kWN = 4;
constexpr int kBM = kWM * (kTM / 4) * 16;  // 128
constexpr int kBN = kWN * (kTN / 4) * 32;  // 256
constexpr int kBK = 32;
constexpr int kComputeWarps = kWM * kWN;
constexpr int kThreads = kComputeWarps * 32;
constexpr int kStages = 4;
constexpr int kAStageF = kBK * kBM;  // floats per stage
constexpr int kBStageF = kBK * kBN;
constexpr uint32_t kStageBytes = (kAStageF + kBStageF) * 4;  // 48 KiB
constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
constexpr int kGroupM = 8;  // raster group (M tiles sweeping the N tiles together), batched kernels
// Raster group of the single-GEMM kernel: 64 tile rows (8192 rows) sweep the
// N tiles together; at 8192^3 that measured 60.7 vs 59.7 TFLOP/s for 8 rows
// (interleaved A/B, 3 rounds each, the same bits).
constexpr int kGroupMSingle = 64;
// Raster group of a single GEMM on the persistent row-major-A kernel: at
// 8192^3 groups of 8-64 tile rows run at the same 62.0 TFLOP/s, and 16 moves
// the fewest DRAM bytes (2.81 GB per launch; 8 rows: 3.44 GB).
constexpr int kGroupMSingleWs = 16;

struct SArgs {
    float *C;
    int64_t M, N, K;
    float alpha, beta;
    const float *bias;
    int relu;
    int *status;
    uint64_t wait_ns;
    int group_m;  // raster group in M tiles
    // Split-K: with ksplit > 1, CTA (split s, tile t) sums k-blocks
    // [s * kb_per_split, (s + 1) * kb_per_split) and stores its raw sums to
    // partial[s][M][N]; sgemm_splitk_reduce_kernel finishes the outputs.
    int ksplit;
    int64_t kb_per_split;
    float *partial;
};

// kPack selects the FFMA form of the 16 x 8 outer product (each output is
// the same fmaf chain over k in every form, so results are bit-identical):
//   0  scalar FFMA, 128 per k;
//   1  packed FFMA2 (__ffma2_rn, sm_100) on row pairs: (acc[i][j], acc[i+1][j])
//      += (a[i], a[i+1]) * (b[j], b[j]) -- 64 issue slots per k instead of 128;
//   2  packed FFMA2 on column pairs: (acc[i][j], acc[i][j+1]) += (a[i], a[i]) * (b[j], b[j+1]).
// Form 1 is the fastest (8192^3: 60.2 TF/s, vs 59.0 for form 2 and 52.2 for
// form 0): it duplicates 8 values per k (b) where form 2 duplicates 16 (a).
// Reading (a, a) pairs from an At written duplicated costs more than the
// register moves it saves (53.8 TF/s: twice the A tile, 3 stages instead of 4).
template <int kPack>
__global__ void __launch_bounds__(kThreads, 1)
    sgemm_tma_kernel(const __grid_constant__ CUtensorMap tmAt, const __grid_constant__ CUtensorMap tmB, SArgs args) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    float *As = reinterpret_cast<float *>(smem);
    float *Bs = As + kStages * kAStageF;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *full = bars;
    uint64_t *empty = bars + kStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 2 * kStages);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t tiles_m = (args.M + kBM - 1) / kBM, tiles_n = (args.N + kBN - 1) / kBN;
    const int64_t ntiles = tiles_m * tiles_n;
    // split (k range) and tile of this CTA; grouped raster within a split
    const int64_t split = args.ksplit > 1 ? static_cast<int64_t>(blockIdx.x) / ntiles : 0;
    const int64_t t = static_cast<int64_t>(blockIdx.x) - split * ntiles;
    const int64_t group_m = args.group_m;
    const int64_t span = group_m * tiles_n;
    const int64_t g = t / span;
    const int64_t first = g * group_m;
    const int64_t gm = tiles_m - first < group_m ? tiles_m - first : group_m;
    const int64_t r = t - g * span;
    const int64_t m0 = (first + r % gm) * kBM, n0 = (r / gm) * kBN;
    const int64_t ktiles_all = (args.K + kBK - 1) / kBK;
    // this CTA's k-blocks: kb0 + [0, ktiles)
    const int64_t kb0 = args.ksplit > 1 ? split * args.kb_per_split : 0;
    const int64_t ktiles = args.ksplit > 1
                               ? (ktiles_all - kb0 < args.kb_per_split ? ktiles_all - kb0 : args.kb_per_split)
                               : ktiles_all;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmAt);
        prefetch_tensormap(&tmB);
    }
    __syncthreads();

    const bool loader = tid == 0;
    int64_t issued = 0;  // k-blocks whose loads warp 0's lane 0 has issued
    auto issue = [&](int64_t kt) {
        const int s = static_cast<int>(kt % kStages);
        const int32_t kc = static_cast<int32_t>((kb0 + kt) * kBK);
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(As + s * kAStageF, &tmAt, &full[s], static_cast<int32_t>(m0), kc);
        tma_load_2d(Bs + s * kBStageF, &tmB, &full[s], static_cast<int32_t>(n0), kc);
        ++issued;
    };
    if (loader)
        for (int64_t kt = 0; kt < kStages && kt < ktiles; ++kt) issue(kt);

    const int wm = warp / kWN, wn = warp % kWN;
    const int ty = lane >> 3, tx = lane & 7;
    const int row_base = wm * (kTM / 4) * 16 + ty * 4;
    const int col_base = wn * (kTN / 4) * 32 + tx * 4;

    // acc2 holds the 16 x 8 outputs as pairs: rows (2p, 2p+1) of column j at
    // acc2[p][j] for kPack 0/1, columns (2q, 2q+1) of row i at acc2[i][q] for kPack 2.
    constexpr bool kColPairs = kPack == 2;
    constexpr int kP0 = kColPairs ? kTM : kTM / 2, kP1 = kColPairs ? kTN / 2 : kTN;
    float2 acc2[kP0][kP1];
#pragma unroll
    for (int i = 0; i < kP0; ++i)
#pragma unroll
        for (int j = 0; j < kP1; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
    auto acc_at = [&](int i, int j) -> float & {
        if (kColPairs) return (j & 1) ? acc2[i][j >> 1].y : acc2[i][j >> 1].x;
        return (i & 1) ? acc2[i >> 1][j].y : acc2[i >> 1][j].x;
    };

    auto load_frags = [&](const float *as, const float *bs, int kk, float (&af)[kTM], float (&bf)[kTN]) {
#pragma unroll
        for (int q = 0; q < kTM / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(as + kk * kBM + row_base + q * 16);
            af[q * 4 + 0] = v.x;
            af[q * 4 + 1] = v.y;
            af[q * 4 + 2] = v.z;
            af[q * 4 + 3] = v.w;
        }
#pragma unroll
        for (int q = 0; q < kTN / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(bs + kk * kBN + col_base + q * 32);
            bf[q * 4 + 0] = v.x;
            bf[q * 4 + 1] = v.y;
            bf[q * 4 + 2] = v.z;
            bf[q * 4 + 3] = v.w;
        }
    };

    bool ok = true;
    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int s = static_cast<int>(kt % kStages);
        const uint32_t ph = static_cast<uint32_t>((kt / kStages) & 1);
        const bool w = mbar_wait(&full[s], ph, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x32, args.wait_ns);
        if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
        }
        const float *as = As + s * kAStageF;
        const float *bs = Bs + s * kBStageF;
        float af[2][kTM], bf[2][kTN];
        load_frags(as, bs, 0, af[0], bf[0]);
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            if (kk + 1 < kBK) load_frags(as, bs, kk + 1, af[(kk + 1) & 1], bf[(kk + 1) & 1]);
            const float *a = af[kk & 1], *b = bf[kk & 1];
            if (kPack == 0) {
#pragma unroll
                for (int i = 0; i < kTM; ++i)
#pragma unroll
                    for (int j = 0; j < kTN; ++j) acc_at(i, j) = fmaf(a[i], b[j], acc_at(i, j));
            } else if (kPack == 1) {
#pragma unroll
                for (int j = 0; j < kTN; ++j) {
                    const float2 bb = make_float2(b[j], b[j]);
#pragma unroll
                    for (int p = 0; p < kTM / 2; ++p)
                        acc2[p][j] = __ffma2_rn(make_float2(a[2 * p], a[2 * p + 1]), bb, acc2[p][j]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < kTM; ++i) {
                    const float2 aa = make_float2(a[i], a[i]);
#pragma unroll
                    for (int q = 0; q < kTN / 2; ++q)
                        acc2[i][q] = __ffma2_rn(aa, make_float2(b[2 * q], b[2 * q + 1]), acc2[i][q]);
                }
            }
        }
        // every lane's reads of this stage are done: release it
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // Refill the stage released one k-block ago with the block S ahead of it.
        if (loader && kt >= 1) {
            const int64_t done = kt - 1, next = done + kStages;
            if (next < ktiles) {
                const int ds = static_cast<int>(done % kStages);
                const uint32_t dph = static_cast<uint32_t>((done / kStages) & 1);
                if (!mbar_wait(&empty[ds], dph, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x31, args.wait_ns)) {
                    ok = false;
                } else {
                    issue(next);
                }
            }
        }
        if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
        }
    }
    if (!ok) {
        if (loader && issued) {
            // Loads in flight complete on their full barriers: wait for them
            // (bounded) before the CTA's shared memory goes away.
            const int64_t first_pending = issued > kStages ? issued - kStages : 0;
            for (int64_t kt = first_pending; kt < issued; ++kt)
                mbar_wait_drain(&full[kt % kStages], static_cast<uint32_t>((kt / kStages) & 1), 1000000000ull);
        }
        return;
    }

    if (args.ksplit > 1) {
        // raw sums of this k range; the reduce applies alpha, beta, bias, ReLU
        float *P = args.partial + split * args.M * args.N;
#pragma unroll
        for (int gi = 0; gi < kTM / 4; ++gi) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t row = m0 + row_base + gi * 16 + i;
                if (row >= args.M) continue;
#pragma unroll
                for (int gj = 0; gj < kTN / 4; ++gj) {
                    const int64_t col = n0 + col_base + gj * 32;
                    if (col >= args.N) continue;
                    *reinterpret_cast<float4 *>(P + row * args.N + col) =
                        make_float4(acc_at(gi * 4 + i, gj * 4 + 0), acc_at(gi * 4 + i, gj * 4 + 1),
                                    acc_at(gi * 4 + i, gj * 4 + 2), acc_at(gi * 4 + i, gj * 4 + 3));
                }
            }
        }
        return;
    }
    const bool read_c = args.beta != 0.0f;
#pragma unroll
    for (int gi = 0; gi < kTM / 4; ++gi) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = m0 + row_base + gi * 16 + i;
            if (row >= args.M) continue;
            float *crow = args.C + row * args.N;
#pragma unroll
            for (int gj = 0; gj < kTN / 4; ++gj) {
                const int64_t col = n0 + col_base + gj * 32;
                if (col >= args.N) continue;  // N % 4 == 0: the 4-vector is all in or all out
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = args.alpha * acc_at(gi * 4 + i, gj * 4 + e);
                if (read_c) {
                    const float4 old = *reinterpret_cast<const float4 *>(crow + col);
                    o[0] = fmaf(args.beta, old.x, o[0]);
                    o[1] = fmaf(args.beta, old.y, o[1]);
                    o[2] = fmaf(args.beta, old.z, o[2]);
                    o[3] = fmaf(args.beta, old.w, o[3]);
                }
                if (args.bias || args.relu) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (args.bias) o[e] += args.bias[col + e];
                        if (args.relu) o[e] = o[e] > 0.0f ? o[e] : 0.0f;
                    }
                }
                *reinterpret_cast<float4 *>(crow + col) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// The same FFMA loop fed from row-major A directly, batched (the default for
// strided-batched calls; on single large GEMMs the transposed-A kernel above
// is faster, 60.2 vs 55.5 TFLOP/s at 8192^3, since it loads a 16-byte A
// fragment where this one loads four 4-byte values).  A tiles arrive as they
// lie in memory, As[m][k] (box 32 k x 128 m), with the 128-byte swizzle:
// 16-byte chunk c of row r sits at chunk c ^ (r % 8).  A thread owns rows
// wm*64 + ty + 4i (i < 16), so at any k the four row groups of a warp read
// four consecutive rows -- four distinct chunks, no bank conflicts -- and
// each a value is one 4-byte shared load; the row pair (i, i+1) of an FFMA2
// comes from two such loads straight into a register pair, so no transpose
// pass and no extra moves for A (b is duplicated as in form 1).  Operands
// are 3-D tensor maps (x innermost, then rows, then batch), so a tile never
// reads across a batch boundary and out-of-range rows/columns arrive as
// zeros.
//
// CTA shapes, the same per-thread work (16 x 8 outputs):
//   WN = 4: 8 warps, 128 x 256 tiles, 4 stages of 48 KiB -- one CTA per SM;
//     with A transposed in shared memory (XP, the default) or read as 4-byte
//     fragments (variant 24).
//   WN = 2: 4 warps, 128 x 128 tiles, 3 stages of 32 KiB -- two CTAs per SM,
//     so one CTA's prologue (the first TMA round trip) and epilogue (the C
//     stores) overlap the other's FFMA loop (variant 25; slower on the
//     4096 x 256^3 batched workload, 51.5 vs 54.0 TFLOP/s).
//   sgemm_tma_rowa_ws_kernel: the XP form, persistent, with a producer
//     warpgroup that also transposes A (the default).
// (A persistent form of WN = 4 whose load stream ran across tile boundaries,
// loaded by a compute warp, measured 45.1 vs 53.7 TFLOP/s on 4096 x 256^3:
// the bookkeeping took it to 255 registers and slowed the FFMA loop more than
// it hid.)
struct RArgs {
    float *C;
    int64_t M, N, K, sC, tiles_m, tiles_n;
    float alpha, beta;
    const float *bias;
    int relu;
    int *status;
    uint64_t wait_ns;
    int64_t tiles;    // work units of the whole call (the persistent form): tiles x splits
    int64_t group_m;  // raster group in tile rows
    // Split-K (the persistent form, batch 1): unit u is split u / tiles' k
    // blocks [s * kb_per_split, ...) of tile u % tiles, whose raw sums go to
    // partial[s][M][N]; sgemm_splitk_reduce_kernel finishes the outputs.
    int ksplit;
    int64_t kb_per_split;
    float *partial;
};

// (batch, first row, first column) of tile t: batches in order, each
// batch's tiles raster-grouped by group_m tile rows.
__device__ __forceinline__ void rowa_tile(const RArgs &args, int64_t t, int bn, int64_t &batch, int64_t &m0,
                                          int64_t &n0) {
    const int64_t per_batch = args.tiles_m * args.tiles_n;
    batch = t / per_batch;
    const int64_t tb = t - batch * per_batch;
    const int64_t span = args.group_m * args.tiles_n;
    const int64_t g = tb / span;
    const int64_t first = g * args.group_m;
    const int64_t gm = args.tiles_m - first < args.group_m ? args.tiles_m - first : args.group_m;
    const int64_t r = tb - g * span;
    m0 = (first + r % gm) * kBM;
    n0 = (r / gm) * bn;
}

// Work unit u of the persistent form: its tile (rowa_tile), split and k
// blocks [kb0, kb0 + nk).
__device__ __forceinline__ void rowa_unit(const RArgs &args, int64_t u, int bn, int64_t ktiles_all,
                                          int64_t &batch, int64_t &m0, int64_t &n0, int64_t &split, int64_t &kb0,
                                          int64_t &nk) {
    split = 0;
    kb0 = 0;
    nk = ktiles_all;
    if (args.ksplit > 1) {
        const int64_t per_split = args.tiles / args.ksplit;
        split = u / per_split;
        u -= split * per_split;
        kb0 = split * args.kb_per_split;
        nk = ktiles_all - kb0 < args.kb_per_split ? ktiles_all - kb0 : args.kb_per_split;
        if (nk < 0) nk = 0;
    }
    rowa_tile(args, u, bn, batch, m0, n0);
}

template <int WN, bool XP>
struct RowaCfg {
    static constexpr int BN = WN * (kTN / 4) * 32;  // 256 or 128
    static constexpr int WARPS = kWM * WN;
    static constexpr int THREADS = WARPS * 32;
    static constexpr int STAGES = WN == 4 ? 4 : 3;
    static constexpr int MIN_BLOCKS = WN == 4 ? 1 : 2;
    static constexpr int B_STAGE_F = kBK * BN;
    static constexpr uint32_t STAGE_BYTES = (kAStageF + B_STAGE_F) * 4;
    static constexpr int XPOSE_BYTES = XP ? 2 * kAStageF * 4 : 0;  // two transposed A tiles
    static constexpr int SMEM = STAGES * STAGE_BYTES + XPOSE_BYTES + 1024 + 256;
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Barrier 1 over `threads` threads that returns whether `pred` held in all of
// them (bar.red.and): every thread reaches it each k-block, failed waits
// included, so no warp can be left waiting on warps that gave up.
__device__ __forceinline__ bool bar1_and(bool pred, int threads) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(out)
        : "r"(pred ? 1u : 0u), "r"(threads)
        : "memory");
    return out != 0;
}

// XP = true: the warps transpose each landed
// A tile into At_s[k][m] (two buffers, alternating by k-block) before the
// FFMA loop reads it, so A fragments are 16-byte loads of four rows as in
// sgemm_tma_kernel instead of four 4-byte loads; one barrier per k-block
// separates the transpose from the reads.  Same per-element arithmetic (and
// bits) as XP = false.
template <int WN, bool XP>
__global__ void __launch_bounds__(RowaCfg<WN, XP>::THREADS, RowaCfg<WN, XP>::MIN_BLOCKS)
    sgemm_tma_rowa_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          RArgs args) {
    using namespace sm100;
    using Cf = RowaCfg<WN, XP>;
    constexpr int S = Cf::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    float *As = reinterpret_cast<float *>(smem);  // stages of [128 m][32 k], swizzled
    float *Bs = As + S * kAStageF;                // stages of [32 k][BN n]
    float *At_s = reinterpret_cast<float *>(smem + S * Cf::STAGE_BYTES);  // XP: 2 x [32 k][128 m]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * Cf::STAGE_BYTES + Cf::XPOSE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 2 * S);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int64_t batch, m0, n0;
    rowa_tile(args, blockIdx.x, Cf::BN, batch, m0, n0);
    const int64_t ktiles = (args.K + kBK - 1) / kBK;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], Cf::WARPS);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    __syncthreads();

    const bool loader = tid == 0;
    int64_t issued = 0;
    auto issue = [&](int64_t kt) {
        const int s = static_cast<int>(kt % S);
        mbar_arrive_expect_tx(&full[s], Cf::STAGE_BYTES);
        tma_load_3d(As + s * kAStageF, &tmA, &full[s], static_cast<int32_t>(kt * kBK), static_cast<int32_t>(m0),
                    static_cast<int32_t>(batch));
        tma_load_3d(Bs + s * Cf::B_STAGE_F, &tmB, &full[s], static_cast<int32_t>(n0), static_cast<int32_t>(kt * kBK),
                    static_cast<int32_t>(batch));
        ++issued;
    };
    if (loader)
        for (int64_t kt = 0; kt < S && kt < ktiles; ++kt) issue(kt);

    const int wm = warp / WN, wn = warp % WN;
    const int ty = lane >> 3, tx = lane & 7;
    const int row0 = wm * (kTM / 4) * 16 + ty;  // this thread's rows: row0 + 4i (XP: row_base + 16q + j)
    const int row_base = wm * (kTM / 4) * 16 + ty * 4;
    const int col_base = wn * (kTN / 4) * 32 + tx * 4;
    // Swizzle of row r = row0 + 4i: (r % 8) = ty + 4 (i & 1); float k of that
    // row sits at r*32 + (k ^ (4 (r % 8))).
    const int swz_even = ty << 2, swz_odd = (ty + 4) << 2;

    float2 acc2[kTM / 2][kTN];
#pragma unroll
    for (int i = 0; i < kTM / 2; ++i)
#pragma unroll
        for (int j = 0; j < kTN; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
    auto acc_at = [&](int i, int j) -> float & { return (i & 1) ? acc2[i >> 1][j].y : acc2[i >> 1][j].x; };

    auto load_frags = [&](const float *as, const float *bs, int kk, float (&af)[kTM], float (&bf)[kTN]) {
        if constexpr (XP) {
#pragma unroll
            for (int q = 0; q < kTM / 4; ++q) {
                const float4 v = *reinterpret_cast<const float4 *>(as + kk * kBM + row_base + q * 16);
                af[q * 4 + 0] = v.x;
                af[q * 4 + 1] = v.y;
                af[q * 4 + 2] = v.z;
                af[q * 4 + 3] = v.w;
            }
        } else {
            const float *ae = as + row0 * 32 + (kk ^ swz_even);
            const float *ao = as + row0 * 32 + (kk ^ swz_odd);
#pragma unroll
            for (int i = 0; i < kTM; ++i) af[i] = (i & 1) ? ao[4 * i * 32] : ae[4 * i * 32];
        }
#pragma unroll
        for (int q = 0; q < kTN / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(bs + kk * Cf::BN + col_base + q * 32);
            bf[q * 4 + 0] = v.x;
            bf[q * 4 + 1] = v.y;
            bf[q * 4 + 2] = v.z;
            bf[q * 4 + 3] = v.w;
        }
    };

    bool ok = true;
    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int s = static_cast<int>(kt % S);
        const uint32_t ph = static_cast<uint32_t>((kt / S) & 1);
        bool w = ok && mbar_wait(&full[s], ph, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x34, args.wait_ns);
        w = __all_sync(0xffffffffu, w);
        const float *as;
        if constexpr (XP) {
            // A tile -> At_s[kt & 1] as [k][m]: thread q of 1024 moves the
            // 16-byte chunk c = q / 128 (k = 4c..4c+3) of row m = q % 128, so a
            // warp reads 32 rows (4 wavefronts, the swizzle spreads the chunks)
            // and writes 32 consecutive m of each k (conflict-free).
            float *at = At_s + (kt & 1) * kAStageF;
            if (w) {
                const float *src = As + s * kAStageF;
#pragma unroll
                for (int r = 0; r < 1024 / Cf::THREADS; ++r) {
                    const int q = r * Cf::THREADS + tid;
                    const int m = q & 127, c = q >> 7;
                    const float4 v = *reinterpret_cast<const float4 *>(src + m * 32 + ((c ^ (m & 7)) << 2));
                    at[(4 * c + 0) * kBM + m] = v.x;
                    at[(4 * c + 1) * kBM + m] = v.y;
                    at[(4 * c + 2) * kBM + m] = v.z;
                    at[(4 * c + 3) * kBM + m] = v.w;
                }
            }
            // Every warp's transpose is done (and every warp's wait held)
            // before any warp reads it; a warp arriving here has also finished
            // reading the buffer it overwrote, from two k-blocks ago.
            if (!bar1_and(w, Cf::THREADS)) {
                ok = false;
                break;
            }
            as = at;
        } else {
            if (!w) {
                ok = false;
                break;
            }
            as = As + s * kAStageF;
        }
        const float *bs = Bs + s * Cf::B_STAGE_F;
        float af[2][kTM], bf[2][kTN];
        load_frags(as, bs, 0, af[0], bf[0]);
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            if (kk + 1 < kBK) load_frags(as, bs, kk + 1, af[(kk + 1) & 1], bf[(kk + 1) & 1]);
            const float *a = af[kk & 1], *b = bf[kk & 1];
#pragma unroll
            for (int j = 0; j < kTN; ++j) {
                const float2 bb = make_float2(b[j], b[j]);
#pragma unroll
                for (int p = 0; p < kTM / 2; ++p)
                    acc2[p][j] = __ffma2_rn(make_float2(a[2 * p], a[2 * p + 1]), bb, acc2[p][j]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (loader && kt >= 1) {
            const int64_t done = kt - 1, next = done + S;
            if (next < ktiles) {
                const int ds = static_cast<int>(done % S);
                const uint32_t dph = static_cast<uint32_t>((done / S) & 1);
                if (!mbar_wait(&empty[ds], dph, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x33, args.wait_ns)) {
                    ok = false;
                } else {
                    issue(next);
                }
            }
        }
        if constexpr (XP) {
            // a failed refill reaches the other warps at the next barrier
            ok = __all_sync(0xffffffffu, ok);
        } else if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
        }
    }
    if (!ok) {
        if (loader && issued) {
            const int64_t first_pending = issued > S ? issued - S : 0;
            for (int64_t kt = first_pending; kt < issued; ++kt)
                mbar_wait_drain(&full[kt % S], static_cast<uint32_t>((kt / S) & 1), 1000000000ull);
        }
        return;
    }

    float *Cb = args.C + batch * args.sC;
    const bool read_c = args.beta != 0.0f;
#pragma unroll
    for (int i = 0; i < kTM; ++i) {
        const int64_t row = m0 + (XP ? row_base + (i >> 2) * 16 + (i & 3) : row0 + 4 * i);
        if (row >= args.M) continue;
        float *crow = Cb + row * args.N;
#pragma unroll
        for (int gj = 0; gj < kTN / 4; ++gj) {
            const int64_t col = n0 + col_base + gj * 32;
            if (col >= args.N) continue;  // N % 4 == 0: the 4-vector is all in or all out
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = args.alpha * acc_at(i, gj * 4 + e);
            if (read_c) {
                const float4 old = *reinterpret_cast<const float4 *>(crow + col);
                o[0] = fmaf(args.beta, old.x, o[0]);
                o[1] = fmaf(args.beta, old.y, o[1]);
                o[2] = fmaf(args.beta, old.z, o[2]);
                o[3] = fmaf(args.beta, old.w, o[3]);
            }
            if (args.bias || args.relu) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (args.bias) o[e] += args.bias[col + e];
                    if (args.relu) o[e] = o[e] > 0.0f ? o[e] : 0.0f;
                }
            }
            *reinterpret_cast<float4 *>(crow + col) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

// Split-K finish: C = alpha * (P_0 + P_1 + ... + P_{S-1}) (+ beta * C, + bias,
// ReLU), the partial sums added in split order -- the same bits on every run
// and for every tiling of the output.  4 elements per thread (N % 4 == 0).
__global__ void __launch_bounds__(256) sgemm_splitk_reduce_kernel(const float *__restrict__ P, int S, int64_t M,
                                                                  int64_t N, float *__restrict__ C, float alpha,
                                                                  float beta, const float *__restrict__ bias, int relu) {
    const int64_t MN = M * N;
    for (int64_t q = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; q < MN;
         q += static_cast<int64_t>(gridDim.x) * blockDim.x * 4) {
        float4 s = *reinterpret_cast<const float4 *>(P + q);
        for (int i = 1; i < S; ++i) {
            const float4 v = *reinterpret_cast<const float4 *>(P + i * MN + q);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        float o[4] = {alpha * s.x, alpha * s.y, alpha * s.z, alpha * s.w};
        if (beta != 0.0f) {
            const float4 old = *reinterpret_cast<const float4 *>(C + q);
            o[0] = fmaf(beta, old.x, o[0]);
            o[1] = fmaf(beta, old.y, o[1]);
            o[2] = fmaf(beta, old.z, o[2]);
            o[3] = fmaf(beta, old.w, o[3]);
        }
        if (bias || relu) {
            const int64_t col = q % N;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (bias) o[e] += bias[col + e];
                if (relu) o[e] = o[e] > 0.0f ? o[e] : 0.0f;
            }
        }
        *reinterpret_cast<float4 *>(C + q) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// Warp-specialised persistent form of the XP kernel: two FFMA warpgroups and a
// producer warpgroup (384 threads launched at 168 registers each, 64512 in
// all; the producer warpgroup gives up all but 56 per thread with
// setmaxnreg.dec and the FFMA warpgroups take 224 with setmaxnreg.inc:
// 128 x 56 + 256 x 224 = 64512, the launch's own total, so the increase never
// waits).  CTA b takes tiles b, b + gridDim.x, ...; the producer's
// lane 0 streams the k-blocks of all of them through the 4-stage ring,
// waiting only on the "empty" barriers, so the next tile's first stages land
// while the FFMA warps finish and store the current one, and none of the
// loading bookkeeping sits in the FFMA warps.  Same per-element arithmetic
// (and bits) as the other forms.
//   PX = false: the FFMA warps transpose each A tile into At_s, meet at a
//     256-thread barrier (the producer never joins it), run the FFMA loop and
//     release the stage.
//   PX = true: the producer warpgroup's other three warps transpose each
//     landed A tile into At_s (two buffers, k-block g into buffer g & 1) and
//     arrive on that buffer's "xfull" barrier; the FFMA warps wait on it (and
//     on the stage's "full" barrier, for B), run the FFMA loop and arrive on
//     "empty" (the stage) and "xempty" (the buffer).  The FFMA warps then meet
//     no CTA-wide barrier, as in sgemm_tma_kernel.
template <bool PX>
__global__ void __launch_bounds__(384, 1)
    sgemm_tma_rowa_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             RArgs args) {
    using namespace sm100;
    using Cf = RowaCfg<4, true>;
    constexpr int S = Cf::STAGES;
    constexpr int NC = Cf::THREADS;  // FFMA threads (8 warps)
    constexpr int NX = 96;           // PX: transposing threads (producer warps 1-3)
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    float *As = reinterpret_cast<float *>(smem);
    float *Bs = As + S * kAStageF;
    float *At_s = reinterpret_cast<float *>(smem + S * Cf::STAGE_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * Cf::STAGE_BYTES + Cf::XPOSE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *xfull = bars + 2 * S;      // PX: At_s buffer b transposed
    uint64_t *xempty = bars + 2 * S + 2; // PX: At_s buffer b read by all FFMA warps
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 2 * S + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t ktiles = (args.K + kBK - 1) / kBK;
    const int64_t ntiles = (args.tiles - static_cast<int64_t>(blockIdx.x) + gridDim.x - 1) / gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], Cf::WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&xfull[b], NX / 32);
            mbar_init(&xempty[b], Cf::WARPS);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    __syncthreads();

    if (warp >= Cf::WARPS) {
        // ------------------------------------------------ producer warpgroup
        asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
        if (PX && warp > Cf::WARPS) {
            // A transposer: k-block g's landed A tile ([128 m][32 k], 128-byte
            // swizzle) into At_s buffer g & 1 as [32 k][128 m].
            const int xt = tid - NC - 32;
            int64_t g = 0;
            for (int64_t ti = 0; ti < ntiles; ++ti) {
                int64_t batch, m0, n0, split, kb0, nk;
                rowa_unit(args, blockIdx.x + ti * gridDim.x, Cf::BN, ktiles, batch, m0, n0, split, kb0, nk);
                bool w = true;
                for (int64_t kt = 0; kt < nk && w; ++kt, ++g) {
                    const int s = static_cast<int>(g % S), b = static_cast<int>(g & 1);
                    w = mbar_wait(&full[s], static_cast<uint32_t>((g / S) & 1), abort_flag, args.status,
                                  B2B_DEVSTAT_TIMEOUT | 0x37, args.wait_ns);
                    if (w && g >= 2)
                        w = mbar_wait(&xempty[b], static_cast<uint32_t>(((g >> 1) - 1) & 1), abort_flag, args.status,
                                      B2B_DEVSTAT_TIMEOUT | 0x38, args.wait_ns);
                    w = __all_sync(0xffffffffu, w);
                    if (!w) break;
                    const float *src = As + s * kAStageF;
                    float *at = At_s + b * kAStageF;
#pragma unroll 1
                    for (int q = xt; q < 1024; q += NX) {
                        const int m = q & 127, c = q >> 7;
                        const float4 v = *reinterpret_cast<const float4 *>(src + m * 32 + ((c ^ (m & 7)) << 2));
                        at[(4 * c + 0) * kBM + m] = v.x;
                        at[(4 * c + 1) * kBM + m] = v.y;
                        at[(4 * c + 2) * kBM + m] = v.z;
                        at[(4 * c + 3) * kBM + m] = v.w;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xfull[b]);
                }
                if (!w) break;
            }
            return;
        }
        if (warp == Cf::WARPS && lane == 0) {
            int64_t g = 0;
            bool ok = true;
            for (int64_t ti = 0; ti < ntiles && ok; ++ti) {
                int64_t batch, m0, n0, split, kb0, nk;
                rowa_unit(args, blockIdx.x + ti * gridDim.x, Cf::BN, ktiles, batch, m0, n0, split, kb0, nk);
                for (int64_t kt = 0; kt < nk; ++kt, ++g) {
                    const int s = static_cast<int>(g % S);
                    if (g >= S && !mbar_wait(&empty[s], static_cast<uint32_t>((g / S - 1) & 1), abort_flag,
                                             args.status, B2B_DEVSTAT_TIMEOUT | 0x35, args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], Cf::STAGE_BYTES);
                    tma_load_3d(As + s * kAStageF, &tmA, &full[s], static_cast<int32_t>((kb0 + kt) * kBK),
                                static_cast<int32_t>(m0), static_cast<int32_t>(batch));
                    tma_load_3d(Bs + s * Cf::B_STAGE_F, &tmB, &full[s], static_cast<int32_t>(n0),
                                static_cast<int32_t>((kb0 + kt) * kBK), static_cast<int32_t>(batch));
                }
            }
            if (!ok && g > 0) {
                // loads in flight complete on their full barriers before the
                // CTA's shared memory goes away
                const int64_t first_pending = g > S ? g - S : 0;
                for (int64_t q = first_pending; q < g; ++q)
                    mbar_wait_drain(&full[q % S], static_cast<uint32_t>((q / S) & 1), 1000000000ull);
            }
        }
        return;
    }

    // ---------------------------------------------------- FFMA warps
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
    const int wm = warp / 4, wn = warp % 4;
    const int ty = lane >> 3, tx = lane & 7;
    const int row_base = wm * (kTM / 4) * 16 + ty * 4;
    const int col_base = wn * (kTN / 4) * 32 + tx * 4;
    float2 acc2[kTM / 2][kTN];
    auto acc_at = [&](int i, int j) -> float & { return (i & 1) ? acc2[i >> 1][j].y : acc2[i >> 1][j].x; };
    auto load_frags = [&](const float *as, const float *bs, int kk, float (&af)[kTM], float (&bf)[kTN]) {
#pragma unroll
        for (int q = 0; q < kTM / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(as + kk * kBM + row_base + q * 16);
            af[q * 4 + 0] = v.x;
            af[q * 4 + 1] = v.y;
            af[q * 4 + 2] = v.z;
            af[q * 4 + 3] = v.w;
        }
#pragma unroll
        for (int q = 0; q < kTN / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4 *>(bs + kk * Cf::BN + col_base + q * 32);
            bf[q * 4 + 0] = v.x;
            bf[q * 4 + 1] = v.y;
            bf[q * 4 + 2] = v.z;
            bf[q * 4 + 3] = v.w;
        }
    };
    int64_t g = 0;
    bool ok = true;
#pragma unroll 1
    for (int64_t ti = 0; ti < ntiles && ok; ++ti) {
#pragma unroll
        for (int i = 0; i < kTM / 2; ++i)
#pragma unroll
            for (int j = 0; j < kTN; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
        int64_t nk;
        {
            int64_t b_, m_, n_, s_, k_;
            rowa_unit(args, blockIdx.x + ti * gridDim.x, Cf::BN, ktiles, b_, m_, n_, s_, k_, nk);
        }
        for (int64_t kt = 0; kt < nk; ++kt, ++g) {
            const int s = static_cast<int>(g % S);
            float *at = At_s + (g & 1) * kAStageF;
            if constexpr (PX) {
                bool w = mbar_wait(&xfull[g & 1], static_cast<uint32_t>((g >> 1) & 1), abort_flag, args.status,
                                   B2B_DEVSTAT_TIMEOUT | 0x39, args.wait_ns);
                if (w)
                    w = mbar_wait(&full[s], static_cast<uint32_t>((g / S) & 1), abort_flag, args.status,
                                  B2B_DEVSTAT_TIMEOUT | 0x36, args.wait_ns);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
            } else {
                bool w = mbar_wait(&full[s], static_cast<uint32_t>((g / S) & 1), abort_flag, args.status,
                                   B2B_DEVSTAT_TIMEOUT | 0x36, args.wait_ns);
                w = __all_sync(0xffffffffu, w);
                if (w) {
                    const float *src = As + s * kAStageF;
#pragma unroll
                    for (int r = 0; r < 1024 / NC; ++r) {
                        const int q = r * NC + tid;
                        const int m = q & 127, c = q >> 7;
                        const float4 v = *reinterpret_cast<const float4 *>(src + m * 32 + ((c ^ (m & 7)) << 2));
                        at[(4 * c + 0) * kBM + m] = v.x;
                        at[(4 * c + 1) * kBM + m] = v.y;
                        at[(4 * c + 2) * kBM + m] = v.z;
                        at[(4 * c + 3) * kBM + m] = v.w;
                    }
                }
                if (!bar1_and(w, NC)) {
                    ok = false;
                    break;
                }
            }
            const float *bs = Bs + s * Cf::B_STAGE_F;
            float af[2][kTM], bf[2][kTN];
            load_frags(at, bs, 0, af[0], bf[0]);
#pragma unroll
            for (int kk = 0; kk < kBK; ++kk) {
                if (kk + 1 < kBK) load_frags(at, bs, kk + 1, af[(kk + 1) & 1], bf[(kk + 1) & 1]);
                const float *a = af[kk & 1], *b = bf[kk & 1];
#pragma unroll
                for (int j = 0; j < kTN; ++j) {
                    const float2 bb = make_float2(b[j], b[j]);
#pragma unroll
                    for (int p = 0; p < kTM / 2; ++p)
                        acc2[p][j] = __ffma2_rn(make_float2(a[2 * p], a[2 * p + 1]), bb, acc2[p][j]);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[s]);
                if (PX) mbar_arrive(&xempty[g & 1]);
            }
        }
        if (!ok) break;
        int64_t batch, m0, n0, split, kb0, nk_;
        rowa_unit(args, blockIdx.x + ti * gridDim.x, Cf::BN, ktiles, batch, m0, n0, split, kb0, nk_);
        if (args.ksplit > 1) {
            // raw sums of this k range; the reduce applies alpha, beta, bias, ReLU
            float *P = args.partial + split * args.M * args.N;
#pragma unroll
            for (int i = 0; i < kTM; ++i) {
                const int64_t row = m0 + row_base + (i >> 2) * 16 + (i & 3);
                if (row >= args.M) continue;
#pragma unroll
                for (int gj = 0; gj < kTN / 4; ++gj) {
                    const int64_t col = n0 + col_base + gj * 32;
                    if (col >= args.N) continue;
                    *reinterpret_cast<float4 *>(P + row * args.N + col) =
                        make_float4(acc_at(i, gj * 4 + 0), acc_at(i, gj * 4 + 1), acc_at(i, gj * 4 + 2),
                                    acc_at(i, gj * 4 + 3));
                }
            }
            continue;
        }
        float *Cb = args.C + batch * args.sC;
        const bool read_c = args.beta != 0.0f;
#pragma unroll
        for (int i = 0; i < kTM; ++i) {
            const int64_t row = m0 + row_base + (i >> 2) * 16 + (i & 3);
            if (row >= args.M) continue;
            float *crow = Cb + row * args.N;
#pragma unroll
            for (int gj = 0; gj < kTN / 4; ++gj) {
                const int64_t col = n0 + col_base + gj * 32;
                if (col >= args.N) continue;  // N % 4 == 0: the 4-vector is all in or all out
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = args.alpha * acc_at(i, gj * 4 + e);
                if (read_c) {
                    const float4 old = *reinterpret_cast<const float4 *>(crow + col);
                    o[0] = fmaf(args.beta, old.x, o[0]);
                    o[1] = fmaf(args.beta, old.y, o[1]);
                    o[2] = fmaf(args.beta, old.z, o[2]);
                    o[3] = fmaf(args.beta, old.w, o[3]);
                }
                if (args.bias || args.relu) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (args.bias) o[e] += args.bias[col + e];
                        if (args.relu) o[e] = o[e] > 0.0f ? o[e] : 0.0f;
                    }
                }
                *reinterpret_cast<float4 *>(crow + col) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// At[k][m] = A[m][k]: 32 x 32 tiles through shared memory (padded row).
__global__ void __launch_bounds__(256) transpose_f32_kernel(const float *__restrict__ A, float *__restrict__ At,
                                                            int64_t M, int64_t K) {
    __shared__ float tile[32][33];
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 32, k0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
        const int64_t m = m0 + j, k = k0 + tx;
        if (m < M && k < K) tile[j][tx] = A[m * K + k];
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < 32; j += 8) {
        const int64_t k = k0 + j, m = m0 + tx;
        if (k < K && m < M) At[k * M + m] = tile[tx][j];
    }
}

}  // namespace

namespace b2b {

bool sgemm_tma_eligible(int64_t M, int64_t N, int64_t K, const void *A, const void *B, const void *C,
                        bool any_size) {
    // N >= 1024 keeps the transpose below ~3.5% of the GEMM's time; any_size
    // drops that preference (and M >= 128) for calls that must take this
    // kernel (the tiles of a split host-slice call).
    return M % 4 == 0 && N % 4 == 0 && aligned16(A) && aligned16(B) && aligned16(C) &&
           (any_size || (M >= kBM && N >= 1024)) && K >= kBK && (K + kBK - 1) / kBK < (int64_t(1) << 30) &&
           M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31) && K <= 65535LL * 32;
}

// Split-K factor for an M x N x K SGEMM on the TMA-fed kernel: the S in
// {1, 2, 3, 4, 6, 8} with the least estimated time, where the GEMM costs
// waves x k-blocks per CTA (a 128 x 256 x 32 k-block takes ~5.2 us at the
// kernel's FFMA rate) and a split adds the reduce (reading S partials and
// writing C, 4 (S + 1) M N bytes at ~6 TB/s: the partials' writes hide under
// the compute-bound GEMM) plus a launch.  Each split keeps at least 8
// k-blocks.  Taken when it saves 5% or more: grids under one wave (1024^3:
// 32 tiles, S = 4) and wave counts just past a whole number (4096^3: 3.46
// waves, S = 2; 4096 x 4096 x 1024, S = 2: 54.3 vs 47.8 TFLOP/s unsplit;
// 4096 x 1024 x 4096, S = 8: 56.1 vs 52.7; 2048 x 4096 x 2048, S = 4: 55.5
// vs 50.8).
int sgemm_ksplit(int sm_count, int64_t M, int64_t N, int64_t K) {
    const double tiles = static_cast<double>(((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN));
    const int64_t kt = (K + kBK - 1) / kBK;
    const double kb_us = 5.2;
    auto est = [&](int S) {
        const double waves = std::ceil(tiles * S / sm_count);
        const double kbs = static_cast<double>((kt + S - 1) / S);
        double t = waves * kbs * kb_us;
        if (S > 1) t += 4.0 * (S + 1) * static_cast<double>(M) * static_cast<double>(N) / 6e12 * 1e6 + 4.0;
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

int launch_sgemm_tma(b2b_handle *h, int64_t M, int64_t N, int64_t K, float alpha, float beta, const float *A,
                     const float *B, float *C, const float *bias, int relu, int pack) {
    const int pk = pack == 1 || pack == 2 ? pack : 0;
    auto kern = pk == 1 ? sgemm_tma_kernel<1> : pk == 2 ? sgemm_tma_kernel<2> : sgemm_tma_kernel<0>;
    // The split: forced by the caller (a host-slice call's tiles take the
    // whole GEMM's, so every tile sums the same k ranges), else chosen here.
    const int64_t ktiles = (K + kBK - 1) / kBK;
    int S = h->sgemm_ksplit_forced > 0 ? h->sgemm_ksplit_forced : sgemm_ksplit(h->sm_count, M, N, K);
    if (S > ktiles) S = static_cast<int>(ktiles);
    if (S < 1) S = 1;
    const int64_t kbps = (ktiles + S - 1) / S;
    const size_t part_bytes = S > 1 ? static_cast<size_t>(S) * static_cast<size_t>(M) * static_cast<size_t>(N) * 4 : 0;
    auto reduce = [&](const float *partial) -> int {
        const int64_t quads = M * N / 4;
        int64_t blocks = (quads + 255) / 256;
        const int64_t cap = 8LL * h->sm_count;
        if (blocks > cap) blocks = cap;
        sgemm_splitk_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, h->stream>>>(partial, S, M, N, C, alpha,
                                                                                          beta, bias, relu);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? B2B_OK : fail_cuda(e, "sgemm split-K reduce launch");
    };
    // The persistent warp-specialised kernel on row-major A, whose producer
    // warpgroup transposes A in shared memory: no transpose pass through
    // global memory, workspace only for a split's partial sums, the same bits
    // (each split sums its k range from zero, as below).
    if (pk == 1 && h->sgemm_variant == 0 && sgemm_tma_rowa_eligible(M, N, K, M * K, K * N, M * N, 1, A, B, C)) {
        float *partial = nullptr;
        if (S > 1) {
            void *pws = nullptr;
            if (int rc = workspace(h, part_bytes, &pws)) return rc;
            partial = static_cast<float *>(pws);
        }
        if (int rc = launch_sgemm_tma_rowa(h, M, N, K, alpha, beta, A, M * K, B, K * N, C, M * N, 1, bias, relu, S,
                                           kbps, partial))
            return rc;
        return S > 1 ? reduce(partial) : B2B_OK;
    }
    const size_t at_bytes = (static_cast<size_t>(M) * static_cast<size_t>(K) * 4 + 255) / 256 * 256;
    void *ws = nullptr;
    if (int rc = workspace(h, at_bytes + part_bytes, &ws)) return rc;
    float *At = static_cast<float *>(ws);
    float *partial = S > 1 ? reinterpret_cast<float *>(static_cast<char *>(ws) + at_bytes) : nullptr;
    const dim3 tgrid(static_cast<unsigned>((M + 31) / 32), static_cast<unsigned>((K + 31) / 32));
    transpose_f32_kernel<<<tgrid, 256, 0, h->stream>>>(A, At, M, K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgemm transpose launch");
    CUtensorMap tmAt, tmB;
    int rc = encode_tma_2d(&tmAt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, At, static_cast<uint64_t>(K),
                           static_cast<uint64_t>(M), kBM, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tma_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, B, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                       kBN, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    {
        static std::mutex mu;
        static bool attr_set[3][64] = {};
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[pk][h->device & 63]) {
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
            if (e != cudaSuccess) return fail_cuda(e, "sgemm smem attribute");
            attr_set[pk][h->device & 63] = true;
        }
    }
    const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    if (tiles * S > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "sgemm: grid exceeds 2^31-1 tiles");
    SArgs args{C, M, N, K, alpha, beta, bias, relu, h->d_status, h->wait_limit_ns,
               h->sgemm_group_m > 0 ? h->sgemm_group_m : kGroupMSingle, S, kbps, partial};
    kern<<<static_cast<unsigned>(tiles * S), kThreads, kSmem, h->stream>>>(tmAt, tmB, args);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "sgemm TMA launch");
    return S > 1 ? reduce(partial) : B2B_OK;
}

bool sgemm_tma_rowa_eligible(int64_t M, int64_t N, int64_t K, int64_t sA, int64_t sB, int64_t sC, int64_t batch,
                             const void *A, const void *B, const void *C) {
    // 16-byte row and batch pitches for the tensor maps and the float4 C
    // accesses; 32-bit TMA coordinates.
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return false;
    if (K % 4 || N % 4 || sA % 4 || sB % 4 || sC % 4) return false;
    if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return false;
    if (batch > 1 && (sA < M * K || sB < K * N || sC < M * N)) return false;
    const int64_t lim = int64_t(1) << 31;
    if (M >= lim || N >= lim || K >= lim || batch >= lim) return false;
    const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + 127) / 128) * batch;  // the 128-wide form's count
    return tiles < lim;
}

// Whether a single SGEMM of the given kernel variant takes the TMA-fed path:
// by default (variant 0) the persistent row-major-A kernel wherever it
// applies (N and K multiples of 4, 16-byte aligned operands; no size limit,
// since it needs no transpose pass to amortise), else the transposed-A
// kernel where sgemm_tma_eligible allows it; variants 20-22 force the
// transposed-A kernel's forms.  run_sgemm, the host-slice call's split and
// b2b_sgemm_splits all decide with this, so they agree on the split.
bool sgemm_tma_path(int variant, int64_t M, int64_t N, int64_t K, const void *A, const void *B, const void *C,
                    bool any_size) {
    if (variant == 0 && sgemm_tma_rowa_eligible(M, N, K, M * K, K * N, M * N, 1, A, B, C)) return true;
    if (variant != 0 && !(variant >= 20 && variant <= 22)) return false;
    return sgemm_tma_eligible(M, N, K, A, B, C, any_size);
}

namespace {

template <int WN, bool XP>
int launch_rowa(b2b_handle *h, const CUtensorMap &tmA, const CUtensorMap &tmB, RArgs args, int64_t batch) {
    using Cf = RowaCfg<WN, XP>;
    {
        static std::mutex mu;
        static bool attr_set[64] = {};
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[h->device & 63]) {
            cudaError_t e =
                cudaFuncSetAttribute(sgemm_tma_rowa_kernel<WN, XP>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM);
            if (e != cudaSuccess) return fail_cuda(e, "sgemm (row-major A) smem attribute");
            attr_set[h->device & 63] = true;
        }
    }
    args.tiles_n = (args.N + Cf::BN - 1) / Cf::BN;
    const int64_t blocks = args.tiles_m * args.tiles_n * batch;
    if (blocks > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "sgemm: grid exceeds 2^31-1 tiles");
    sgemm_tma_rowa_kernel<WN, XP><<<static_cast<unsigned>(blocks), Cf::THREADS, Cf::SMEM, h->stream>>>(tmA, tmB, args);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "sgemm (row-major A) TMA launch");
}

template <bool PX>
int launch_rowa_ws(b2b_handle *h, const CUtensorMap &tmA, const CUtensorMap &tmB, RArgs args, int64_t batch) {
    using Cf = RowaCfg<4, true>;
    {
        static std::mutex mu;
        static bool attr_set[64] = {};
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set[h->device & 63]) {
            cudaError_t e = cudaFuncSetAttribute(sgemm_tma_rowa_ws_kernel<PX>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM);
            if (e != cudaSuccess) return fail_cuda(e, "sgemm (row-major A, persistent) smem attribute");
            attr_set[h->device & 63] = true;
        }
    }
    args.tiles_n = (args.N + Cf::BN - 1) / Cf::BN;
    args.tiles = args.tiles_m * args.tiles_n * batch * (args.ksplit > 1 ? args.ksplit : 1);
    if (args.tiles > 0x7fffffffLL) return fail(B2B_ERR_INVALID_ARG, "sgemm: grid exceeds 2^31-1 tiles");
    // one CTA per SM: its shared memory allows no second one
    const int64_t grid = args.tiles < h->sm_count ? args.tiles : h->sm_count;
    sgemm_tma_rowa_ws_kernel<PX><<<static_cast<unsigned>(grid), 384, Cf::SMEM, h->stream>>>(tmA, tmB, args);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "sgemm (row-major A, persistent) TMA launch");
}

}  // namespace

int launch_sgemm_tma_rowa(b2b_handle *h, int64_t M, int64_t N, int64_t K, float alpha, float beta, const float *A,
                          int64_t sA, const float *B, int64_t sB, float *C, int64_t sC, int64_t batch,
                          const float *bias, int relu, int ksplit, int64_t kb_per_split, float *partial) {
    if (ksplit > 1 && (batch != 1 || h->sgemm_variant != 0 || partial == nullptr || kb_per_split <= 0))
        return fail(B2B_ERR_INVALID_ARG, "sgemm: split-K takes the persistent kernel on one GEMM only");
    if (batch == 1) {  // a single GEMM: the batch pitch is never used, keep it a legal multiple of 16
        sA = M * K;
        sB = K * N;
        sC = M * N;
    }
    const int64_t tiles_m = (M + kBM - 1) / kBM;
    // The persistent warp-specialised kernel, 128 x 256 tiles with A
    // transposed in shared memory by the producer warpgroup (4096 x 256^3:
    // 58.8 TFLOP/s, against 56.5 when the FFMA warps transpose it behind a
    // CTA-wide barrier per k-block, variant 27; 54.3 for the one-CTA-per-tile
    // form of variant 26 and 54.1 for the 4-byte A fragments of variant 24);
    // variant 25 takes the 128 x 128 form
    // (two CTAs per SM), which measured slower (51.5 vs 54.0): half the B tile
    // per CTA costs more L2 -> SM traffic per flop than overlapping two CTAs'
    // prologues and epilogues saves.
    const bool narrow = h->sgemm_variant == 25;
    const bool plain = h->sgemm_variant == 24;
    const bool per_tile = h->sgemm_variant == 26;
    const int bn = narrow ? RowaCfg<2, false>::BN : RowaCfg<4, true>::BN;
    CUtensorMap tmA, tmB;
    int rc = encode_tma_3d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, A, static_cast<uint64_t>(K),
                           static_cast<uint64_t>(M), static_cast<uint64_t>(batch), static_cast<uint64_t>(K) * 4,
                           static_cast<uint64_t>(sA) * 4, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tma_3d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                       static_cast<uint64_t>(batch), static_cast<uint64_t>(N) * 4, static_cast<uint64_t>(sB) * 4, bn,
                       kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    const int64_t group_m = batch > 1 ? kGroupM : (h->sgemm_group_m > 0 ? h->sgemm_group_m : kGroupMSingleWs);
    RArgs args{C,       M,          N,           K,    sC,      tiles_m, 0,      alpha,
               beta,    bias,       relu,        h->d_status, h->wait_limit_ns, 0, group_m,
               ksplit > 1 ? ksplit : 1, kb_per_split, partial};
    if (narrow) return launch_rowa<2, false>(h, tmA, tmB, args, batch);
    if (plain) return launch_rowa<4, false>(h, tmA, tmB, args, batch);
    if (per_tile) return launch_rowa<4, true>(h, tmA, tmB, args, batch);
    if (h->sgemm_variant == 27) return launch_rowa_ws<false>(h, tmA, tmB, args, batch);
    return launch_rowa_ws<true>(h, tmA, tmB, args, batch);
}

}  // namespace b2b
