// hgemm_tc.cu -- HGEMM on the 5th-generation tensor cores (tcgen05 + TMEM +
// TMA), f16 in, f32 accumulate, f16 out.
//
// Operation: C <- alpha * A * B + beta * C, row-major A[M x K], B[K x N],
// C[M x N] in IEEE binary16, the operation of cublas-rs's hgemm_half
// (crates/cublas-l3/src/hgemm.rs:55-125) and the slot its tensor-core variant
// leaves as todo! (hgemm.rs:189-193).  Accumulation is f32 as in the
// reference; the f16 result is rounded to nearest even (the reference
// truncates, hgemm.rs:34-51).
//
// Design (one CTA per SM, persistent):
//   * CTA tile 128 x 256, k-block 64, one tcgen05.mma.cta_group::1 of shape
//     M=128 N=256 K=16 per 16-wide k step, accumulators in TMEM.
//   * A tiles are K-major (rows of A are contiguous in k); B tiles are
//     MN-major (rows of B are contiguous in n) and are consumed as such
//     through the instruction descriptor's B-major bit, so B is never
//     transposed in memory.
//   * TMA loads both operands with 128-byte swizzle into a 4-stage ring
//     (48 KiB per stage), completing on per-stage "full" mbarriers; the MMA
//     warp frees a stage with tcgen05.commit on its "empty" mbarrier.
//   * Two TMEM accumulators (2 x 256 columns): the epilogue drains one tile
//     while the MMA warp fills the other.
//   * Warp roles: warp 0 = TMA producer, warp 1 = TMEM allocator + MMA
//     issuer, warps 2..5 = epilogue (TMEM -> registers -> alpha/beta -> f16
//     -> global).  Warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31.
//   * Every mbarrier wait is bounded; a wait that gives up records a status
//     code, raises the CTA's abort flag, and the roles drain their in-flight
//     TMA loads and MMAs before TMEM is freed and the CTA exits.
//   * No TMA multicast: each CTA loads its own tiles from this GPU's memory.
//
// Shapes that TMA cannot describe (K or N not a multiple of 8, or operands
// not 16-byte aligned) are copied into zero-padded workspace and run on the
// tensor cores when the GEMM is large enough to pay for the copies
// (launch_hgemm); small ones run hgemm_simt_kernel below, a plain CUDA-core
// kernel with the same arithmetic.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace {

namespace hg {
constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KiB
constexpr int B_BOX_N = 64;            // one TMA box of B: 64 (n) x 64 (k)
constexpr int B_BOX_BYTES = B_BOX_N * BK * 2;  // 8 KiB
constexpr int B_BYTES = BK * BN * 2;   // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = BN;           // f32 columns per accumulator
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int THREADS = 192;
constexpr int EPI_THREADS = 128;
constexpr int GROUP_M = 16;            // raster group for L2 reuse
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// Instruction descriptor: f16 x f16 -> f32, A K-major, B MN-major, 128 x 256.
constexpr uint32_t IDESC = sm100::idesc_f32acc(0, 0, 1, BM, BN);
}  // namespace hg

struct HgemmArgs {
    uint16_t *C;
    int M, N, K;
    float alpha, beta;
    int *status;
    uint64_t wait_ns;
    int group_m;  // pair kernels' raster group (pair-tile rows); 0 = the kernel's default
    // Fused all-gather (pair kernels, beta == 0): when ndst > 0 the epilogue
    // writes element (r, c) of this rank's panel to dst[d][r * ldc + col_off + c]
    // for every d -- each rank's full row-major C, peers' mapped through CUDA IPC.
    int ndst;
    int64_t ldc, col_off;
    uint16_t *dst[8];
    // With mc set, the gather goes through that NVLink multicast address
    // instead (one store reaches every rank's C); dst/ndst are then unused.
    uint16_t *mc;
    int rotate;  // fused all-gather: rotate the destination order per CTA pair
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int &tm, int &tn) {
    const int span = hg::GROUP_M * tiles_n;
    const int g = t / span;
    const int first = g * hg::GROUP_M;
    const int gm = min(tiles_m - first, hg::GROUP_M);
    const int r = t - g * span;
    tm = first + r % gm;
    tn = r / gm;
}

// Writes 32 consecutive f16 outputs of one row (alpha already applied to v):
// 4 x 16-byte stores when the whole chunk is in range, else element-wise.
__device__ __forceinline__ void store_c_chunk(uint16_t *crow, int col0, int N, float (&v)[32], bool read_c,
                                              float beta) {
    if (col0 + 32 <= N) {
        uint4 *dst = reinterpret_cast<uint4 *>(crow + col0);
        if (read_c) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint4 old = dst[j];
                const __half2 *oh = reinterpret_cast<const __half2 *>(&old);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float2 of = __half22float2(oh[e]);
                    v[j * 8 + e * 2 + 0] = fmaf(beta, of.x, v[j * 8 + e * 2 + 0]);
                    v[j * 8 + e * 2 + 1] = fmaf(beta, of.y, v[j * 8 + e * 2 + 1]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint4 o;
            __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(v[j * 8 + e * 2], v[j * 8 + e * 2 + 1]);
            dst[j] = o;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (col0 + i < N) {
                float x = v[i];
                if (read_c) x = fmaf(beta, __half2float(__ushort_as_half(crow[col0 + i])), x);
                crow[col0 + i] = __half_as_ushort(__float2half_rn(x));
            }
        }
    }
}

// Grouped raster over a tiles_m x tiles_n grid: `group` consecutive M tiles
// sweep the N tiles together, so their A and B panels stay in L2.
__device__ __forceinline__ void tile_coords_g(int t, int tiles_m, int tiles_n, int group, int &tm, int &tn) {
    const int span = group * tiles_n;
    const int g = t / span;
    const int first = g * group;
    const int gm = min(tiles_m - first, group);
    const int r = t - g * span;
    tm = first + r % gm;
    tn = r / gm;
}

__global__ void __launch_bounds__(hg::THREADS, 1)
    hgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    HgemmArgs args) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzle atoms need 1024-byte aligned tiles.
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t *sA = smem;                                   // STAGES x 16 KiB
    uint8_t *sB = smem + hg::STAGES * hg::A_BYTES;        // STAGES x 32 KiB
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + hg::STAGES * hg::STAGE_BYTES);
    uint64_t *full = bars;                 // [STAGES]
    uint64_t *empty = bars + hg::STAGES;   // [STAGES]
    uint64_t *tfull = bars + 2 * hg::STAGES;       // [2]
    uint64_t *tempty = bars + 2 * hg::STAGES + 2;  // [2]
    uint64_t *drain = bars + 2 * hg::STAGES + 4;   // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * hg::STAGES + 5);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tiles_m = (args.M + hg::BM - 1) / hg::BM;
    const int tiles_n = (args.N + hg::BN - 1) / hg::BN;
    const int num_tiles = tiles_m * tiles_n;
    const int kblocks = (args.K + hg::BK - 1) / hg::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < hg::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], hg::EPI_THREADS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, hg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;  // loads issued (for draining on abort)
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, tiles_m, tiles_n, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 1,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], hg::STAGE_BYTES);
                    uint8_t *a_dst = sA + stage * hg::A_BYTES;
                    uint8_t *b_dst = sB + stage * hg::B_BYTES;
                    tma_load_2d(a_dst, &tmA, &full[stage], kb * hg::BK, tm * hg::BM);
#pragma unroll
                    for (int j = 0; j < hg::BN / hg::B_BOX_N; ++j)
                        tma_load_2d(b_dst + j * hg::B_BOX_BYTES, &tmB, &full[stage], tn * hg::BN + j * hg::B_BOX_N,
                                    kb * hg::BK);
                    ++issued;
                    if (++stage == hg::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Drain: every stage whose last load was issued must see that
                // load land before the CTA may exit.
                const uint32_t n = issued < (uint32_t)hg::STAGES ? issued : (uint32_t)hg::STAGES;
                int s = stage;
                uint32_t ph = phase;
                for (uint32_t i = 0; i < n; ++i) {
                    if (--s < 0) {
                        s = hg::STAGES - 1;
                        ph ^= 1u;
                    }
                    mbar_wait_drain(&full[s], ph, 1000000000ull);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // One thread issues every tcgen05.mma and tcgen05.commit.
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued_any = false;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 2,
                               args.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * hg::ACC_COLS);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 3,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + stage * hg::A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * hg::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < hg::BK / 16; ++kk) {
                        // A: K-major SW128, 8-row atoms 1024 B apart; a 16-wide
                        // k step moves 32 B inside the swizzle row.
                        const uint64_t adesc = sdesc_sw128(a_base + kk * 32, 16, 1024);
                        // B: MN-major SW128, 64-wide n chunks one TMA box
                        // (8 KiB) apart, 8-row k groups 1024 B apart; a 16-wide
                        // k step moves 16 rows = 2048 B.
                        const uint64_t bdesc = sdesc_sw128(b_base + kk * 2048, hg::B_BOX_BYTES, 1024);
                        umma_f16(d_tmem, adesc, bdesc, hg::IDESC, (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(&empty[stage]);
                    issued_any = true;
                    if (++stage == hg::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok && issued_any) {
                // Drain: all MMAs this thread issued must finish before TMEM
                // is freed.
                umma_commit(drain);
                mbar_wait_drain(drain, 0, 1000000000ull);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;             // TMEM lane quarter
        const int row_in_tile = q * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const bool read_c = args.beta != 0.0f;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int tm, tn;
            tile_coords(t, tiles_m, tiles_n, tm, tn);
            bool ok = mbar_wait_sleepy(&tfull[acc], acc_phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 4, args.wait_ns);
            // tcgen05.ld is warp-collective: all lanes take the same branch.
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = tm * hg::BM + row_in_tile;
            const bool row_ok = row < args.M;
            uint16_t *crow = args.C + static_cast<int64_t>(row) * args.N;
#pragma unroll 1
            for (int c = 0; c < hg::BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tmem_base + lane_off + static_cast<uint32_t>(acc * hg::ACC_COLS + c * 32), r);
                tmem_ld_wait();
                if (c == hg::BN / 32 - 1) {
                    // All of this accumulator is in registers: hand it back.
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                const int col0 = tn * hg::BN + c * 32;
                if (!row_ok || col0 >= args.N) continue;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = args.alpha * __uint_as_float(r[i]);
                store_c_chunk(crow, col0, args.N, v, read_c, args.beta);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, hg::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  CTA r of the pair holds
// rows [128r, 128r+128) of the A tile and columns [128r, 128r+128) of the B
// tile in its own shared memory, and its 128 x 256 slice of the accumulator
// in its own TMEM.  Per CTA and 64-wide k-block that is 32 KiB of operands
// for 128x256x64 MACs (the single-CTA kernel moves 48 KiB for the same
// work), which is what relieves the L2 -> SM operand traffic.
//   * Both CTAs' TMA loads (.cta_group::2, no multicast) count their bytes on
//     the leader's (rank 0) "full" barrier, which expects 64 KiB per stage.
//   * The leader's single MMA thread issues every MMA of the pair and commits
//     to both CTAs' "empty" / "tmem full" barriers.
//   * The leader's "tmem empty" barriers count one arrival per epilogue warp
//     of both CTAs (8); the partner's warps arrive remotely.
//   * Epilogue with beta == 0: each warp moves its 32 TMEM lanes x 64 columns
//     to registers, scales, rounds to f16, writes them to a 4 KiB staging
//     buffer in the 128-byte-swizzled layout and issues one TMA store of the
//     32 x 64 box (two buffers per warp, recycled once the bulk group that
//     used them has read them).  That replaces 32-row-scattered 16-byte
//     stores; with beta != 0 C is read and written by the threads.
namespace hg2 {
// NSPLIT = number of N=256 MMAs per 16-wide k step.  1: 256 x 256 pair tiles,
// two 256-column TMEM accumulators (the epilogue overlaps the next tile).
// 2: 256 x 512 pair tiles (each MMA's A tile feeds two B halves), one
// 512-column accumulator; per CTA and k-block 48 KiB move for 128x512x64
// MACs, a quarter fewer operand bytes per flop than NSPLIT = 1, at the cost
// of an epilogue that the next tile's MMAs wait for.
template <int NSPLIT>
struct Cfg {
    static constexpr int BM = 128;              // rows per CTA (256 per pair)
    static constexpr int BN = 256 * NSPLIT;     // columns per pair tile
    static constexpr int BN_HALF = 128;         // B columns each CTA loads per MMA
    static constexpr int BK = 64;
    static constexpr int STAGES = NSPLIT == 1 ? 6 : 4;
    static constexpr int A_BYTES = BM * BK * 2;             // 16 KiB
    static constexpr int B_BOX_N = 64;
    static constexpr int B_BOX_BYTES = B_BOX_N * BK * 2;    // 8 KiB
    static constexpr int B_SPLIT_BYTES = BK * BN_HALF * 2;  // 16 KiB per MMA
    static constexpr int B_BYTES = NSPLIT * B_SPLIT_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int PAIR_STAGE_BYTES = 2 * STAGE_BYTES;
    static constexpr int ACC_COLS = BN;
    static constexpr int ACC_BUFS = NSPLIT == 1 ? 2 : 1;
    static constexpr int TMEM_COLS = ACC_BUFS * ACC_COLS;  // 512 either way
    static constexpr int EPI_WARPS_PAIR = 8;
    static constexpr int GROUP_M = 16;  // raster group, in 256-row pair tiles
    // Epilogue staging for the TMA-store path: two 4 KiB buffers (32 rows x
    // 64 f16 columns, 128-byte swizzle) per epilogue warp.
    static constexpr int EPI_BUF_BYTES = 32 * 64 * 2;
    static constexpr int EPI_BYTES = 4 * 2 * EPI_BUF_BYTES;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
    static constexpr uint32_t IDESC = sm100::idesc_f32acc(0, 0, 1, 256, 256);
    static_assert(TMEM_COLS == 512, "TMEM holds 512 columns");
    static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};
constexpr int THREADS = 192;
}  // namespace hg2

// HALVES (256 x 512 tiles only): the accumulator is released in two
// 256-column halves.  The epilogue arrives on tempty[0] once it has read
// columns 0..255 and on tempty[1] after columns 256..511; the MMA issuer
// starts the next tile as soon as half 0 is free, issuing the hs = 0 MMAs of
// the first STAGES k-blocks (the stages the producer loaded meanwhile), then
// waits for half 1 and issues those k-blocks' hs = 1 MMAs before going on as
// usual.  Each column's k order is unchanged, so the bits are the same.
template <int NSPLIT, bool HALVES>
__global__ void __launch_bounds__(hg2::THREADS, 1)
    hgemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, HgemmArgs args) {
    using namespace sm100;
    using Cf = hg2::Cfg<NSPLIT>;
    static_assert(!HALVES || NSPLIT == 2, "accumulator halves need the 256 x 512 tile");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t *sA = smem;
    uint8_t *sB = smem + Cf::STAGES * Cf::A_BYTES;
    uint8_t *stg = smem + Cf::STAGES * Cf::STAGE_BYTES;  // epilogue staging, 1024-aligned
    uint64_t *bars = reinterpret_cast<uint64_t *>(stg + Cf::EPI_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + Cf::STAGES;
    uint64_t *tfull = bars + 2 * Cf::STAGES;
    uint64_t *tempty = bars + 2 * Cf::STAGES + 2;
    uint64_t *drain = bars + 2 * Cf::STAGES + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * Cf::STAGES + 5);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int npairs = static_cast<int>(gridDim.x >> 1);
    const int tiles_m = (args.M + 2 * Cf::BM - 1) / (2 * Cf::BM);
    const int tiles_n = (args.N + Cf::BN - 1) / Cf::BN;
    const int num_tiles = tiles_m * tiles_n;
    const int kblocks = (args.K + Cf::BK - 1) / Cf::BK;
    const int group_m = args.group_m > 0 ? args.group_m : Cf::GROUP_M;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cf::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], Cf::EPI_WARPS_PAIR);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        prefetch_tensormap(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cf::TMEM_COLS);
        tmem_relinquish_pair();
    }
    // Both CTAs' barriers must be initialised before either signals the other.
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            bool ok = true;
            for (int t = pair; t < num_tiles && ok; t += npairs) {
                int tm, tn;
                tile_coords_g(t, tiles_m, tiles_n, group_m, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x11,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full_leader = mapa_shared(smem_u32(&full[stage]), 0);
                    if (leader) mbar_arrive_expect_tx(&full[stage], Cf::PAIR_STAGE_BYTES);
                    uint8_t *a_dst = sA + stage * Cf::A_BYTES;
                    uint8_t *b_dst = sB + stage * Cf::B_BYTES;
                    tma_load_2d_pair(a_dst, &tmA, full_leader, kb * Cf::BK,
                                     tm * 2 * Cf::BM + static_cast<int>(rank) * Cf::BM);
#pragma unroll
                    for (int hs = 0; hs < NSPLIT; ++hs)
#pragma unroll
                        for (int j = 0; j < Cf::BN_HALF / Cf::B_BOX_N; ++j)
                            tma_load_2d_pair(b_dst + hs * Cf::B_SPLIT_BYTES + j * Cf::B_BOX_BYTES, &tmB, full_leader,
                                             tn * Cf::BN + hs * 256 + static_cast<int>(rank) * Cf::BN_HALF +
                                                 j * Cf::B_BOX_N,
                                             kb * Cf::BK);
                    ++issued;
                    if (++stage == Cf::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok && issued) {
                if (leader) {
                    // Loads in flight complete on this CTA's full barriers.
                    const uint32_t n = issued < (uint32_t)Cf::STAGES ? issued : (uint32_t)Cf::STAGES;
                    int s = stage;
                    uint32_t ph = phase;
                    for (uint32_t i = 0; i < n; ++i) {
                        if (--s < 0) {
                            s = Cf::STAGES - 1;
                            ph ^= 1u;
                        }
                        mbar_wait_drain(&full[s], ph, 1000000000ull);
                    }
                } else {
                    // The partner's loads complete on the leader's barriers,
                    // which it cannot poll: give them a bounded grace period.
                    const uint64_t t0 = globaltimer_ns();
                    while (globaltimer_ns() - t0 < 2000000ull) {
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader only)
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued_any = false;
            for (int t = pair; t < num_tiles && ok; t += npairs) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x12,
                               args.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cf::ACC_COLS);
                int kb0 = 0;
                if constexpr (HALVES) {
                    // Half 0 is free: the hs = 0 MMAs of the first P k-blocks,
                    // holding their stages.
                    const int P = kblocks < Cf::STAGES ? kblocks : Cf::STAGES;
                    const int stage0 = stage;
                    for (int kb = 0; kb < P; ++kb) {
                        if (!mbar_wait(&full[stage], phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x13,
                                       args.wait_ns)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_base = smem_u32(sA + stage * Cf::A_BYTES);
                        const uint32_t b_base = smem_u32(sB + stage * Cf::B_BYTES);
#pragma unroll
                        for (int kk = 0; kk < Cf::BK / 16; ++kk)
                            umma_f16_pair(d_tmem, sdesc_sw128(a_base + kk * 32, 16, 1024),
                                          sdesc_sw128(b_base + kk * 2048, Cf::B_BOX_BYTES, 1024), Cf::IDESC,
                                          (kb | kk) != 0 ? 1u : 0u);
                        issued_any = true;
                        if (++stage == Cf::STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    // Half 1: its MMAs of those k-blocks, then the stages go back.
                    if (!mbar_wait(&tempty[1], acc_phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x15,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kb = 0; kb < P; ++kb) {
                        const int s = (stage0 + kb) % Cf::STAGES;
                        const uint32_t a_base = smem_u32(sA + s * Cf::A_BYTES);
                        const uint32_t b_base = smem_u32(sB + s * Cf::B_BYTES);
#pragma unroll
                        for (int kk = 0; kk < Cf::BK / 16; ++kk)
                            umma_f16_pair(d_tmem + 256u, sdesc_sw128(a_base + kk * 32, 16, 1024),
                                          sdesc_sw128(b_base + Cf::B_SPLIT_BYTES + kk * 2048, Cf::B_BOX_BYTES, 1024),
                                          Cf::IDESC, (kb | kk) != 0 ? 1u : 0u);
                        umma_commit_pair(&empty[s], 0x3);
                    }
                    kb0 = P;
                }
                for (int kb = kb0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x13,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(sA + stage * Cf::A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * Cf::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < Cf::BK / 16; ++kk) {
                        const uint64_t adesc = sdesc_sw128(a_base + kk * 32, 16, 1024);
#pragma unroll
                        for (int hs = 0; hs < NSPLIT; ++hs) {
                            const uint64_t bdesc =
                                sdesc_sw128(b_base + hs * Cf::B_SPLIT_BYTES + kk * 2048, Cf::B_BOX_BYTES, 1024);
                            umma_f16_pair(d_tmem + static_cast<uint32_t>(hs * 256), adesc, bdesc, Cf::IDESC,
                                          (kb | kk) != 0 ? 1u : 0u);
                        }
                    }
                    umma_commit_pair(&empty[stage], 0x3);
                    issued_any = true;
                    if (++stage == Cf::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tfull[acc], 0x3);
                if (++acc == Cf::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok && issued_any) {
                umma_commit_pair(drain, 0x1);
                mbar_wait_drain(drain, 0, 1000000000ull);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (both CTAs)
        const int q = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * Cf::BM + q * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const bool read_c = args.beta != 0.0f;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t nstore = 0;
        for (int t = pair; t < num_tiles; t += npairs) {
            int tm, tn;
            tile_coords_g(t, tiles_m, tiles_n, group_m, tm, tn);
            bool ok = mbar_wait_sleepy(&tfull[acc], acc_phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x14,
                                args.wait_ns);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = tm * 2 * Cf::BM + row_in_tile;
            const bool row_ok = row < args.M;
            uint16_t *crow = args.C + static_cast<int64_t>(row) * args.N;
            if (!read_c) {
                // TMEM -> registers -> alpha -> f16 -> swizzled staging -> TMA
                // store of a 32-row x 64-column box; the store clips rows and
                // columns outside C.
                const int row0 = tm * 2 * Cf::BM + static_cast<int>(rank) * Cf::BM + q * 32;
                uint8_t *wbuf = stg + (warp - 2) * 2 * Cf::EPI_BUF_BYTES;
#pragma unroll 1
                for (int c = 0; c < Cf::BN / 64; ++c) {
                    uint32_t r0[32], r1[32];
                    __syncwarp();
                    const uint32_t taddr = tmem_base + lane_off + static_cast<uint32_t>(acc * Cf::ACC_COLS + c * 64);
                    tmem_ld_32x32b_x32(taddr, r0);
                    tmem_ld_32x32b_x32(taddr + 32, r1);
                    tmem_ld_wait();
                    if (c == Cf::BN / 64 - 1 || (HALVES && c == Cf::BN / 128 - 1)) {
                        // this warp has read the whole accumulator (or, with
                        // HALVES, its first half): one arrival per warp on the
                        // leader's barrier
                        uint64_t *bar = HALVES ? &tempty[c == Cf::BN / 64 - 1 ? 1 : 0] : &tempty[acc];
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if (leader)
                                mbar_arrive(bar);
                            else
                                mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
                        }
                    }
                    const int col0 = tn * Cf::BN + c * 64;
                    if (col0 >= args.N || row0 >= args.M) continue;  // warp-uniform
                    uint8_t *buf = wbuf + (nstore & 1) * Cf::EPI_BUF_BYTES;
                    if (lane == 0) bulk_wait_group_read<1>();  // the store that used buf last has read it
                    __syncwarp();
                    uint8_t *rowp = buf + lane * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t *src = j < 4 ? r0 + 8 * j : r1 + 8 * (j - 4);
                        uint4 o;
                        __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            oh[e] = __floats2half2_rn(args.alpha * __uint_as_float(src[2 * e]),
                                                      args.alpha * __uint_as_float(src[2 * e + 1]));
                        // 128-byte swizzle: 16-byte chunk j of row r sits at chunk j ^ (r % 8)
                        *reinterpret_cast<uint4 *>(rowp + ((j ^ (lane & 7)) << 4)) = o;
                    }
                    if (args.ndst > 0 || args.mc != nullptr) {
                        // Fused all-gather: 16-byte chunk q = lane + 32t of the box
                        // (row q / 8, columns 8 (q % 8) ..) is read back from its
                        // swizzled slot and stored to every rank's C; each store
                        // instruction covers four whole 128-byte row segments.
                        __syncwarp();
                        uint4 v[8];
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const int qq = lane + 32 * t, rr = qq >> 3, jj = qq & 7;
                            v[t] = *reinterpret_cast<const uint4 *>(buf + rr * 128 + ((jj ^ (rr & 7)) << 4));
                        }
                        if (args.mc != nullptr) {
                            uint16_t *base = args.mc + args.col_off;
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                const int qq = lane + 32 * t;
                                const int grow = row0 + (qq >> 3), gcol = col0 + (qq & 7) * 8;
                                if (grow < args.M && gcol < args.N)
                                    multimem_st_v4(base + static_cast<int64_t>(grow) * args.ldc + gcol, v[t]);
                            }
                        }
#pragma unroll 1
                        for (int i = 0; i < args.ndst; ++i) {
                            // rotate: each CTA pair starts on another rank, so the
                            // ranks' stores spread over every receiving link
                            const int d = args.rotate ? (i + pair) % args.ndst : i;
                            uint16_t *base = args.dst[d] + args.col_off;
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                const int qq = lane + 32 * t;
                                const int grow = row0 + (qq >> 3), gcol = col0 + (qq & 7) * 8;
                                if (grow < args.M && gcol < args.N)
                                    *reinterpret_cast<uint4 *>(base + static_cast<int64_t>(grow) * args.ldc + gcol) =
                                        v[t];
                            }
                        }
                        ++nstore;
                        continue;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, buf, col0, row0);
                        bulk_commit_group();
                    }
                    ++nstore;
                }
                if (++acc == Cf::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
                continue;
            }
#pragma unroll 1
            for (int c = 0; c < Cf::BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tmem_base + lane_off + static_cast<uint32_t>(acc * Cf::ACC_COLS + c * 32), r);
                tmem_ld_wait();
                if (c == Cf::BN / 32 - 1 || (HALVES && c == Cf::BN / 64 - 1)) {
                    // This warp's share of the accumulator (with HALVES, of
                    // its first half) is in registers: one arrival per warp
                    // on the leader's barrier.
                    uint64_t *bar = HALVES ? &tempty[c == Cf::BN / 32 - 1 ? 1 : 0] : &tempty[acc];
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (leader)
                            mbar_arrive(bar);
                        else
                            mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
                    }
                }
                const int col0 = tn * Cf::BN + c * 32;
                if (!row_ok || col0 >= args.N) continue;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = args.alpha * __uint_as_float(r[i]);
                store_c_chunk(crow, col0, args.N, v, read_c, args.beta);
            }
            if (++acc == Cf::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // Every TMA store of this warp has completed before the CTA exits.
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cf::TMEM_COLS);
    }
}

// Generic CUDA-core HGEMM for shapes the TMA path cannot describe: 64x64
// tile, 4x4 outputs per thread, f32 accumulate, any M/N/K and alignment.
__global__ void __launch_bounds__(256) hgemm_simt_kernel(const uint16_t *__restrict__ A,
                                                         const uint16_t *__restrict__ B, uint16_t *__restrict__ C,
                                                         int64_t M, int64_t N, int64_t K, float alpha, float beta) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int idx = tid + i * 256;  // 1024 = 64 rows x 16 k
            int r = idx >> 4, kc = idx & 15;
            int64_t gr = m0 + r, gk = k0 + kc;
            As[kc][r] = (gr < M && gk < K) ? __half2float(__ushort_as_half(A[gr * K + gk])) : 0.0f;
            int kr = idx >> 6, c = idx & 63;
            int64_t gk2 = k0 + kr, gc = n0 + c;
            Bs[kr][c] = (gk2 < K && gc < N) ? __half2float(__ushort_as_half(B[gk2 * N + gc])) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t r = m0 + ty * 4 + i;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t c = n0 + tx * 4 + j;
            if (c >= N) continue;
            float v = alpha * acc[i][j];
            if (beta != 0.0f) v = fmaf(beta, __half2float(__ushort_as_half(C[r * N + c])), v);
            C[r * N + c] = __half_as_ushort(__float2half_rn(v));
        }
    }
}

int encode_2d_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                  uint32_t box_rows) {
    return b2b::encode_tma_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rows, cols, box_cols, box_rows);
}

}  // namespace

namespace b2b {

bool hgemm_tc_eligible(size_t m, size_t n, size_t k, const void *A, const void *B, const void *C) {
    return (k % 8 == 0) && (n % 8 == 0) && aligned16(A) && aligned16(B) && aligned16(C) && m < (1ull << 31) &&
           n < (1ull << 31) && k < (1ull << 31) && ((m + 127) / 128) * ((n + 255) / 256) < (1ull << 31);
}

namespace {

struct DeviceLaunchState {
    bool attr1 = false;
    bool attr2[3] = {false, false, false};
    int max_pairs[3] = {0, 0, 0};  // co-resident CTA pairs of hgemm_tc2_kernel<1,0>, <2,0>, <2,1>
};
DeviceLaunchState g_hgemm_state[64];
std::mutex g_hgemm_mu;

template <int NSPLIT, bool HALVES>
int max_pairs_of(b2b_handle *h, cudaLaunchConfig_t &cfg) {
    using Cf = hg2::Cfg<NSPLIT>;
    constexpr int slot = NSPLIT - 1 + (HALVES ? 1 : 0);
    std::lock_guard<std::mutex> lk(g_hgemm_mu);
    DeviceLaunchState &st = g_hgemm_state[h->device & 63];
    if (!st.attr2[slot]) {
        cudaError_t e = cudaFuncSetAttribute(hgemm_tc2_kernel<NSPLIT, HALVES>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES);
        if (e != cudaSuccess) {
            fail_cuda(e, "hgemm pair smem attribute");
            return -1;
        }
        cfg.gridDim = dim3(2 * (h->sm_count / 2));
        int clusters = 0;
        e = cudaOccupancyMaxActiveClusters(&clusters, (void *)hgemm_tc2_kernel<NSPLIT, HALVES>, &cfg);
        if (e != cudaSuccess) {
            fail_cuda(e, "cudaOccupancyMaxActiveClusters");
            return -1;
        }
        st.max_pairs[slot] = clusters > 0 ? clusters : h->sm_count / 2;
        st.attr2[slot] = true;
    }
    return st.max_pairs[slot];
}

template <int NSPLIT, bool HALVES>
int launch_pair_kernel(b2b_handle *h, const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmC,
                       const HgemmArgs &args, size_t m, size_t n, int max_pairs) {
    using Cf = hg2::Cfg<NSPLIT>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(hg2::THREADS);
    cfg.dynamicSmemBytes = Cf::SMEM_BYTES;
    cfg.stream = h->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const size_t tiles = ((m + 255) / 256) * ((n + Cf::BN - 1) / Cf::BN);
    const int pairs = static_cast<int>(tiles < static_cast<size_t>(max_pairs) ? tiles : max_pairs);
    cfg.gridDim = dim3(2 * pairs);
    cudaError_t e = cudaLaunchKernelEx(&cfg, hgemm_tc2_kernel<NSPLIT, HALVES>, tmA, tmB, tmC, args);
    if (e != cudaSuccess) return fail_cuda(e, "hgemm tcgen05 pair launch");
    return B2B_OK;
}

// Pair-kernel choice: 256 x 512 tiles when K is long enough to amortise
// their unoverlapped epilogue (K >= 2048; measured on 8192 x 8192: 256 x 256
// wins at K = 1024, 256 x 512 from K = 4096 on) and they still give every
// co-resident pair at least one tile; else 256 x 256.  hgemm_variant 2 / 3
// forces one.
int launch_pairs(b2b_handle *h, const CUtensorMap &tmA, const CUtensorMap &tmB, const HgemmArgs &args, size_t m,
                 size_t n) {
    // C as 32-row x 64-column boxes with the 128-byte swizzle (TMA-store epilogue).
    CUtensorMap tmC;
    if (int rc = encode_2d_f16(&tmC, args.C, m, n, 64, 32)) return rc;
    cudaLaunchConfig_t probe = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    probe.blockDim = dim3(hg2::THREADS);
    probe.stream = h->stream;
    probe.attrs = attr;
    probe.numAttrs = 1;
    probe.dynamicSmemBytes = hg2::Cfg<2>::SMEM_BYTES;
    const int wide_pairs = max_pairs_of<2, false>(h, probe);
    if (wide_pairs < 0) return B2B_ERR_CUDA;
    const size_t wide_tiles = ((m + 255) / 256) * ((n + 511) / 512);
    // A fused all-gather makes the epilogue long (its stores cross NVLink to
    // every rank): keep the double-buffered accumulators of the 256 x 256
    // tiles so the next tile's MMAs run meanwhile.
    const bool wide = h->hgemm_variant == 3 || h->hgemm_variant == 4 ||
                      (h->hgemm_variant != 2 && args.ndst <= 1 && n >= 512 &&
                                                 args.K >= 2048 && wide_tiles >= static_cast<size_t>(wide_pairs));
    if (wide) {
        if (h->hgemm_variant == 3) return launch_pair_kernel<2, false>(h, tmA, tmB, tmC, args, m, n, wide_pairs);
        const int halves_pairs = max_pairs_of<2, true>(h, probe);
        if (halves_pairs < 0) return B2B_ERR_CUDA;
        return launch_pair_kernel<2, true>(h, tmA, tmB, tmC, args, m, n, halves_pairs);
    }
    probe.dynamicSmemBytes = hg2::Cfg<1>::SMEM_BYTES;
    const int pairs = max_pairs_of<1, false>(h, probe);
    if (pairs < 0) return B2B_ERR_CUDA;
    return launch_pair_kernel<1, false>(h, tmA, tmB, tmC, args, m, n, pairs);
}
}  // namespace

// HGEMM whose epilogue scatters the panel into every rank's C (see
// HgemmArgs::ndst).  Sets *done when the CTA-pair kernel took the call
// (beta == 0, pair-kernel shapes, 16-byte aligned destinations); otherwise
// the caller falls back to compute-then-copy.
int launch_hgemm_gather_fused(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                              const uint16_t *B, uint16_t *const *dst, int ndst, int self, size_t ldc, size_t col_off,
                              bool *done) {
    *done = false;
    uint16_t *cself = dst[self] + col_off;
    if (!hgemm_tc_eligible(m, n, k, A, B, cself) || m <= static_cast<size_t>(hg::BM) || h->force_single_cta ||
        h->hgemm_variant == 1 || ldc % 8 != 0 || col_off % 8 != 0 || ndst > 8)
        return B2B_OK;
    for (int d = 0; d < ndst; ++d)
        if (!aligned16(dst[d])) return B2B_OK;
    CUtensorMap tmA, tmB;
    int rc = encode_2d_f16(&tmA, A, m, k, hg::BK, hg::BM);
    if (rc) return rc;
    rc = encode_2d_f16(&tmB, B, k, n, hg::B_BOX_N, hg::BK);
    if (rc) return rc;
    HgemmArgs args{cself, (int)m, (int)n, (int)k, alpha, 0.0f, h->d_status, h->wait_limit_ns, h->hgemm_group_m,
                   ndst, static_cast<int64_t>(ldc), static_cast<int64_t>(col_off), {}, nullptr,
                   h->gather_rotate};
    for (int d = 0; d < ndst; ++d) args.dst[d] = dst[d];
    rc = launch_pairs(h, tmA, tmB, args, m, n);
    if (rc == B2B_OK) *done = true;
    return rc;
}

// Same as launch_hgemm_gather_fused, the destinations being every member
// of an NVLink multicast object mapped at `mc` (own buffer at `own`).
int launch_hgemm_gather_multicast(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                                  const uint16_t *B, uint16_t *mc, uint16_t *own, size_t ldc, size_t col_off,
                                  bool *done) {
    *done = false;
    uint16_t *cself = own + col_off;
    if (!hgemm_tc_eligible(m, n, k, A, B, cself) || m <= static_cast<size_t>(hg::BM) || h->force_single_cta ||
        h->hgemm_variant == 1 || ldc % 8 != 0 || col_off % 8 != 0 || !aligned16(mc))
        return B2B_OK;
    CUtensorMap tmA, tmB;
    int rc = encode_2d_f16(&tmA, A, m, k, hg::BK, hg::BM);
    if (rc) return rc;
    rc = encode_2d_f16(&tmB, B, k, n, hg::B_BOX_N, hg::BK);
    if (rc) return rc;
    HgemmArgs args{cself, (int)m, (int)n, (int)k, alpha, 0.0f, h->d_status, h->wait_limit_ns, h->hgemm_group_m,
                   0, static_cast<int64_t>(ldc), static_cast<int64_t>(col_off), {}, mc};
    rc = launch_pairs(h, tmA, tmB, args, m, n);
    if (rc == B2B_OK) *done = true;
    return rc;
}

namespace {

// Copies a rows x cols f16 matrix (row pitch src_ld elements) into dst with
// row pitch dst_ld >= cols, zero-filling columns cols..dst_ld-1 and rows
// rows..dst_rows-1.  Stream-ordered (capturable) memset/memcpy nodes only.
int pad_copy_f16(b2b_handle *h, uint16_t *dst, size_t dst_ld, size_t dst_rows, const uint16_t *src, size_t src_ld,
                 size_t rows, size_t cols) {
    cudaError_t e = cudaSuccess;
    if (dst_ld > cols)
        e = cudaMemset2DAsync(dst + cols, dst_ld * 2, 0, (dst_ld - cols) * 2, rows, h->stream);
    if (e == cudaSuccess && dst_rows > rows)
        e = cudaMemsetAsync(dst + rows * dst_ld, 0, (dst_rows - rows) * dst_ld * 2, h->stream);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(dst, dst_ld * 2, src, src_ld * 2, cols * 2, rows, cudaMemcpyDeviceToDevice, h->stream);
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "hgemm padding copy");
}

int launch_hgemm_tc(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                    float beta, uint16_t *C);

}  // namespace

// HGEMM entry: the tensor-core kernels where the tensor maps can describe the
// operands; else, for GEMMs large enough (m*n*k >= 2^27) that the tensor
// cores pay for the copies, the operands the maps cannot describe (K or N not
// a multiple of 8, or not 16-byte aligned) are copied into zero-padded
// workspace (K and N rounded up to 8; the zero columns of A and rows of B add
// exact zeros to every sum, so each output is the same f32 sum as without
// padding), the padded GEMM runs on the tensor cores and C's columns are
// copied back; smaller ones run the CUDA-core kernel.  hgemm_variant 5
// forces the CUDA-core kernel for those shapes.
int launch_hgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                 float beta, uint16_t *C) {
    if (hgemm_tc_eligible(m, n, k, A, B, C)) return launch_hgemm_tc(h, m, n, k, alpha, A, B, beta, C);
    const size_t k8 = (k + 7) / 8 * 8, n8 = (n + 7) / 8 * 8;
    const double work = static_cast<double>(m) * static_cast<double>(n) * static_cast<double>(k);
    if (h->hgemm_variant != 5 && work >= 134217728.0 && m < (1ull << 31) && n8 < (1ull << 31) && k8 < (1ull << 31) &&
        ((m + 127) / 128) * ((n8 + 255) / 256) < (1ull << 31)) {
        const bool pad_a = k8 != k || !aligned16(A);
        const bool pad_b = k8 != k || n8 != n || !aligned16(B);
        const bool pad_c = n8 != n || !aligned16(C);
        auto up = [](size_t b) { return (b + 255) / 256 * 256; };
        const size_t bytes_a = pad_a ? up(m * k8 * 2) : 0, bytes_b = pad_b ? up(k8 * n8 * 2) : 0,
                     bytes_c = pad_c ? up(m * n8 * 2) : 0;
        void *ws = nullptr;
        if (int rc = workspace(h, bytes_a + bytes_b + bytes_c, &ws)) return rc;
        uint8_t *w = static_cast<uint8_t *>(ws);
        const uint16_t *a = A, *b = B;
        uint16_t *c = C;
        int rc = B2B_OK;
        if (pad_a) {
            uint16_t *ap = reinterpret_cast<uint16_t *>(w);
            rc = pad_copy_f16(h, ap, k8, m, A, k, m, k);
            a = ap;
        }
        if (rc == B2B_OK && pad_b) {
            uint16_t *bp = reinterpret_cast<uint16_t *>(w + bytes_a);
            rc = pad_copy_f16(h, bp, n8, k8, B, n, k, n);
            b = bp;
        }
        if (rc == B2B_OK && pad_c) {
            c = reinterpret_cast<uint16_t *>(w + bytes_a + bytes_b);
            // beta != 0 reads C: bring it in (the padding columns' outputs
            // are discarded, so they need no defined value)
            if (beta != 0.0f) {
                cudaError_t e = cudaMemcpy2DAsync(c, n8 * 2, C, n * 2, n * 2, m, cudaMemcpyDeviceToDevice, h->stream);
                if (e != cudaSuccess) rc = fail_cuda(e, "hgemm padding copy");
            }
        }
        if (rc == B2B_OK) rc = launch_hgemm_tc(h, m, n8, k8, alpha, a, b, beta, c);
        if (rc == B2B_OK && pad_c) {
            cudaError_t e = cudaMemcpy2DAsync(C, n * 2, c, n8 * 2, n * 2, m, cudaMemcpyDeviceToDevice, h->stream);
            if (e != cudaSuccess) rc = fail_cuda(e, "hgemm padding copy back");
        }
        return rc;
    }
    dim3 grid(static_cast<unsigned>((n + 63) / 64), static_cast<unsigned>((m + 63) / 64));
    if (grid.y > 65535u) return fail(B2B_ERR_INVALID_ARG, "hgemm: m too large for the generic path");
    hgemm_simt_kernel<<<grid, 256, 0, h->stream>>>(A, B, C, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "hgemm generic launch");
    return B2B_OK;
}

namespace {

int launch_hgemm_tc(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                    float beta, uint16_t *C) {
    CUtensorMap tmA, tmB;
    int rc = encode_2d_f16(&tmA, A, m, k, hg::BK, hg::BM);
    if (rc) return rc;
    rc = encode_2d_f16(&tmB, B, k, n, hg::B_BOX_N, hg::BK);
    if (rc) return rc;
    HgemmArgs args{C, (int)m, (int)n, (int)k, alpha, beta, h->d_status, h->wait_limit_ns, h->hgemm_group_m, 0, 0, 0, {}, nullptr};
    // More than one 128-row tile: CTA pairs with 256 x 256 tiles.
    if (m > static_cast<size_t>(hg::BM) && !h->force_single_cta && h->hgemm_variant != 1)
        return launch_pairs(h, tmA, tmB, args, m, n);
    {
        std::lock_guard<std::mutex> lk(g_hgemm_mu);
        DeviceLaunchState &st = g_hgemm_state[h->device & 63];
        if (!st.attr1) {
            cudaError_t e =
                cudaFuncSetAttribute(hgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, hg::SMEM_BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "hgemm smem attribute");
            st.attr1 = true;
        }
    }
    const int tiles = static_cast<int>(((m + hg::BM - 1) / hg::BM) * ((n + hg::BN - 1) / hg::BN));
    const int grid = tiles < h->sm_count ? tiles : h->sm_count;
    hgemm_tc_kernel<<<grid, hg::THREADS, hg::SMEM_BYTES, h->stream>>>(tmA, tmB, args);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "hgemm tcgen05 launch");
    return B2B_OK;
}

}  // namespace

}  // namespace b2b
