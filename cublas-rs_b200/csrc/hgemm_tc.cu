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
// not 16-byte aligned) run hgemm_simt_kernel below, a plain CUDA-core kernel
// with the same arithmetic.
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
            bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 4, args.wait_ns);
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
                if (col0 + 32 <= args.N) {
                    uint4 *dst = reinterpret_cast<uint4 *>(crow + col0);
                    if (read_c) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint4 old = dst[j];
                            const __half2 *oh = reinterpret_cast<const __half2 *>(&old);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                float2 of = __half22float2(oh[e]);
                                v[j * 8 + e * 2 + 0] = fmaf(args.beta, of.x, v[j * 8 + e * 2 + 0]);
                                v[j * 8 + e * 2 + 1] = fmaf(args.beta, of.y, v[j * 8 + e * 2 + 1]);
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
                        if (col0 + i < args.N) {
                            float x = v[i];
                            if (read_c) x = fmaf(args.beta, __half2float(__ushort_as_half(crow[col0 + i])), x);
                            crow[col0 + i] = __half_as_ushort(__float2half_rn(x));
                        }
                    }
                }
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

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major [rows x cols] f16 matrix, box of box_cols (inner) x box_rows,
// 128-byte swizzle, out-of-range elements read as zero.
int encode_2d_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                  uint32_t box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return b2b::fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return b2b::fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return B2B_OK;
}

}  // namespace

namespace b2b {

bool hgemm_tc_eligible(size_t m, size_t n, size_t k, const void *A, const void *B, const void *C) {
    return (k % 8 == 0) && (n % 8 == 0) && aligned16(A) && aligned16(B) && aligned16(C) && m < (1ull << 31) &&
           n < (1ull << 31) && k < (1ull << 31) && ((m + 127) / 128) * ((n + 255) / 256) < (1ull << 31);
}

int launch_hgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                 float beta, uint16_t *C) {
    if (hgemm_tc_eligible(m, n, k, A, B, C)) {
        CUtensorMap tmA, tmB;
        int rc = encode_2d_f16(&tmA, A, m, k, hg::BK, hg::BM);
        if (rc) return rc;
        rc = encode_2d_f16(&tmB, B, k, n, hg::B_BOX_N, hg::BK);
        if (rc) return rc;
        static bool attr_set[64] = {};
        if (h->device >= 64 || !attr_set[h->device]) {
            cudaError_t e =
                cudaFuncSetAttribute(hgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, hg::SMEM_BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "hgemm smem attribute");
            if (h->device < 64) attr_set[h->device] = true;
        }
        const int tiles = static_cast<int>(((m + hg::BM - 1) / hg::BM) * ((n + hg::BN - 1) / hg::BN));
        const int grid = tiles < h->sm_count ? tiles : h->sm_count;
        HgemmArgs args{C, (int)m, (int)n, (int)k, alpha, beta, h->d_status, h->wait_limit_ns};
        hgemm_tc_kernel<<<grid, hg::THREADS, hg::SMEM_BYTES, h->stream>>>(tmA, tmB, args);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "hgemm tcgen05 launch");
        return B2B_OK;
    }
    dim3 grid(static_cast<unsigned>((n + 63) / 64), static_cast<unsigned>((m + 63) / 64));
    if (grid.y > 65535u) return fail(B2B_ERR_INVALID_ARG, "hgemm: m too large for the generic path");
    hgemm_simt_kernel<<<grid, 256, 0, h->stream>>>(A, B, C, (int64_t)m, (int64_t)n, (int64_t)k, alpha, beta);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "hgemm generic launch");
    return B2B_OK;
}

}  // namespace b2b
