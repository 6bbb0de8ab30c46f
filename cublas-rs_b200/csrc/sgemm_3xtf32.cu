// sgemm_3xtf32.cu -- opt-in split-precision SGEMM on the tensor cores
// (B2B_ALGO_3XTF32).  No counterpart in the reference, whose tensor-core
// slot is a todo! (crates/cublas-l3/src/hgemm.rs:189-193); the result is the
// same C <- alpha * A * B + beta * C as sgemm.rs:31-360 with row-major f32
// operands.
//
// Each f32 x is split as hi = x with its 13 low mantissa bits cleared (what
// the tcgen05 kind::tf32 datapath reads from an f32 operand) and
// lo = x - hi (exact in f32).  A*B is then accumulated in f32 as
//     hi(A) hi(B) + hi(A) lo(B) + lo(A) hi(B)
// with three kind::tf32 MMAs per 8-wide k step; the dropped lo*lo term and
// the truncation of lo to tf32 leave a per-product error near 2^-21, far
// inside the FP32 bound 4*K*eps.  Non-finite inputs are not supported (the
// split of +-inf is NaN).
//
// Layout (CTA pairs, like the HGEMM pair kernel): a cluster of two CTAs owns
// a 256 x 256 tile; CTA r holds rows [128r, 128r+128) of the A tile and
// columns [128r, 128r+128) of the B tile; k-blocks of 32 (one 128-byte
// swizzle row of f32).  B is MN-major, which for 32-bit operands tcgen05
// reads only in the 128-byte swizzle with 32-byte atomicity (TMA
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, descriptor layout type 1).  Per stage each CTA has 64 KiB: raw A and B tiles
// (TMA) and their lo tiles, which four "split" warps compute in place from
// the raw tiles (same swizzled byte offsets, so no layout work) -- nothing
// is staged in global memory.  Roles per CTA (320 threads): warp 0 TMA,
// warp 1 TMEM allocation and, in the leader, the single MMA-issuing thread,
// warps 2-5 epilogue, warps 6-9 split.
//   full[s]  (each CTA) : its own 32 KiB of raw operands landed (TMA tx).
//   split[s] (leader)   : both CTAs' split warps wrote lo (8 arrivals).
//   empty[s] (each CTA) : the pair's MMAs on stage s finished (commit).
//   tfull / tempty      : accumulator handoff, as in the HGEMM kernel.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace {

namespace x3 {
constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BN_CTA = 128;
constexpr int BK = 32;
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK * 4;           // 16 KiB
constexpr int B_BOX_N = 32;                    // TMA box of B: 32 (n) x 32 (k)
constexpr int B_BOX_BYTES = B_BOX_N * BK * 4;  // 4 KiB
constexpr int B_BYTES = BK * BN_CTA * 4;       // 16 KiB
constexpr int RAW_BYTES = A_BYTES + B_BYTES;   // 32 KiB per CTA per stage
constexpr int STAGE_BYTES = 2 * RAW_BYTES;     // raw + lo
constexpr int ACC_COLS = BN;
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int THREADS = 320;
constexpr int SPLIT_WARP0 = 6;
constexpr int SPLIT_THREADS = 128;
constexpr int SPLIT_ARRIVALS = 8;  // 4 split warps x 2 CTAs
constexpr int EPI_WARPS_PAIR = 8;
constexpr int GROUP_M = 16;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t IDESC = sm100::idesc_f32acc(2, 0, 1, 256, BN);  // tf32 x tf32 -> f32, B MN-major
}  // namespace x3

struct X3Args {
    float *C;
    int M, N, K;
    float alpha, beta;
    int *status;
    uint64_t wait_ns;
    const float *bias;  // optional per-column bias (nullptr: none)
    int relu;           // apply max(0, .) last
};

__device__ __forceinline__ void x3_tile(int t, int tiles_m, int tiles_n, int &tm, int &tn) {
    const int span = x3::GROUP_M * tiles_n;
    const int g = t / span;
    const int first = g * x3::GROUP_M;
    const int gm = min(tiles_m - first, x3::GROUP_M);
    const int r = t - g * span;
    tm = first + r % gm;
    tn = r / gm;
}

__device__ __forceinline__ float x3_epi(float x, const float *bias, int relu, int col) {
    if (bias) x += bias[col];
    if (relu) x = x > 0.0f ? x : 0.0f;
    return x;
}

__device__ __forceinline__ void store_c_f32(float *crow, int col0, int N, float (&v)[32], bool read_c, float beta,
                                            const float *bias, int relu) {
    if (col0 + 32 <= N) {
        float4 *dst = reinterpret_cast<float4 *>(crow + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (read_c) {
                const float4 old = dst[j];
                o.x = fmaf(beta, old.x, o.x);
                o.y = fmaf(beta, old.y, o.y);
                o.z = fmaf(beta, old.z, o.z);
                o.w = fmaf(beta, old.w, o.w);
            }
            if (bias || relu) {
                const int c = col0 + 4 * j;
                o.x = x3_epi(o.x, bias, relu, c);
                o.y = x3_epi(o.y, bias, relu, c + 1);
                o.z = x3_epi(o.z, bias, relu, c + 2);
                o.w = x3_epi(o.w, bias, relu, c + 3);
            }
            dst[j] = o;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (col0 + i < N) {
                float x = v[i];
                if (read_c) x = fmaf(beta, crow[col0 + i], x);
                crow[col0 + i] = x3_epi(x, bias, relu, col0 + i);
            }
        }
    }
}

__global__ void __launch_bounds__(x3::THREADS, 1)
    sgemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        X3Args args) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    // stage s: [A raw | B raw | A lo | B lo]
    auto a_raw = [&](int s) { return smem + s * x3::STAGE_BYTES; };
    auto b_raw = [&](int s) { return smem + s * x3::STAGE_BYTES + x3::A_BYTES; };
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + x3::STAGES * x3::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *split = bars + x3::STAGES;
    uint64_t *empty = bars + 2 * x3::STAGES;
    uint64_t *tfull = bars + 3 * x3::STAGES;
    uint64_t *tempty = bars + 3 * x3::STAGES + 2;
    uint64_t *drain = bars + 3 * x3::STAGES + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * x3::STAGES + 5);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int npairs = static_cast<int>(gridDim.x >> 1);
    const int tiles_m = (args.M + 2 * x3::BM - 1) / (2 * x3::BM);
    const int tiles_n = (args.N + x3::BN - 1) / x3::BN;
    const int num_tiles = tiles_m * tiles_n;
    const int kblocks = (args.K + x3::BK - 1) / x3::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < x3::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&split[s], x3::SPLIT_ARRIVALS);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], x3::EPI_WARPS_PAIR);
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
        tmem_alloc_pair(tmem_slot, x3::TMEM_COLS);
        tmem_relinquish_pair();
    }
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
                x3_tile(t, tiles_m, tiles_n, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x21,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], x3::RAW_BYTES);
                    tma_load_2d(a_raw(stage), &tmA, &full[stage], kb * x3::BK,
                                tm * 2 * x3::BM + static_cast<int>(rank) * x3::BM);
#pragma unroll
                    for (int j = 0; j < x3::BN_CTA / x3::B_BOX_N; ++j)
                        tma_load_2d(b_raw(stage) + j * x3::B_BOX_BYTES, &tmB, &full[stage],
                                    tn * x3::BN + static_cast<int>(rank) * x3::BN_CTA + j * x3::B_BOX_N, kb * x3::BK);
                    ++issued;
                    if (++stage == x3::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok && issued) {
                const uint32_t n = issued < (uint32_t)x3::STAGES ? issued : (uint32_t)x3::STAGES;
                int s = stage;
                uint32_t ph = phase;
                for (uint32_t i = 0; i < n; ++i) {
                    if (--s < 0) {
                        s = x3::STAGES - 1;
                        ph ^= 1u;
                    }
                    mbar_wait_drain(&full[s], ph, 1000000000ull);
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
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x22,
                               args.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * x3::ACC_COLS);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&split[stage], phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x23,
                                   args.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(a_raw(stage)), b_hi = smem_u32(b_raw(stage));
                    const uint32_t a_lo = a_hi + x3::RAW_BYTES, b_lo = b_hi + x3::RAW_BYTES;
#pragma unroll
                    for (int kk = 0; kk < x3::BK / 8; ++kk) {
                        // A: K-major SW128, 8-wide k step = 32 bytes in the row.
                        // B: MN-major 128-byte swizzle with 32-byte atoms
                        //    (4-row atoms 512 bytes apart), 32-wide n chunks
                        //    4 KiB apart, 8-wide k step = 8 rows = 1024 bytes.
                        const uint64_t ah = sdesc_sw128(a_hi + kk * 32, 16, 1024);
                        const uint64_t al = sdesc_sw128(a_lo + kk * 32, 16, 1024);
                        const uint64_t bh = sdesc_sw128_base32b(b_hi + kk * 1024, x3::B_BOX_BYTES, 512);
                        const uint64_t bl = sdesc_sw128_base32b(b_lo + kk * 1024, x3::B_BOX_BYTES, 512);
                        umma_tf32_pair(d_tmem, al, bh, x3::IDESC, (kb | kk) != 0 ? 1u : 0u);
                        umma_tf32_pair(d_tmem, ah, bl, x3::IDESC, 1u);
                        umma_tf32_pair(d_tmem, ah, bh, x3::IDESC, 1u);
                    }
                    umma_commit_pair(&empty[stage], 0x3);
                    issued_any = true;
                    if (++stage == x3::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tfull[acc], 0x3);
                if (++acc == 2) {
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
    } else if (warp >= x3::SPLIT_WARP0) {
        // ------------------------------------------------ split (both CTAs)
        const int st = threadIdx.x - x3::SPLIT_WARP0 * 32;  // 0..127
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = pair; t < num_tiles && ok; t += npairs) {
            for (int kb = 0; kb < kblocks; ++kb) {
                bool w = mbar_wait(&full[stage], phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x24,
                                   args.wait_ns);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
                const float4 *src = reinterpret_cast<const float4 *>(a_raw(stage));
                float4 *dst = reinterpret_cast<float4 *>(a_raw(stage) + x3::RAW_BYTES);
#pragma unroll 4
                for (int i = st; i < x3::RAW_BYTES / 16; i += x3::SPLIT_THREADS) {
                    const float4 v = src[i];
                    float4 lo;
                    lo.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
                    lo.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
                    lo.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
                    lo.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
                    dst[i] = lo;
                }
                // The MMAs read lo through the async proxy.
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (leader)
                        mbar_arrive(&split[stage]);
                    else
                        mbar_arrive_cluster(mapa_shared(smem_u32(&split[stage]), 0));
                }
                if (++stage == x3::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue (both CTAs)
        const int q = warp & 3;
        const int row_in_tile = static_cast<int>(rank) * x3::BM + q * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const bool read_c = args.beta != 0.0f;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = pair; t < num_tiles; t += npairs) {
            int tm, tn;
            x3_tile(t, tiles_m, tiles_n, tm, tn);
            bool ok = mbar_wait_sleepy(&tfull[acc], acc_phase, abort_flag, args.status, B2B_DEVSTAT_TIMEOUT | 0x25,
                                       args.wait_ns);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int row = tm * 2 * x3::BM + row_in_tile;
            const bool row_ok = row < args.M;
            float *crow = args.C + static_cast<int64_t>(row) * args.N;
#pragma unroll 1
            for (int c = 0; c < x3::BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tmem_base + lane_off + static_cast<uint32_t>(acc * x3::ACC_COLS + c * 32), r);
                tmem_ld_wait();
                if (c == x3::BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (leader)
                            mbar_arrive(&tempty[acc]);
                        else
                            mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
                    }
                }
                const int col0 = tn * x3::BN + c * 32;
                if (!row_ok || col0 >= args.N) continue;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = args.alpha * __uint_as_float(r[i]);
                store_c_f32(crow, col0, args.N, v, read_c, args.beta, args.bias, args.relu);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, x3::TMEM_COLS);
    }
}

std::mutex g_x3_mu;
int g_x3_pairs[64] = {};

}  // namespace

namespace b2b {

int launch_sgemm_3xtf32(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                        float beta, float *C) {
    return launch_sgemm_3xtf32_bias(h, m, n, k, alpha, A, B, beta, C, nullptr, 0);
}

int launch_sgemm_3xtf32_bias(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                             const float *B, float beta, float *C, const float *bias, int relu) {
    const bool eligible = (k % 4 == 0) && (n % 4 == 0) && aligned16(A) && aligned16(B) && aligned16(C) &&
                          m < (1ull << 31) && n < (1ull << 31) && k < (1ull << 31);
    // Shapes TMA cannot describe run the FFMA SGEMM (same result contract).
    if (!eligible) return launch_sgemm_bias(h, m, n, k, alpha, A, B, beta, C, bias, relu);
    CUtensorMap tmA, tmB;
    int rc = encode_tma_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, A, m, k, x3::BK, x3::BM);
    if (rc) return rc;
    rc = encode_tma_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, B, k, n, x3::B_BOX_N, x3::BK,
                       CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(x3::THREADS);
    cfg.dynamicSmemBytes = x3::SMEM_BYTES;
    cfg.stream = h->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int max_pairs;
    {
        std::lock_guard<std::mutex> lk(g_x3_mu);
        int &mp = g_x3_pairs[h->device & 63];
        if (mp == 0) {
            cudaError_t e =
                cudaFuncSetAttribute(sgemm_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, x3::SMEM_BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "3xtf32 smem attribute");
            cfg.gridDim = dim3(2 * (h->sm_count / 2));
            int clusters = 0;
            e = cudaOccupancyMaxActiveClusters(&clusters, (void *)sgemm_3xtf32_kernel, &cfg);
            if (e != cudaSuccess) return fail_cuda(e, "cudaOccupancyMaxActiveClusters");
            mp = clusters > 0 ? clusters : h->sm_count / 2;
        }
        max_pairs = mp;
    }
    const size_t tiles = ((m + 255) / 256) * ((n + x3::BN - 1) / x3::BN);
    const int pairs = static_cast<int>(tiles < static_cast<size_t>(max_pairs) ? tiles : max_pairs);
    cfg.gridDim = dim3(2 * pairs);
    X3Args args{C, (int)m, (int)n, (int)k, alpha, beta, h->d_status, h->wait_limit_ns, bias, relu};
    cudaError_t e = cudaLaunchKernelEx(&cfg, sgemm_3xtf32_kernel, tmA, tmB, args);
    if (e != cudaSuccess) return fail_cuda(e, "3xtf32 launch");
    return B2B_OK;
}

}  // namespace b2b
