// internal.h -- handle layout, error plumbing and kernel-launch declarations
// shared by the translation units of libb2blas.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "b2blas.h"

// Device status word values written by kernels whose waits are bounded.
// The low byte names the wait that gave up.
#define B2B_DEVSTAT_TIMEOUT 0x100
// Layout of the handle's 256-byte device status block (zeroed at creation):
//   byte   0: int status word (bounded-wait timeouts)
//   byte  64: unsigned reduction ticket counter (back to 0 after each reduction)
//   byte 128: 8-byte result slot of the blocking reductions
#define B2B_STATUS_REDUCE_COUNTER 64
#define B2B_STATUS_REDUCE_RESULT 128

struct b2b_handle {
    int device = 0;
    int sm_count = 0;
    int sm_clock_khz = 0;
    cudaStream_t own_stream = nullptr;  // created by b2b_create
    cudaStream_t stream = nullptr;      // where work is issued (own or caller's)
    int *d_status = nullptr;            // device status block (layout above)
    cudaEvent_t switch_event = nullptr; // orders a newly set stream behind the previous one
    // Grow-only device scratch for kernels that need it (split reductions).
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    // Grow-only device staging for the host-slice calls (operands copied in).
    void *staging = nullptr;
    size_t staging_bytes = 0;
    // Streams and events of the host-slice calls' copy pipeline (created on
    // first use): `up` carries host-to-device copies, `down` device-to-host.
    cudaStream_t copy_stream = nullptr;  // up
    cudaStream_t down_stream = nullptr;
    // Second compute lane of the host-slice GEMM pipeline: consecutive tiles
    // alternate between `stream` and this one (each with its own workspace),
    // so one tile's last wave overlaps the next tile's first.
    cudaStream_t compute2 = nullptr;
    void *workspace2 = nullptr;
    size_t workspace2_bytes = 0;
    cudaEvent_t *pipe_events = nullptr;
    int pipe_event_count = 0;
    // Copy scheduling of large host-slice GEMMs: 0 = phased (device-to-host
    // copies start after the last host-to-device copy), 1 = full duplex (both
    // directions at once).  Which is faster depends on the host's PCIe/memory
    // path, so the first two large calls try one each and later calls use the
    // faster (B2B_COPY_MODE=0/1 forces one).
    int copy_mode_forced = -1;
    int host_panels = 8;                // row panels of a large host-slice GEMM (B2B_HOST_PANELS)
    int host_col_panels = 0;            // column panels of B in a large host-slice GEMM; 0 = auto (B2B_HOST_COL_PANELS)
    int host_lanes = 2;                 // compute lanes of the host-slice GEMM pipeline, 1 or 2 (B2B_HOST_LANES)
    double copy_mode_ms_per_gb[2] = {0.0, 0.0};
    // Upper bound on any single bounded device wait, in nanoseconds.
    uint64_t wait_limit_ns = 2000000000ull;
    // HGEMM: use the single-CTA tensor-core kernel even where the CTA-pair
    // kernel applies (B2B_HGEMM_SINGLE_CTA=1; for comparisons and tests).
    bool force_single_cta = false;
    // SGEMM kernel configuration (B2B_SGEMM_VARIANT; 0 = the default).
    int sgemm_variant = 0;
    int sgemm_group_m = 0;              // TMA-fed SGEMM raster group override (B2B_SGEMM_GROUP_M; 0 = default)
    // TMA-fed SGEMM split-K factor for the next launches (0 = chosen per call;
    // set by host-slice calls so that their tiles share the whole GEMM's k
    // ranges; B2B_SGEMM_KSPLIT sets it for every call, 1 turns split-K off).
    int sgemm_ksplit_forced = 0;
    int hgemm_variant = 0;              // 0 auto, 1 single CTA, 2 pair 256x256, 3 pair 256x512
    int hgemm_group_m = 0;              // pair kernels' raster group override (0 = default)
    int gather_rotate = 1;              // fused gather: rotate destinations per CTA pair (B2B_GATHER_ROTATE=0: off)
    int64_t gemv_seg_bytes = 16384;     // GEMV-N row segment size (B2B_GEMV_SEG_KB)
    // DGEMM kernel configuration (B2B_DGEMM_VARIANT; 0 = the default).
    int dgemm_variant = 0;
    int dgemm_ksplit_forced = 0;        // DGEMM split-K factor forced (B2B_DGEMM_KSPLIT, host-slice tiles); 0 = choose
    size_t noalloc_limit_floats = 0;    // b2b_sgemv_noalloc: lower scratch limit (0 = the whole array)
};

namespace b2b {

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const std::string &msg);
int fail_cuda(cudaError_t e, const char *what);

// Makes the handle's device current for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(const b2b_handle *h);
    ~DeviceGuard();
};

// Returns a device pointer to at least `bytes` of handle scratch (grown in
// stream order on the handle's stream).
int workspace(b2b_handle *h, size_t bytes, void **ptr);
int staging(b2b_handle *h, size_t bytes, void **ptr);
// CTAs of `kernel` (launched with `threads` threads and `smem` dynamic
// shared bytes) that are resident on the whole GPU at once: the occupancy
// per SM times the SM count, cached per kernel and device.  Grid-stride
// kernels launch exactly this many so no partial second wave runs.
int resident_ctas(b2b_handle *h, const void *kernel, int threads, size_t smem);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tensor map of a row-major [rows x cols] matrix for 2-D TMA tile loads:
// box of box_cols (inner, contiguous) x box_rows, 128-byte swizzle (by default),
// out-of-range elements read as zero (tma_host.cu).
int encode_tma_2d(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base, uint64_t rows,
                  uint64_t cols, uint32_t box_cols, uint32_t box_rows,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
// 3-D map: dim0 innermost (contiguous), dim1 with pitch stride1_bytes, dim2
// with pitch stride2_bytes; box box0 x box1 x 1.
int encode_tma_3d(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base, uint64_t dim0,
                  uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                  uint32_t box1, CUtensorMapSwizzle swizzle);

// ---- kernel launchers (each returns a b2b_status) --------------------------
int launch_sgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                 float beta, float *C);
int launch_sgemm_bias(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                      float beta, float *C, const float *bias, int relu);
int launch_sgemm_3xtf32_bias(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                             const float *B, float beta, float *C, const float *bias, int relu);
int launch_dgemm(b2b_handle *h, size_t m, size_t n, size_t k, double alpha, const double *A, const double *B,
                 double beta, double *C);
int launch_sgemm_strided_batched(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                                 size_t sa, const float *B, size_t sb, float beta, float *C, size_t sc,
                                 size_t batch);
int launch_hgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                 float beta, uint16_t *C);
int launch_sgemm_3xtf32(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                        const float *B, float beta, float *C);
bool dgemm_dmma_eligible(int64_t N, int64_t K, const void *A, const void *B, const void *C);
bool sgemm_tma_eligible(int64_t M, int64_t N, int64_t K, const void *A, const void *B, const void *C,
                        bool any_size = false);
bool sgemm_tma_path(int variant, int64_t M, int64_t N, int64_t K, const void *A, const void *B, const void *C,
                    bool any_size = false);
int sgemm_ksplit(int sm_count, int64_t M, int64_t N, int64_t K);
int launch_sgemm_tma(b2b_handle *h, int64_t M, int64_t N, int64_t K, float alpha, float beta, const float *A,
                     const float *B, float *C, const float *bias, int relu, int pack);
// The TMA-fed FFMA kernel reading row-major A directly (no transpose pass),
// batched over 3-D tensor maps; batch 1 for a single GEMM.
bool sgemm_tma_rowa_eligible(int64_t M, int64_t N, int64_t K, int64_t sA, int64_t sB, int64_t sC, int64_t batch,
                             const void *A, const void *B, const void *C);
// ksplit > 1 (batch 1 only): split-K on the persistent kernel, raw partial
// sums of split s to partial[s][M][N] (kb_per_split k-blocks each); the
// caller runs the reduce.
int launch_sgemm_tma_rowa(b2b_handle *h, int64_t M, int64_t N, int64_t K, float alpha, float beta, const float *A,
                          int64_t sA, const float *B, int64_t sB, float *C, int64_t sC, int64_t batch,
                          const float *bias, int relu, int ksplit = 1, int64_t kb_per_split = 0,
                          float *partial = nullptr);
int dgemm_ksplit(int sm_count, int64_t M, int64_t N, int64_t K);
int launch_dgemm_dmma(b2b_handle *h, int64_t M, int64_t N, int64_t K, double alpha, double beta, const double *A,
                      const double *B, double *C);
int launch_sgemv(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const float *A, const float *x,
                 float beta, float *y);
int launch_sreduce(b2b_handle *h, int op, size_t n, const float *x, const float *y, void *d_out);
int launch_dgemv(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A, const double *x,
                 double beta, double *y);
int launch_hgemv(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A, const uint16_t *x,
                 float beta, uint16_t *y);
int launch_saxpy(b2b_handle *h, size_t n, float alpha, const float *x, float *y);
int launch_panels_to_rowmajor(b2b_handle *h, size_t elem_bytes, size_t m, size_t g, const size_t *widths,
                              const void *panels, void *C);

}  // namespace b2b
