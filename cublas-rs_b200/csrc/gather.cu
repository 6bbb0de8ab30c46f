// gather.cu -- column-sharded GEMM with the all-gather folded in, and the
// CUDA IPC helpers that give each rank device pointers to its peers' buffers.
//
// Rank g of G computes C[:, col_off : col_off + n] = alpha * A * B_g (+ beta
// * that panel) and the result must end up in every rank's full row-major C
// (m x ldc).  The reference is single-device (crates/cublas-rs/src/lib.rs:
// 57-68) and has none of this; the usual multi-GPU recipe is a GEMM into a
// panel, an NCCL all-gather of the panels and a re-layout pass.  Here:
//   * HGEMM, beta == 0, shapes of the CTA-pair kernel: the epilogue stores
//     each finished 32 x 64 box straight into every rank's C over NVLink
//     (coalesced 16-byte stores through IPC-mapped pointers), so the
//     transfer overlaps the next tiles' MMAs and no re-layout is needed;
//   * otherwise: the panel is computed into handle workspace and copied into
//     every rank's C with 2-D copies (peer copies for the other ranks).
// Callers must order consumers of C behind every rank's call (a barrier or
// collective after the call, as for the all-gather it replaces).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <string>

#include "internal.h"

using namespace b2b;

namespace b2b {
int launch_hgemm_gather_fused(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                              const uint16_t *B, uint16_t *const *dst, int ndst, int self, size_t ldc, size_t col_off,
                              bool *done);
int launch_hgemm_gather_multicast(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                                  const uint16_t *B, uint16_t *mc, uint16_t *own, size_t ldc, size_t col_off,
                                  bool *done);
}

namespace {

template <typename T>
int check_gather(b2b_handle *h, const char *fn, size_t m, size_t n, size_t k, const void *A, const void *B,
                 size_t ldc, size_t col_off, T *const *dst, int ndst, int self) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (!dst || ndst < 1 || ndst > 8 || self < 0 || self >= ndst)
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": need 1..8 destinations and self < ndst");
    for (int d = 0; d < ndst; ++d)
        if (!dst[d]) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL destination");
    if (col_off > ldc || n > ldc - col_off)
        return fail(B2B_ERR_DIMENSION, std::string(fn) + ": panel [col_off, col_off + n) exceeds ldc");
    if (m != 0 && n != 0 && k != 0 && (!A || !B)) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL operand");
    if (m != 0 && ldc > SIZE_MAX / m / sizeof(T)) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": sizes overflow");
    return B2B_OK;
}

// Compute the panel into workspace, then scatter it to every destination.
template <typename T, typename S, typename Launch>
int gather_generic(b2b_handle *h, size_t m, size_t n, size_t k, S alpha, const T *A, const T *B, S beta, size_t ldc,
                   size_t col_off, T *const *dst, int ndst, int self, Launch launch) {
    const size_t es = sizeof(T);
    void *ws = nullptr;
    if (int rc = workspace(h, m * n * es, &ws)) return rc;
    T *panel = static_cast<T *>(ws);
    cudaError_t e = cudaSuccess;
    if (beta != S(0))
        e = cudaMemcpy2DAsync(panel, n * es, dst[self] + col_off, ldc * es, n * es, m, cudaMemcpyDeviceToDevice,
                              h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "gather: reading the C panel");
    if (int rc = launch(h, m, n, k, alpha, A, B, beta, panel)) return rc;
    for (int i = 0; i < ndst && e == cudaSuccess; ++i) {
        const int d = (self + i) % ndst;  // own copy first; ranks start on different peers
        e = cudaMemcpy2DAsync(dst[d] + col_off, ldc * es, panel, n * es, n * es, m, cudaMemcpyDeviceToDevice,
                              h->stream);
    }
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "gather: panel copies");
}

}  // namespace

extern "C" {

int b2b_hgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
                     float beta, size_t ldc, size_t col_off, uint16_t *const *dst, int ndst, int self_index) {
    if (int rc = check_gather(h, "b2b_hgemm_gather", m, n, k, A, B, ldc, col_off, dst, ndst, self_index)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    DeviceGuard g(h);
    if (beta == 0.0f) {
        bool done = false;
        if (int rc = launch_hgemm_gather_fused(h, m, n, k, alpha, A, B, dst, ndst, self_index, ldc, col_off, &done))
            return rc;
        if (done) return B2B_OK;
    }
    return gather_generic(h, m, n, k, alpha, A, B, beta, ldc, col_off, dst, ndst, self_index, launch_hgemm);
}

int b2b_hgemm_gather_multicast(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                               const uint16_t *B, size_t ldc, size_t col_off, uint16_t *mc, uint16_t *own) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm_gather_multicast: NULL handle");
    if (!mc || !own) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm_gather_multicast: NULL buffer");
    if (col_off > ldc || n > ldc - col_off)
        return fail(B2B_ERR_DIMENSION, "b2b_hgemm_gather_multicast: panel [col_off, col_off + n) exceeds ldc");
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm_gather_multicast: NULL operand");
    if (ldc > SIZE_MAX / m / 2) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm_gather_multicast: sizes overflow");
    DeviceGuard g(h);
    bool done = false;
    if (int rc = launch_hgemm_gather_multicast(h, m, n, k, alpha, A, B, mc, own, ldc, col_off, &done)) return rc;
    if (!done)
        return fail(B2B_ERR_NOT_SUPPORTED,
                    "b2b_hgemm_gather_multicast: needs the CTA-pair kernel (m > 128, k and n multiples of 8, "
                    "16-byte aligned operands, ldc and col_off multiples of 8)");
    return B2B_OK;
}

int b2b_sgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                     float beta, size_t ldc, size_t col_off, float *const *dst, int ndst, int self_index) {
    if (int rc = check_gather(h, "b2b_sgemm_gather", m, n, k, A, B, ldc, col_off, dst, ndst, self_index)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    DeviceGuard g(h);
    return gather_generic(h, m, n, k, alpha, A, B, beta, ldc, col_off, dst, ndst, self_index, launch_sgemm);
}

int b2b_dgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, double alpha, const double *A, const double *B,
                     double beta, size_t ldc, size_t col_off, double *const *dst, int ndst, int self_index) {
    if (int rc = check_gather(h, "b2b_dgemm_gather", m, n, k, A, B, ldc, col_off, dst, ndst, self_index)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    DeviceGuard g(h);
    return gather_generic(h, m, n, k, alpha, A, B, beta, ldc, col_off, dst, ndst, self_index, launch_dgemm);
}

int b2b_ipc_get_handle(b2b_handle *h, void *dptr, void *handle) {
    if (!h || !dptr || !handle) return fail(B2B_ERR_INVALID_ARG, "b2b_ipc_get_handle: NULL argument");
    DeviceGuard g(h);
    cudaIpcMemHandle_t hd;
    const cudaError_t e = cudaIpcGetMemHandle(&hd, dptr);
    if (e != cudaSuccess) return fail_cuda(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(hd) == B2B_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &hd, sizeof(hd));
    return B2B_OK;
}

int b2b_ipc_open_handle(b2b_handle *h, const void *handle, void **dptr) {
    if (!h || !handle || !dptr) return fail(B2B_ERR_INVALID_ARG, "b2b_ipc_open_handle: NULL argument");
    DeviceGuard g(h);
    cudaIpcMemHandle_t hd;
    memcpy(&hd, handle, sizeof(hd));
    *dptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(dptr, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail_cuda(e, "cudaIpcOpenMemHandle");
    return B2B_OK;
}

int b2b_ipc_close_handle(b2b_handle *h, void *dptr) {
    if (!h || !dptr) return fail(B2B_ERR_INVALID_ARG, "b2b_ipc_close_handle: NULL argument");
    DeviceGuard g(h);
    const cudaError_t e = cudaIpcCloseMemHandle(dptr);
    if (e != cudaSuccess) return fail_cuda(e, "cudaIpcCloseMemHandle");
    return B2B_OK;
}

}  // extern "C"
