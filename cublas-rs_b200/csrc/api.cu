// api.cu -- C-ABI entry points: argument validation, then dispatch to the
// kernel launchers.  Device-pointer flavours only; the host-slice flavours
// are in host_slices.cu.
//
// Validation mirrors the reference's rules and adds the checks it lacks:
//   * m, n, k (and batch) == 0 -> B2B_OK, no launch (sgemm.rs:379-381).
//   * NULL handle or operand pointers -> B2B_ERR_INVALID_ARG.
//   * element counts whose byte size overflows 64 bits -> B2B_ERR_INVALID_ARG
//     (the reference casts to u32 and can silently wrap, batched.rs:142-152).
#include <cuda_runtime.h>
#include <stdint.h>

#include <string.h>

#include <string>

#include "internal.h"

using namespace b2b;

namespace {

bool mul_ok(size_t a, size_t b, size_t *out) {
    if (a != 0 && b > SIZE_MAX / a) return false;
    *out = a * b;
    return true;
}

bool bytes_ok(size_t a, size_t b, size_t elem) {
    size_t t;
    return mul_ok(a, b, &t) && mul_ok(t, elem, &t);
}

int check_algo(int algo, const char *fn, bool allow_3xtf32) {
    if (algo < B2B_ALGO_DEFAULT || algo > B2B_ALGO_3XTF32 || (algo == B2B_ALGO_3XTF32 && !allow_3xtf32))
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": unknown algo " + std::to_string(algo));
    return B2B_OK;
}

}  // namespace

extern "C" {

int b2b_sgemm(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
              float beta, float *C) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm: NULL handle");
    if (int rc = check_algo(algo, "b2b_sgemm", true)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm: NULL operand");
    if (!bytes_ok(m, k, 4) || !bytes_ok(k, n, 4) || !bytes_ok(m, n, 4))
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm: sizes overflow");
    DeviceGuard g(h);
    if (algo == B2B_ALGO_3XTF32) return launch_sgemm_3xtf32(h, m, n, k, alpha, A, B, beta, C);
    return launch_sgemm(h, m, n, k, alpha, A, B, beta, C);
}

int b2b_sgemm_splits(b2b_handle *h, size_t m, size_t n, size_t k, int *splits) {
    if (!h || !splits) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_splits: NULL argument");
    *splits = 1;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    const int64_t M = static_cast<int64_t>(m), N = static_cast<int64_t>(n), K = static_cast<int64_t>(k);
    if (!sgemm_tma_path(h->sgemm_variant, M, N, K, nullptr, nullptr, nullptr, h->sgemm_ksplit_forced > 1))
        return B2B_OK;
    int S = h->sgemm_ksplit_forced > 0 ? h->sgemm_ksplit_forced : sgemm_ksplit(h->sm_count, M, N, K);
    const int64_t kt = (K + 31) / 32;
    if (S > kt) S = static_cast<int>(kt);
    *splits = S < 1 ? 1 : S;
    return B2B_OK;
}

int b2b_set_sgemm_splits(b2b_handle *h, int splits) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_set_sgemm_splits: NULL handle");
    if (splits < 0 || splits > 16) return fail(B2B_ERR_INVALID_ARG, "b2b_set_sgemm_splits: splits must be 0..16");
    h->sgemm_ksplit_forced = splits;
    return B2B_OK;
}

int b2b_sgemm_bias(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A,
                   const float *B, float beta, float *C, const float *bias, int relu) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_bias: NULL handle");
    if (int rc = check_algo(algo, "b2b_sgemm_bias", true)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_bias: NULL operand");
    if (!bytes_ok(m, k, 4) || !bytes_ok(k, n, 4) || !bytes_ok(m, n, 4))
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_bias: sizes overflow");
    DeviceGuard g(h);
    const int r = relu ? 1 : 0;
    if (algo == B2B_ALGO_3XTF32) return launch_sgemm_3xtf32_bias(h, m, n, k, alpha, A, B, beta, C, bias, r);
    return launch_sgemm_bias(h, m, n, k, alpha, A, B, beta, C, bias, r);
}

int b2b_dgemm(b2b_handle *h, int algo, size_t m, size_t n, size_t k, double alpha, const double *A,
              const double *B, double beta, double *C) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_dgemm: NULL handle");
    if (int rc = check_algo(algo, "b2b_dgemm", false)) return rc;
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_dgemm: NULL operand");
    if (!bytes_ok(m, k, 8) || !bytes_ok(k, n, 8) || !bytes_ok(m, n, 8))
        return fail(B2B_ERR_INVALID_ARG, "b2b_dgemm: sizes overflow");
    DeviceGuard g(h);
    return launch_dgemm(h, m, n, k, alpha, A, B, beta, C);
}

int b2b_hgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, const uint16_t *B,
              float beta, uint16_t *C) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm: NULL handle");
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm: NULL operand");
    if (!bytes_ok(m, k, 2) || !bytes_ok(k, n, 2) || !bytes_ok(m, n, 2))
        return fail(B2B_ERR_INVALID_ARG, "b2b_hgemm: sizes overflow");
    DeviceGuard g(h);
    return launch_hgemm(h, m, n, k, alpha, A, B, beta, C);
}

int b2b_sgemm_strided_batched(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                              size_t stride_a, const float *B, size_t stride_b, float beta, float *C,
                              size_t stride_c, size_t batch) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_strided_batched: NULL handle");
    if (m == 0 || n == 0 || k == 0 || batch == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_strided_batched: NULL operand");
    if (!bytes_ok(batch, stride_a + m * k, 4) || !bytes_ok(batch, stride_b + k * n, 4) ||
        !bytes_ok(batch, stride_c + m * n, 4))
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_strided_batched: sizes overflow");
    DeviceGuard g(h);
    return launch_sgemm_strided_batched(h, m, n, k, alpha, A, stride_a, B, stride_b, beta, C, stride_c, batch);
}

int b2b_sgemv(b2b_handle *h, int algo, int trans, size_t m, size_t n, float alpha, const float *A, const float *x,
              float beta, float *y) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv: NULL handle");
    if (int rc = check_algo(algo, "b2b_sgemv", false)) return rc;
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv: trans must be B2B_OP_N or B2B_OP_T");
    if (m == 0 || n == 0) return B2B_OK;
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv: NULL operand");
    if (!bytes_ok(m, n, 4)) return fail(B2B_ERR_INVALID_ARG, "b2b_sgemv: sizes overflow");
    DeviceGuard g(h);
    return launch_sgemv(h, trans, m, n, alpha, A, x, beta, y);
}

int b2b_dgemv(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A, const double *x,
              double beta, double *y) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_dgemv: NULL handle");
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, "b2b_dgemv: trans must be B2B_OP_N or B2B_OP_T");
    if (m == 0 || n == 0) return B2B_OK;  // gemv.rs:458-460
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, "b2b_dgemv: NULL operand");
    if (!bytes_ok(m, n, 8)) return fail(B2B_ERR_INVALID_ARG, "b2b_dgemv: sizes overflow");
    DeviceGuard g(h);
    return launch_dgemv(h, trans, m, n, alpha, A, x, beta, y);
}

int b2b_hgemv(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A, const uint16_t *x,
              float beta, uint16_t *y) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemv: NULL handle");
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, "b2b_hgemv: trans must be B2B_OP_N or B2B_OP_T");
    if (m == 0 || n == 0) return B2B_OK;
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemv: NULL operand");
    if (!bytes_ok(m, n, 2)) return fail(B2B_ERR_INVALID_ARG, "b2b_hgemv: sizes overflow");
    DeviceGuard g(h);
    return launch_hgemv(h, trans, m, n, alpha, A, x, beta, y);
}

int b2b_sreduce_async(b2b_handle *h, int op, size_t n, const float *x, const float *y, void *d_result) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_sreduce_async: NULL handle");
    if (op < B2B_REDUCE_DOT || op > B2B_REDUCE_IAMAX)
        return fail(B2B_ERR_INVALID_ARG, "b2b_sreduce_async: unknown op " + std::to_string(op));
    if (!d_result) return fail(B2B_ERR_INVALID_ARG, "b2b_sreduce_async: NULL result");
    if (!bytes_ok(n, 1, 4)) return fail(B2B_ERR_INVALID_ARG, "b2b_sreduce_async: size overflows");
    DeviceGuard g(h);
    if (n == 0) {
        const cudaError_t e = cudaMemsetAsync(d_result, 0, op == B2B_REDUCE_IAMAX ? 8 : 4, h->stream);
        return e == cudaSuccess ? B2B_OK : fail_cuda(e, "b2b_sreduce_async: memset");
    }
    if (!x || (op == B2B_REDUCE_DOT && !y)) return fail(B2B_ERR_INVALID_ARG, "b2b_sreduce_async: NULL operand");
    return launch_sreduce(h, op, n, x, y, d_result);
}

namespace {

// Blocking flavour: reduce into the handle's result slot, copy it out on the
// handle's stream and wait (the reference's *_dev functions return the value,
// dot.rs:75-77).
int reduce_to_host(b2b_handle *h, const char *fn, int op, size_t n, const float *x, const float *y, void *result) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (!result) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL result");
    const size_t rb = op == B2B_REDUCE_IAMAX ? 8 : 4;
    if (n == 0) {  // dot.rs:66-68
        memset(result, 0, rb);
        return B2B_OK;
    }
    if (!x || (op == B2B_REDUCE_DOT && !y)) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL operand");
    if (!bytes_ok(n, 1, 4)) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": size overflows");
    DeviceGuard g(h);
    void *slot = reinterpret_cast<char *>(h->d_status) + B2B_STATUS_REDUCE_RESULT;
    if (int rc = launch_sreduce(h, op, n, x, y, slot)) return rc;
    uint64_t v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, slot, rb, cudaMemcpyDeviceToHost, h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return fail_cuda(e, (std::string(fn) + ": result copy").c_str());
    memcpy(result, &v, rb);
    return B2B_OK;
}

}  // namespace

int b2b_sdot(b2b_handle *h, size_t n, const float *x, const float *y, float *result) {
    return reduce_to_host(h, "b2b_sdot", B2B_REDUCE_DOT, n, x, y, result);
}

int b2b_snrm2(b2b_handle *h, size_t n, const float *x, float *result) {
    return reduce_to_host(h, "b2b_snrm2", B2B_REDUCE_NRM2, n, x, nullptr, result);
}

int b2b_sasum(b2b_handle *h, size_t n, const float *x, float *result) {
    return reduce_to_host(h, "b2b_sasum", B2B_REDUCE_ASUM, n, x, nullptr, result);
}

int b2b_isamax(b2b_handle *h, size_t n, const float *x, size_t *result) {
    uint64_t r = 0;
    const int rc = reduce_to_host(h, "b2b_isamax", B2B_REDUCE_IAMAX, n, x, nullptr, result ? &r : nullptr);
    if (rc == B2B_OK) *result = static_cast<size_t>(r);
    return rc;
}

int b2b_saxpy(b2b_handle *h, size_t n, float alpha, const float *x, float *y) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_saxpy: NULL handle");
    if (n == 0) return B2B_OK;
    if (!x || !y) return fail(B2B_ERR_INVALID_ARG, "b2b_saxpy: NULL operand");
    if (!bytes_ok(n, 1, 4)) return fail(B2B_ERR_INVALID_ARG, "b2b_saxpy: size overflows");
    DeviceGuard g(h);
    return launch_saxpy(h, n, alpha, x, y);
}

int b2b_panels_to_rowmajor(b2b_handle *h, size_t elem_bytes, size_t m, size_t g, const size_t *widths,
                           const void *panels, void *C) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_panels_to_rowmajor: NULL handle");
    if (g == 0 || !widths) return fail(B2B_ERR_INVALID_ARG, "b2b_panels_to_rowmajor: no panels");
    if (m == 0) return B2B_OK;
    if (!panels || !C) return fail(B2B_ERR_INVALID_ARG, "b2b_panels_to_rowmajor: NULL buffer");
    DeviceGuard gd(h);
    return launch_panels_to_rowmajor(h, elem_bytes, m, g, widths, panels, C);
}

}  // extern "C"
