// host_slices.cu -- the host-slice ("_simple") flavours: copy the operands in,
// run the kernel, copy the result out, block until it is on the host.
//
// Mirrors cublas_l3::sgemm_* / dgemm_* / hgemm_half / strided_batched_sgemm /
// batched_sgemm and cublas_l2::sgemv* / cublas_l1::saxpy host launchers
// (crates/cublas-l3/src/sgemm.rs:401-424, hgemm.rs:135-187,
// batched.rs:162-261, crates/cublas-l2/src/gemv.rs:266-305,
// crates/cublas-l1/src/saxpy.rs:45-66), including their length checks, which
// the reference enforces with assert! and which return B2B_ERR_DIMENSION here.
//
// Differences, all in the data movement, none in the results:
//   * Device staging is a grow-only buffer owned by the handle instead of
//     three fresh allocations per call.
//   * C is not uploaded when beta == 0 (it is not read).
//   * The GEMMs split M into row panels and pipeline them over three
//     streams: B goes up first, then panel p's rows of A (and C) go up on the
//     upload stream while panel p-1 computes; each panel's C comes back on
//     the download stream.  Whether downloads may run while uploads are
//     still going (full duplex) or should wait for the last upload (phased)
//     depends on the host: some PCIe/host-memory paths lose most of their
//     bandwidth when both directions run at once.  Large calls therefore try
//     each schedule once and keep the faster.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <chrono>
#include <new>
#include <string>
#include <utility>
#include <vector>

#include "internal.h"

using namespace b2b;

namespace {

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int dim_err(const char *fn, const char *what, size_t expected, size_t got) {
    return fail(B2B_ERR_DIMENSION, std::string(fn) + ": dimension mismatch in " + what + ": expected " +
                                       std::to_string(expected) + ", got " + std::to_string(got));
}

// The handle's copy streams and at least `nev` events (created on first use).
int pipe_setup(b2b_handle *h, int nev) {
    cudaError_t e = cudaSuccess;
    if (!h->down_stream) e = cudaStreamCreateWithFlags(&h->down_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess && !h->compute2) e = cudaStreamCreateWithFlags(&h->compute2, cudaStreamNonBlocking);
    if (e == cudaSuccess && h->pipe_event_count < nev) {
        cudaEvent_t *ev = new (std::nothrow) cudaEvent_t[nev];
        if (!ev) return fail(B2B_ERR_ALLOC, "pipeline events: out of host memory");
        int i = 0;
        for (; i < h->pipe_event_count; ++i) ev[i] = h->pipe_events[i];
        for (; i < nev && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            for (int j = h->pipe_event_count; j < i - 1; ++j) cudaEventDestroy(ev[j]);
            delete[] ev;
        } else {
            delete[] h->pipe_events;
            h->pipe_events = ev;
            h->pipe_event_count = nev;
        }
    }
    if (e != cudaSuccess) return fail_cuda(e, "pipeline setup");
    return B2B_OK;
}

int finish(b2b_handle *h) {
    cudaError_t e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "host-slice call");
    int st = 0;
    e = cudaMemcpy(&st, h->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "reading device status");
    if (st) {
        cudaMemset(h->d_status, 0, sizeof(int));
        return fail(B2B_ERR_DEVICE_TIMEOUT, "a bounded device wait gave up (status " + std::to_string(st) + ")");
    }
    return B2B_OK;
}

// Pipelined host-slice GEMM for element type T, with `launch` the device
// launcher for one row panel.
// While alive, the handle issues work on its second compute lane: stream
// and workspace swap with compute2 / workspace2 (a launch's scratch, such as
// the SGEMM's transposed A, must not be shared by two lanes in flight).
struct SecondLane {
    b2b_handle *h;
    explicit SecondLane(b2b_handle *hh) : h(hh) { swap_lane(); }
    ~SecondLane() { swap_lane(); }
    void swap_lane() {
        std::swap(h->stream, h->compute2);
        std::swap(h->workspace, h->workspace2);
        std::swap(h->workspace_bytes, h->workspace2_bytes);
    }
    SecondLane(const SecondLane &) = delete;
    SecondLane &operator=(const SecondLane &) = delete;
};

// Copy schedule for a pipelined call (see b2b_handle::copy_mode_*): 0 phased
// (downloads wait for the last upload), 1 full duplex.  Large calls try each
// once, then keep the faster; small ones stay phased.
int copy_mode(const b2b_handle *h, bool large) {
    if (h->copy_mode_forced >= 0) return h->copy_mode_forced;
    if (!large || h->copy_mode_ms_per_gb[0] == 0.0) return 0;
    if (h->copy_mode_ms_per_gb[1] == 0.0) return 1;
    return h->copy_mode_ms_per_gb[1] < h->copy_mode_ms_per_gb[0] ? 1 : 0;
}

void record_copy_mode(b2b_handle *h, bool large, int mode, std::chrono::steady_clock::time_point t_start,
                      size_t bytes) {
    if (!large || h->copy_mode_forced >= 0) return;
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_start).count();
    const double per_gb = ms / (static_cast<double>(bytes) / 1e9);
    double &slot = h->copy_mode_ms_per_gb[mode];
    slot = slot == 0.0 ? per_gb : (slot < per_gb ? slot : per_gb);
}

template <typename T, typename S, typename Launch>
int gemm_simple(b2b_handle *h, const char *fn, size_t m, size_t n, size_t k, S alpha, const T *A, size_t a_len,
                const T *B, size_t b_len, S beta, T *C, size_t c_len, Launch launch) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    // Same order as the reference: length asserts first, then the early
    // return on empty dimensions (sgemm.rs:469-474).
    if (a_len != m * k) return dim_err(fn, "A length (m*k)", m * k, a_len);
    if (b_len != k * n) return dim_err(fn, "B length (k*n)", k * n, b_len);
    if (c_len != m * n) return dim_err(fn, "C length (m*n)", m * n, c_len);
    if (m == 0 || n == 0 || k == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    DeviceGuard g(h);
    const size_t ea = m * k * sizeof(T), eb = k * n * sizeof(T), ec = m * n * sizeof(T);
    const size_t oa = 0, ob = round_up(ea, 256), oc = ob + round_up(eb, 256);
    void *stage = nullptr;
    int rc = staging(h, oc + round_up(ec, 256), &stage);
    if (rc) return rc;
    T *dA = reinterpret_cast<T *>(static_cast<char *>(stage) + oa);
    T *dB = reinterpret_cast<T *>(static_cast<char *>(stage) + ob);
    T *dC = reinterpret_cast<T *>(static_cast<char *>(stage) + oc);
    const bool up_c = beta != S(0);

    // Tiles of C: row panels of A (~8 for large problems, multiples of 128
    // rows so the tensor-core tiles of a panel start on a tile boundary)
    // times column panels of B (nb of them, multiples of 256 columns).  Each
    // piece is contiguous on the device (2-D copies gather and scatter the
    // host's row-major slices), so tile (i, j) is an ordinary GEMM of A_i and
    // B_j.  Uploads interleave B_j with A_j so that the first tiles, and with
    // them the device-to-host copies of C, start after a fraction of B has
    // arrived instead of all of it.
    const size_t bytes = ea + eb + ec;
    const bool large = bytes >= (size_t(64) << 20);
    int panels = large ? h->host_panels : 1;
    size_t prow = round_up((m + panels - 1) / panels, 128);
    if (prow > m) prow = m;
    panels = static_cast<int>((m + prow - 1) / prow);
    // Column panels shorten the wait for the first tile (it needs only B_0):
    // 4 for f16, whose call the copies bound; 2 for FP32/FP64, whose tiles
    // must stay large (a 1024 x 4096 FP32 tile is 128 CTAs of 128 x 256; the
    // two compute lanes below keep the GPU full across tile boundaries).
    int nb = large ? (h->host_col_panels > 0 ? h->host_col_panels : (sizeof(T) == 2 ? 4 : 2)) : 1;
    size_t pcol = round_up((n + nb - 1) / nb, 256);
    if (pcol > n) pcol = n;
    nb = static_cast<int>((n + pcol - 1) / pcol);
    auto rows_of = [&](int i) { return (static_cast<size_t>(i) + 1) * prow <= m ? prow : m - i * prow; };
    auto cols_of = [&](int j) { return (static_cast<size_t>(j) + 1) * pcol <= n ? pcol : n - j * pcol; };
    // Device layout: A as is (row panels are contiguous), B panel j at
    // dB + k * j * pcol (k x cols_of(j)), C tile (i, j) at
    // dC + i * prow * n + rows_of(i) * j * pcol (rows_of(i) x cols_of(j)).
    auto dB_of = [&](int j) { return dB + k * (static_cast<size_t>(j) * pcol); };
    auto dC_of = [&](int i, int j) { return dC + static_cast<size_t>(i) * prow * n + rows_of(i) * (j * pcol); };

    const int nev = panels + nb + panels * nb + 3;
    if ((rc = pipe_setup(h, nev))) return rc;
    cudaEvent_t *ev_a = h->pipe_events;                    // A_i (and C_i) uploaded
    cudaEvent_t *ev_b = ev_a + panels;                     // B_j uploaded
    cudaEvent_t *ev_c = ev_b + nb;                         // tile (i, j) computed
    cudaEvent_t start_ev = ev_c[panels * nb], up_done = ev_c[panels * nb + 1];
    cudaEvent_t lane2_done = ev_c[panels * nb + 2];
    cudaStream_t up = h->copy_stream, down = h->down_stream;
    const int mode = copy_mode(h, large);
    const auto t_start = std::chrono::steady_clock::now();
    cudaError_t e = cudaSuccess;
    cudaStream_t cs = h->stream;
    const size_t es = sizeof(T);
    // The compute stream's earlier work (e.g. a previous call still using
    // the staging buffer) must finish before the copies overwrite it.
    e = cudaEventRecord(start_ev, cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(up, start_ev, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(h->compute2, start_ev, 0);
    // Upload order: B_0 A_0 B_1 A_1 ... then the remaining A_i (or B_j).
    int na = 0, nbu = 0;  // pieces uploaded so far
    std::vector<std::pair<int, int>> order;  // tiles in the order they become computable
    order.reserve(static_cast<size_t>(panels) * nb);
    while ((na < panels || nbu < nb) && e == cudaSuccess) {
        if (nbu < nb && (nbu <= na || na == panels)) {
            const int j = nbu++;
            const size_t cj = cols_of(j);
            e = cudaMemcpy2DAsync(dB_of(j), cj * es, B + j * pcol, n * es, cj * es, k, cudaMemcpyHostToDevice, up);
            if (e == cudaSuccess) e = cudaEventRecord(ev_b[j], up);
            for (int i = 0; i < na; ++i) order.emplace_back(i, j);
        } else {
            const int i = na++;
            const size_t ri = rows_of(i);
            e = cudaMemcpyAsync(dA + static_cast<size_t>(i) * prow * k, A + static_cast<size_t>(i) * prow * k,
                                ri * k * es, cudaMemcpyHostToDevice, up);
            for (int j = 0; j < nb && e == cudaSuccess && up_c; ++j)
                e = cudaMemcpy2DAsync(dC_of(i, j), cols_of(j) * es, C + static_cast<size_t>(i) * prow * n + j * pcol,
                                      n * es, cols_of(j) * es, ri, cudaMemcpyHostToDevice, up);
            if (e == cudaSuccess) e = cudaEventRecord(ev_a[i], up);
            for (int j = 0; j < nbu; ++j) order.emplace_back(i, j);
        }
    }
    if (e == cudaSuccess) e = cudaEventRecord(up_done, up);
    // Tiles alternate between the two compute lanes (odd ones on compute2).
    for (size_t t = 0; t < order.size() && e == cudaSuccess; ++t) {
        const int i = order[t].first, j = order[t].second;
        const bool second = h->host_lanes == 2 && (t & 1) != 0;
        cudaStream_t ts = second ? h->compute2 : cs;
        e = cudaStreamWaitEvent(ts, ev_a[i], 0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ts, ev_b[j], 0);
        if (e != cudaSuccess) break;
        if (second) {
            SecondLane lane(h);
            rc = launch(h, rows_of(i), cols_of(j), k, alpha, dA + static_cast<size_t>(i) * prow * k, dB_of(j), beta,
                        dC_of(i, j));
        } else {
            rc = launch(h, rows_of(i), cols_of(j), k, alpha, dA + static_cast<size_t>(i) * prow * k, dB_of(j), beta,
                        dC_of(i, j));
        }
        if (rc) {
            cudaStreamSynchronize(up);
            cudaStreamSynchronize(h->compute2);
            cudaStreamSynchronize(cs);
            return rc;
        }
        e = cudaEventRecord(ev_c[i * nb + j], ts);
    }
    // The compute stream ends behind the second lane, so finishing the call
    // (and the next call's start) covers both.
    if (e == cudaSuccess) e = cudaEventRecord(lane2_done, h->compute2);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, lane2_done, 0);
    // Phased mode: the device-to-host copies wait for the last upload.
    if (e == cudaSuccess && mode == 0) e = cudaStreamWaitEvent(down, up_done, 0);
    for (size_t t = 0; t < order.size() && e == cudaSuccess; ++t) {
        const int i = order[t].first, j = order[t].second;
        e = cudaStreamWaitEvent(down, ev_c[i * nb + j], 0);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(C + static_cast<size_t>(i) * prow * n + j * pcol, n * es, dC_of(i, j),
                                  cols_of(j) * es, cols_of(j) * es, rows_of(i), cudaMemcpyDeviceToHost, down);
    }
    cudaError_t e2 = cudaStreamSynchronize(up);
    cudaError_t e3 = cudaStreamSynchronize(down);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = e3;
    if (e != cudaSuccess) {
        cudaStreamSynchronize(h->compute2);
        cudaStreamSynchronize(cs);
        return fail_cuda(e, fn);
    }
    record_copy_mode(h, large, mode, t_start, bytes);
    return finish(h);
}

// Sets one of the handle's forced split-K factors (SGEMM or DGEMM) for its
// lifetime (unless an environment override already forces one), then
// restores it.
struct ForcedKsplit {
    int *field;
    int saved;
    ForcedKsplit(b2b_handle *hh, int b2b_handle::*member, int S)
        : field(hh ? &(hh->*member) : nullptr), saved(field ? *field : 0) {
        if (field && saved == 0) *field = S;
    }
    ~ForcedKsplit() {
        if (field) *field = saved;
    }
};

int h2d(b2b_handle *h, void *d, const void *s, size_t bytes) {
    if (!bytes) return B2B_OK;
    cudaError_t e = cudaMemcpyAsync(d, s, bytes, cudaMemcpyHostToDevice, h->stream);
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "host-to-device copy");
}

int d2h(b2b_handle *h, void *d, const void *s, size_t bytes) {
    if (!bytes) return B2B_OK;
    cudaError_t e = cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToHost, h->stream);
    return e == cudaSuccess ? B2B_OK : fail_cuda(e, "device-to-host copy");
}

}  // namespace

extern "C" {

int b2b_sgemm_simple(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A,
                     size_t a_len, const float *B, size_t b_len, float beta, float *C, size_t c_len) {
    if (algo < B2B_ALGO_DEFAULT || algo > B2B_ALGO_3XTF32)
        return fail(B2B_ERR_INVALID_ARG, "b2b_sgemm_simple: unknown algo " + std::to_string(algo));
    // The tiles of a pipelined call sum the k ranges that the device call on
    // the whole (16-byte aligned) GEMM would: its split-K factor, computed
    // once here, is forced on every tile, so the result has the device call's
    // bits however the output is tiled.
    ForcedKsplit fk(h, &b2b_handle::sgemm_ksplit_forced,
                    h && algo != B2B_ALGO_3XTF32 && m && n && k &&
                            sgemm_tma_path(h->sgemm_variant, static_cast<int64_t>(m), static_cast<int64_t>(n),
                                           static_cast<int64_t>(k), nullptr, nullptr, nullptr)
                        ? sgemm_ksplit(h->sm_count, static_cast<int64_t>(m), static_cast<int64_t>(n),
                                       static_cast<int64_t>(k))
                        : 1);
    return gemm_simple<float, float>(
        h, "b2b_sgemm_simple", m, n, k, alpha, A, a_len, B, b_len, beta, C, c_len,
        [algo](b2b_handle *hh, size_t mm, size_t nn, size_t kk, float al, const float *a, const float *b, float be,
               float *c) {
            return algo == B2B_ALGO_3XTF32 ? launch_sgemm_3xtf32(hh, mm, nn, kk, al, a, b, be, c)
                                           : launch_sgemm(hh, mm, nn, kk, al, a, b, be, c);
        });
}

int b2b_dgemm_simple(b2b_handle *h, int algo, size_t m, size_t n, size_t k, double alpha, const double *A,
                     size_t a_len, const double *B, size_t b_len, double beta, double *C, size_t c_len) {
    if (algo < B2B_ALGO_DEFAULT || algo > B2B_ALGO_DOUBLE_BUF)
        return fail(B2B_ERR_INVALID_ARG, "b2b_dgemm_simple: unknown algo " + std::to_string(algo));
    // As for SGEMM: the whole GEMM's split-K factor on the DMMA path, forced on
    // every tile, so a tiled call has the device call's bits.
    ForcedKsplit fk(h, &b2b_handle::dgemm_ksplit_forced,
                    h && m && n && k && h->dgemm_variant == 0 &&
                            dgemm_dmma_eligible(static_cast<int64_t>(n), static_cast<int64_t>(k), nullptr, nullptr,
                                                nullptr)
                        ? dgemm_ksplit(h->sm_count, static_cast<int64_t>(m), static_cast<int64_t>(n),
                                       static_cast<int64_t>(k))
                        : 1);
    return gemm_simple<double, double>(h, "b2b_dgemm_simple", m, n, k, alpha, A, a_len, B, b_len, beta, C, c_len,
                                       launch_dgemm);
}

int b2b_hgemm_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A, size_t a_len,
                     const uint16_t *B, size_t b_len, float beta, uint16_t *C, size_t c_len) {
    return gemm_simple<uint16_t, float>(h, "b2b_hgemm_simple", m, n, k, alpha, A, a_len, B, b_len, beta, C, c_len,
                                        launch_hgemm);
}

int b2b_sgemm_strided_batched_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                                     size_t a_len, size_t stride_a, const float *B, size_t b_len, size_t stride_b,
                                     float beta, float *C, size_t c_len, size_t stride_c, size_t batch) {
    const char *fn = "b2b_sgemm_strided_batched_simple";
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    // batched.rs:171-173: each slice must hold batch*stride elements.
    if (a_len < batch * stride_a) return dim_err(fn, "A length (>= batch*stride_a)", batch * stride_a, a_len);
    if (b_len < batch * stride_b) return dim_err(fn, "B length (>= batch*stride_b)", batch * stride_b, b_len);
    if (c_len < batch * stride_c) return dim_err(fn, "C length (>= batch*stride_c)", batch * stride_c, c_len);
    if (m == 0 || n == 0 || k == 0 || batch == 0) return B2B_OK;
    if (!A || !B || !C) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    // Every batch must also fit inside its slice.
    const size_t need_a = (batch - 1) * stride_a + m * k, need_b = (batch - 1) * stride_b + k * n,
                 need_c = (batch - 1) * stride_c + m * n;
    if (a_len < need_a) return dim_err(fn, "A length (last batch end)", need_a, a_len);
    if (b_len < need_b) return dim_err(fn, "B length (last batch end)", need_b, b_len);
    if (c_len < need_c) return dim_err(fn, "C length (last batch end)", need_c, c_len);
    DeviceGuard g(h);
    const size_t ea = a_len * 4, eb = b_len * 4, ec = c_len * 4;
    const size_t ob = round_up(ea, 256), oc = ob + round_up(eb, 256);
    void *stage = nullptr;
    int rc = staging(h, oc + round_up(ec, 256), &stage);
    if (rc) return rc;
    float *dA = static_cast<float *>(stage);
    float *dB = reinterpret_cast<float *>(static_cast<char *>(stage) + ob);
    float *dC = reinterpret_cast<float *>(static_cast<char *>(stage) + oc);
    // Packed outputs with beta == 0: C is write-only.  Otherwise upload it
    // so that elements between batches come back unchanged.
    const bool packed = stride_c == m * n;
    const bool up_c = beta != 0.0f || !packed;
    // Chunks of consecutive batches (h->host_panels of them on large calls),
    // pipelined like the GEMMs: chunk c's A, B (and C) ranges go up on the
    // copy stream, its GEMM waits for them on the compute stream, and its C
    // range comes back on the download stream while later chunks still
    // upload (full duplex) or after the last upload (phased).  The device
    // copy mirrors the host layout, gaps included.
    const size_t bytes = ea + eb + (up_c ? ec : 0) + (packed ? batch * m * n * 4 : ec);
    const bool large = bytes >= (size_t(64) << 20);
    size_t chunks = large ? static_cast<size_t>(h->host_panels > 0 ? h->host_panels : 1) : 1;
    if (chunks > batch) chunks = batch;
    const size_t per = (batch + chunks - 1) / chunks;
    chunks = (batch + per - 1) / per;
    if ((rc = pipe_setup(h, static_cast<int>(2 * chunks + 2)))) return rc;
    cudaEvent_t *ev_up = h->pipe_events, *ev_done = ev_up + chunks;
    cudaEvent_t start_ev = ev_done[chunks], up_done = ev_done[chunks + 1];
    cudaStream_t cs = h->stream, up = h->copy_stream, down = h->down_stream;
    const int mode = copy_mode(h, large);
    const auto t_start = std::chrono::steady_clock::now();
    // [first element, end) of chunk c's batches in a strided operand
    auto span = [&](size_t c, size_t stride, size_t mat) {
        const size_t b0 = c * per, b1 = b0 + per < batch ? b0 + per : batch;
        return std::make_pair(b0 * stride, (b1 - 1) * stride + mat);
    };
    cudaError_t e = cudaEventRecord(start_ev, cs);  // earlier users of the staging buffer first
    if (e == cudaSuccess) e = cudaStreamWaitEvent(up, start_ev, 0);
    // Each operand goes up once: a chunk copies only the part of its range
    // beyond what earlier chunks copied (with a zero or overlapping stride,
    // e.g. one A for every batch, later chunks reuse what is already there
    // and nothing is rewritten under a running GEMM).
    size_t hw_a = 0, hw_b = 0, hw_c = 0;
    auto up_range = [&](float *d, const float *hsrc, std::pair<size_t, size_t> r, size_t &hw) {
        const size_t from = r.first > hw ? r.first : hw;
        if (r.second <= from) return cudaSuccess;
        hw = r.second;
        return cudaMemcpyAsync(d + from, hsrc + from, (r.second - from) * 4, cudaMemcpyHostToDevice, up);
    };
    for (size_t c = 0; c < chunks && e == cudaSuccess; ++c) {
        e = up_range(dA, A, span(c, stride_a, m * k), hw_a);
        if (e == cudaSuccess) e = up_range(dB, B, span(c, stride_b, k * n), hw_b);
        if (e == cudaSuccess && up_c) e = up_range(dC, C, span(c, stride_c, m * n), hw_c);
        if (e == cudaSuccess) e = cudaEventRecord(ev_up[c], up);
    }
    if (e == cudaSuccess) e = cudaEventRecord(up_done, up);
    for (size_t c = 0; c < chunks && e == cudaSuccess; ++c) {
        const size_t b0 = c * per, nbat = b0 + per < batch ? per : batch - b0;
        e = cudaStreamWaitEvent(cs, ev_up[c], 0);
        if (e != cudaSuccess) break;
        rc = launch_sgemm_strided_batched(h, m, n, k, alpha, dA + b0 * stride_a, stride_a, dB + b0 * stride_b,
                                          stride_b, beta, dC + b0 * stride_c, stride_c, nbat);
        if (rc) {
            cudaStreamSynchronize(up);
            cudaStreamSynchronize(cs);
            return rc;
        }
        e = cudaEventRecord(ev_done[c], cs);
    }
    if (e == cudaSuccess && mode == 0) e = cudaStreamWaitEvent(down, up_done, 0);
    for (size_t c = 0; c < chunks && e == cudaSuccess; ++c) {
        const auto rcn = span(c, stride_c, m * n);
        e = cudaStreamWaitEvent(down, ev_done[c], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(C + rcn.first, dC + rcn.first, (rcn.second - rcn.first) * 4, cudaMemcpyDeviceToHost,
                                down);
    }
    cudaError_t e2 = cudaStreamSynchronize(up);
    cudaError_t e3 = cudaStreamSynchronize(down);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = e3;
    if (e != cudaSuccess) {
        cudaStreamSynchronize(cs);
        return fail_cuda(e, fn);
    }
    record_copy_mode(h, large, mode, t_start, bytes);
    return finish(h);
}

int b2b_sgemm_batched_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *const *A,
                             const size_t *a_lens, const float *const *B, const size_t *b_lens, float beta,
                             float *const *C, const size_t *c_lens, size_t batch) {
    const char *fn = "b2b_sgemm_batched_simple";
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (batch && (!A || !B || !C || !a_lens || !b_lens || !c_lens))
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice table");
    if (m == 0 || n == 0 || k == 0 || batch == 0) return B2B_OK;
    // batched.rs:236-238: every slice has exactly its matrix's length.
    for (size_t b = 0; b < batch; ++b) {
        if (a_lens[b] != m * k) return dim_err(fn, "a[b] length (m*k)", m * k, a_lens[b]);
        if (b_lens[b] != k * n) return dim_err(fn, "b[b] length (k*n)", k * n, b_lens[b]);
        if (c_lens[b] != m * n) return dim_err(fn, "c[b] length (m*n)", m * n, c_lens[b]);
        if (!A[b] || !B[b] || !C[b]) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    }
    DeviceGuard g(h);
    const size_t sa = m * k, sb = k * n, sc = m * n;
    const size_t ea = batch * sa * 4, eb = batch * sb * 4, ec = batch * sc * 4;
    const size_t ob = round_up(ea, 256), oc = ob + round_up(eb, 256);
    void *stage = nullptr;
    int rc = staging(h, oc + round_up(ec, 256), &stage);
    if (rc) return rc;
    float *dA = static_cast<float *>(stage);
    float *dB = reinterpret_cast<float *>(static_cast<char *>(stage) + ob);
    float *dC = reinterpret_cast<float *>(static_cast<char *>(stage) + oc);
    // Gather the slices straight into the strided device layout (the
    // reference concatenates on the host first, batched.rs:228-242).
    for (size_t b = 0; b < batch; ++b) {
        if ((rc = h2d(h, dA + b * sa, A[b], sa * 4)) || (rc = h2d(h, dB + b * sb, B[b], sb * 4))) return rc;
        if (beta != 0.0f && (rc = h2d(h, dC + b * sc, C[b], sc * 4))) return rc;
    }
    rc = launch_sgemm_strided_batched(h, m, n, k, alpha, dA, sa, dB, sb, beta, dC, sc, batch);
    if (rc) return rc;
    for (size_t b = 0; b < batch; ++b)
        if ((rc = d2h(h, C[b], dC + b * sc, sc * 4))) return rc;
    return finish(h);
}

int b2b_sgemv_simple(b2b_handle *h, int algo, int trans, size_t m, size_t n, float alpha, const float *A,
                     size_t a_len, const float *x, size_t x_len, float beta, float *y, size_t y_len) {
    const char *fn = "b2b_sgemv_simple";
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (algo < B2B_ALGO_DEFAULT || algo > B2B_ALGO_DOUBLE_BUF)
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": unknown algo " + std::to_string(algo));
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": trans must be B2B_OP_N or B2B_OP_T");
    // gemv.rs:279-285: A exactly m*n, x and y at least their op lengths.
    if (a_len != m * n) return dim_err(fn, "A length (m*n)", m * n, a_len);
    const size_t xl = trans == B2B_OP_N ? n : m, yl = trans == B2B_OP_N ? m : n;
    if (x_len < xl) return dim_err(fn, "x length", xl, x_len);
    if (y_len < yl) return dim_err(fn, "y length", yl, y_len);
    if (m == 0 || n == 0) return B2B_OK;
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    DeviceGuard g(h);
    const size_t ea = m * n * 4, ex = xl * 4, ey = yl * 4;
    const size_t ox = round_up(ea, 256), oy = ox + round_up(ex, 256);
    void *stage = nullptr;
    int rc = staging(h, oy + round_up(ey, 256), &stage);
    if (rc) return rc;
    float *dA = static_cast<float *>(stage);
    float *dx = reinterpret_cast<float *>(static_cast<char *>(stage) + ox);
    float *dy = reinterpret_cast<float *>(static_cast<char *>(stage) + oy);
    if ((rc = h2d(h, dA, A, ea)) || (rc = h2d(h, dx, x, ex))) return rc;
    if (beta != 0.0f && (rc = h2d(h, dy, y, ey))) return rc;
    if ((rc = launch_sgemv(h, trans, m, n, alpha, dA, dx, beta, dy))) return rc;
    if ((rc = d2h(h, y, dy, ey))) return rc;
    return finish(h);
}

}  // extern "C"

namespace {

// dgemv / hgemv host launchers (gemv.rs:478-509, 619-673): A exactly m*n,
// x and y at least their op lengths, zero dims return after the checks;
// only the first x_len / y_len elements travel.
template <typename T, typename S, typename Launch>
int gemv_simple(b2b_handle *h, const char *fn, int trans, size_t m, size_t n, S alpha, const T *A, size_t a_len,
                const T *x, size_t x_len, S beta, T *y, size_t y_len, Launch launch) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (trans != B2B_OP_N && trans != B2B_OP_T)
        return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": trans must be B2B_OP_N or B2B_OP_T");
    if (a_len != m * n) return dim_err(fn, "A length (m*n)", m * n, a_len);
    const size_t xl = trans == B2B_OP_N ? n : m, yl = trans == B2B_OP_N ? m : n;
    if (x_len < xl) return dim_err(fn, "x length", xl, x_len);
    if (y_len < yl) return dim_err(fn, "y length", yl, y_len);
    if (m == 0 || n == 0) return B2B_OK;
    if (!A || !x || !y) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    DeviceGuard g(h);
    const size_t ea = m * n * sizeof(T), ex = xl * sizeof(T), ey = yl * sizeof(T);
    const size_t ox = round_up(ea, 256), oy = ox + round_up(ex, 256);
    void *stage = nullptr;
    int rc = staging(h, oy + round_up(ey, 256), &stage);
    if (rc) return rc;
    T *dA = static_cast<T *>(stage);
    T *dx = reinterpret_cast<T *>(static_cast<char *>(stage) + ox);
    T *dy = reinterpret_cast<T *>(static_cast<char *>(stage) + oy);
    if ((rc = h2d(h, dA, A, ea)) || (rc = h2d(h, dx, x, ex))) return rc;
    if (beta != S(0) && (rc = h2d(h, dy, y, ey))) return rc;
    if ((rc = launch(h, trans, m, n, alpha, dA, dx, beta, dy))) return rc;
    if ((rc = d2h(h, y, dy, ey))) return rc;
    return finish(h);
}

}  // namespace

extern "C" {

int b2b_dgemv_simple(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A, size_t a_len,
                     const double *x, size_t x_len, double beta, double *y, size_t y_len) {
    return gemv_simple(h, "b2b_dgemv_simple", trans, m, n, alpha, A, a_len, x, x_len, beta, y, y_len, launch_dgemv);
}

int b2b_hgemv_simple(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A, size_t a_len,
                     const uint16_t *x, size_t x_len, float beta, uint16_t *y, size_t y_len) {
    return gemv_simple(h, "b2b_hgemv_simple", trans, m, n, alpha, A, a_len, x, x_len, beta, y, y_len, launch_hgemv);
}

// sdot / snrm2 / sasum / isamax host launchers (dot.rs:81-96, nrm2.rs:75-87,
// asum.rs:74-86, iamax.rs:88-100): x (and y) at least n long, n == 0 gives
// 0 after the checks, only x[..n] (y[..n]) travel.
static int reduce_simple(b2b_handle *h, const char *fn, int op, size_t n, const float *x, size_t x_len,
                         const float *y, size_t y_len, void *result) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (!result) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL result");
    if (x_len < n) return dim_err(fn, "x length (>= n)", n, x_len);
    if (op == B2B_REDUCE_DOT && y_len < n) return dim_err(fn, "y length (>= n)", n, y_len);
    const size_t rb = op == B2B_REDUCE_IAMAX ? 8 : 4;
    if (n == 0) {
        memset(result, 0, rb);
        return B2B_OK;
    }
    if (!x || (op == B2B_REDUCE_DOT && !y)) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    DeviceGuard g(h);
    const size_t oy = round_up(n * 4, 256), ores = oy + (op == B2B_REDUCE_DOT ? round_up(n * 4, 256) : 0);
    void *stage = nullptr;
    int rc = staging(h, ores + 256, &stage);
    if (rc) return rc;
    float *dx = static_cast<float *>(stage);
    float *dy = reinterpret_cast<float *>(static_cast<char *>(stage) + oy);
    void *dres = static_cast<char *>(stage) + ores;
    if ((rc = h2d(h, dx, x, n * 4))) return rc;
    if (op == B2B_REDUCE_DOT && (rc = h2d(h, dy, y, n * 4))) return rc;
    if ((rc = launch_sreduce(h, op, n, dx, op == B2B_REDUCE_DOT ? dy : nullptr, dres))) return rc;
    uint64_t v = 0;
    if ((rc = d2h(h, &v, dres, rb))) return rc;
    if ((rc = finish(h))) return rc;
    memcpy(result, &v, rb);
    return B2B_OK;
}

int b2b_sdot_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, const float *y, size_t y_len,
                    float *result) {
    return reduce_simple(h, "b2b_sdot_simple", B2B_REDUCE_DOT, n, x, x_len, y, y_len, result);
}

int b2b_snrm2_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, float *result) {
    return reduce_simple(h, "b2b_snrm2_simple", B2B_REDUCE_NRM2, n, x, x_len, nullptr, 0, result);
}

int b2b_sasum_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, float *result) {
    return reduce_simple(h, "b2b_sasum_simple", B2B_REDUCE_ASUM, n, x, x_len, nullptr, 0, result);
}

int b2b_isamax_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, size_t *result) {
    uint64_t r = 0;
    const int rc =
        reduce_simple(h, "b2b_isamax_simple", B2B_REDUCE_IAMAX, n, x, x_len, nullptr, 0, result ? &r : nullptr);
    if (rc == B2B_OK) *result = static_cast<size_t>(r);
    return rc;
}

int b2b_saxpy_simple(b2b_handle *h, size_t n, float alpha, const float *x, size_t x_len, float *y, size_t y_len) {
    const char *fn = "b2b_saxpy_simple";
    if (!h) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL handle");
    if (x_len < n) return dim_err(fn, "x length (>= n)", n, x_len);  // saxpy.rs:53-54
    if (y_len < n) return dim_err(fn, "y length (>= n)", n, y_len);
    if (n == 0) return B2B_OK;
    if (!x || !y) return fail(B2B_ERR_INVALID_ARG, std::string(fn) + ": NULL slice");
    DeviceGuard g(h);
    const size_t oy = round_up(n * 4, 256);
    void *stage = nullptr;
    int rc = staging(h, oy + round_up(n * 4, 256), &stage);
    if (rc) return rc;
    float *dx = static_cast<float *>(stage);
    float *dy = reinterpret_cast<float *>(static_cast<char *>(stage) + oy);
    if ((rc = h2d(h, dx, x, n * 4)) || (rc = h2d(h, dy, y, n * 4))) return rc;
    if ((rc = launch_saxpy(h, n, alpha, dx, dy))) return rc;
    if ((rc = d2h(h, y, dy, n * 4))) return rc;
    return finish(h);
}

}  // extern "C"
