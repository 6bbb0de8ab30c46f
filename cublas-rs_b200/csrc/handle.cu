// handle.cu -- b2b_handle lifecycle, stream, device status word, device
// memory helpers and error reporting.
//
// Replaces what cublas-rs gets from cuda-oxide: the context + default stream
// of Handle::with_device (crates/cublas-rs/src/lib.rs:57-68), the
// DeviceBuffer helpers behind Handle::upload / download (lib.rs:88-97) and
// the PTX module loading (crates/cublas-l3/src/lib.rs:51-61).  There is no
// module loading here: the kernels are linked into this library for sm_100a.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "internal.h"

namespace b2b {

static thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
    g_last_error = msg;
    return code;
}

int fail_cuda(cudaError_t e, const char *what) {
    std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    g_last_error = m;
    if (e == cudaErrorMemoryAllocation) return B2B_ERR_ALLOC;
    return B2B_ERR_CUDA;
}

DeviceGuard::DeviceGuard(const b2b_handle *h) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != h->device) {
        cudaSetDevice(h->device);
        changed = true;
    }
}

DeviceGuard::~DeviceGuard() {
    if (changed) cudaSetDevice(prev);
}

static int grow(b2b_handle *h, void **buf, size_t *have, size_t bytes, void **ptr, const char *what) {
    if (bytes <= *have && *buf) {
        *ptr = *buf;
        return B2B_OK;
    }
    size_t want = bytes < 256 ? 256 : bytes;
    // Stream-ordered free/alloc: work already queued on the stream keeps
    // using the old block until it completes.
    if (*buf) {
        cudaError_t e = cudaFreeAsync(*buf, h->stream);
        if (e != cudaSuccess) return fail_cuda(e, what);
        *buf = nullptr;
        *have = 0;
    }
    cudaError_t e = cudaMallocAsync(buf, want, h->stream);
    if (e != cudaSuccess) {
        *buf = nullptr;
        return fail_cuda(e, what);
    }
    *have = want;
    *ptr = *buf;
    return B2B_OK;
}

int workspace(b2b_handle *h, size_t bytes, void **ptr) {
    return grow(h, &h->workspace, &h->workspace_bytes, bytes, ptr, "workspace allocation");
}

int staging(b2b_handle *h, size_t bytes, void **ptr) {
    return grow(h, &h->staging, &h->staging_bytes, bytes, ptr, "staging allocation");
}

int resident_ctas(b2b_handle *h, const void *kernel, int threads, size_t smem) {
    struct Entry {
        const void *kernel;
        int device, threads;
        size_t smem;
        int ctas;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry &e : cache)
            if (e.kernel == kernel && e.device == h->device && e.threads == threads && e.smem == smem) return e.ctas;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int ctas = per_sm * h->sm_count;
    std::lock_guard<std::mutex> lock(mu);
    cache.push_back(Entry{kernel, h->device, threads, smem, ctas});
    return ctas;
}

}  // namespace b2b

using namespace b2b;

extern "C" {

int b2b_version(void) { return (0 << 16) | (1 << 8) | 0; }

const char *b2b_last_error(void) { return g_last_error.c_str(); }

const char *b2b_status_string(int s) {
    switch (s) {
        case B2B_OK: return "ok";
        case B2B_ERR_CUDA: return "CUDA error";
        case B2B_ERR_DIMENSION: return "dimension mismatch";
        case B2B_ERR_INVALID_ARG: return "invalid argument";
        case B2B_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case B2B_ERR_NOT_SUPPORTED: return "not supported";
        case B2B_ERR_ALLOC: return "allocation failed";
        default: return "unknown status";
    }
}

int b2b_create(int device, b2b_handle **out) {
    if (!out) return fail(B2B_ERR_INVALID_ARG, "b2b_create: out is NULL");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(B2B_ERR_INVALID_ARG, "b2b_create: device " + std::to_string(device) + " out of range (" +
                                             std::to_string(count) + " devices)");
    int prev = -1;
    cudaGetDevice(&prev);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return fail(B2B_ERR_NOT_SUPPORTED, std::string("b2b_create: device ") + prop.name +
                                               " is not sm_100 (this library is built for sm_100a only)");
    b2b_handle *h = new (std::nothrow) b2b_handle();
    if (!h) return fail(B2B_ERR_ALLOC, "b2b_create: out of host memory");
    h->device = device;
    h->sm_count = prop.multiProcessorCount;
    int clk = 0;
    cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
    h->sm_clock_khz = clk;
    e = cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&h->d_status, 256);
    if (e == cudaSuccess) e = cudaMemset(h->d_status, 0, 256);
    if (e != cudaSuccess) {
        int rc = fail_cuda(e, "b2b_create");
        if (h->d_status) cudaFree(h->d_status);
        if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
        if (h->own_stream) cudaStreamDestroy(h->own_stream);
        delete h;
        return rc;
    }
    h->stream = h->own_stream;
    const char *lim = getenv("B2B_WAIT_LIMIT_MS");
    if (lim) {
        long v = atol(lim);
        if (v > 0) h->wait_limit_ns = static_cast<uint64_t>(v) * 1000000ull;
    }
    if (const char *cm = getenv("B2B_COPY_MODE")) h->copy_mode_forced = (cm[0] == '1') ? 1 : (cm[0] == '0' ? 0 : -1);
    if (const char *v = getenv("B2B_HOST_PANELS")) {
        const int p = atoi(v);
        if (p >= 1 && p <= 64) h->host_panels = p;
    }
    if (const char *v = getenv("B2B_HOST_COL_PANELS")) {
        const int p = atoi(v);
        if (p >= 1 && p <= 16) h->host_col_panels = p;
    }
    if (const char *v = getenv("B2B_HOST_LANES")) {
        const int p = atoi(v);
        if (p == 1 || p == 2) h->host_lanes = p;
    }
    const char *single = getenv("B2B_HGEMM_SINGLE_CTA");
    h->force_single_cta = single && single[0] == '1';
    if (const char *v = getenv("B2B_SGEMM_VARIANT")) h->sgemm_variant = atoi(v);
    if (const char *v = getenv("B2B_SGEMM_GROUP_M")) h->sgemm_group_m = atoi(v);
    if (const char *v = getenv("B2B_SGEMM_KSPLIT")) {
        const int ks = atoi(v);
        if (ks >= 0 && ks <= 16) h->sgemm_ksplit_forced = ks;
    }
    if (const char *v = getenv("B2B_HGEMM_VARIANT")) h->hgemm_variant = atoi(v);
    if (const char *v = getenv("B2B_HGEMM_GROUP_M")) h->hgemm_group_m = atoi(v);
    if (const char *v = getenv("B2B_GATHER_ROTATE")) h->gather_rotate = atoi(v) != 0;
    if (const char *v = getenv("B2B_GEMV_SEG_KB")) {
        const long kb = atol(v);
        if (kb > 0) h->gemv_seg_bytes = static_cast<int64_t>(kb) * 1024;
    }
    if (const char *v = getenv("B2B_DGEMM_VARIANT")) h->dgemm_variant = atoi(v);
    if (const char *v = getenv("B2B_DGEMM_KSPLIT")) {
        const int ks = atoi(v);
        if (ks >= 0 && ks <= 16) h->dgemm_ksplit_forced = ks;
    }
    if (const char *v = getenv("B2B_NOALLOC_SCRATCH_FLOATS")) h->noalloc_limit_floats = strtoull(v, nullptr, 10);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    *out = h;
    return B2B_OK;
}

int b2b_destroy(b2b_handle *h) {
    if (!h) return B2B_OK;
    DeviceGuard g(h);
    if (h->own_stream) cudaStreamSynchronize(h->own_stream);
    if (h->stream && h->stream != h->own_stream) cudaStreamSynchronize(h->stream);
    if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
    if (h->down_stream) cudaStreamSynchronize(h->down_stream);
    if (h->compute2) cudaStreamSynchronize(h->compute2);
    for (int i = 0; i < h->pipe_event_count; ++i) cudaEventDestroy(h->pipe_events[i]);
    delete[] h->pipe_events;
    if (h->switch_event) cudaEventDestroy(h->switch_event);
    if (h->down_stream) cudaStreamDestroy(h->down_stream);
    if (h->workspace) cudaFree(h->workspace);
    if (h->workspace2) cudaFree(h->workspace2);
    if (h->compute2) cudaStreamDestroy(h->compute2);
    if (h->staging) cudaFree(h->staging);
    if (h->d_status) cudaFree(h->d_status);
    if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
    if (h->own_stream) cudaStreamDestroy(h->own_stream);
    delete h;
    return B2B_OK;
}

int b2b_get_stream(b2b_handle *h, void **stream) {
    if (!h || !stream) return fail(B2B_ERR_INVALID_ARG, "b2b_get_stream: NULL argument");
    *stream = reinterpret_cast<void *>(h->stream);
    return B2B_OK;
}

int b2b_set_stream(b2b_handle *h, void *stream) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_set_stream: NULL handle");
    cudaStream_t next = stream ? reinterpret_cast<cudaStream_t>(stream) : h->own_stream;
    if (next == h->stream) return B2B_OK;
    // Order the new stream behind the work already queued on the old one:
    // both use the handle's workspace and reduction counter.
    DeviceGuard g(h);
    cudaError_t e = cudaSuccess;
    if (!h->switch_event) e = cudaEventCreateWithFlags(&h->switch_event, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(h->switch_event, h->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(next, h->switch_event, 0);
    if (e != cudaSuccess) return fail_cuda(e, "b2b_set_stream");
    h->stream = next;
    return B2B_OK;
}

int b2b_synchronize(b2b_handle *h) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_synchronize: NULL handle");
    DeviceGuard g(h);
    cudaError_t e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaStreamSynchronize");
    int st = 0;
    e = cudaMemcpy(&st, h->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "reading device status");
    if (st != 0) {
        cudaMemset(h->d_status, 0, sizeof(int));
        char buf[96];
        snprintf(buf, sizeof buf, "a bounded device wait gave up (status 0x%x)", st);
        return fail(B2B_ERR_DEVICE_TIMEOUT, buf);
    }
    return B2B_OK;
}

int b2b_device_info(b2b_handle *h, int *device, int *sm_count, int *sm_clock_khz) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_device_info: NULL handle");
    if (device) *device = h->device;
    if (sm_count) *sm_count = h->sm_count;
    if (sm_clock_khz) *sm_clock_khz = h->sm_clock_khz;
    return B2B_OK;
}

int b2b_malloc(b2b_handle *h, size_t bytes, void **dptr) {
    if (!h || !dptr) return fail(B2B_ERR_INVALID_ARG, "b2b_malloc: NULL argument");
    DeviceGuard g(h);
    *dptr = nullptr;
    cudaError_t e = cudaMalloc(dptr, bytes ? bytes : 1);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc");
    return B2B_OK;
}

int b2b_free(b2b_handle *h, void *dptr) {
    if (!h) return fail(B2B_ERR_INVALID_ARG, "b2b_free: NULL handle");
    if (!dptr) return B2B_OK;
    DeviceGuard g(h);
    // Frees after the work queued on the handle's stream.
    cudaError_t e = cudaStreamSynchronize(h->stream);
    if (e == cudaSuccess) e = cudaFree(dptr);
    if (e != cudaSuccess) return fail_cuda(e, "cudaFree");
    return B2B_OK;
}

int b2b_memcpy_h2d(b2b_handle *h, void *dst, const void *src, size_t bytes) {
    if (!h || (bytes && (!dst || !src))) return fail(B2B_ERR_INVALID_ARG, "b2b_memcpy_h2d: NULL argument");
    if (!bytes) return B2B_OK;
    DeviceGuard g(h);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, h->stream);
    // The source may be pageable and owned by a caller that frees it on
    // return, as DeviceBuffer::from_host allows; finish the copy first.
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "host-to-device copy");
    return B2B_OK;
}

int b2b_memcpy_d2h(b2b_handle *h, void *dst, const void *src, size_t bytes) {
    if (!h || (bytes && (!dst || !src))) return fail(B2B_ERR_INVALID_ARG, "b2b_memcpy_d2h: NULL argument");
    if (!bytes) return B2B_OK;
    DeviceGuard g(h);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "device-to-host copy");
    return B2B_OK;
}

int b2b_memcpy_d2d(b2b_handle *h, void *dst, const void *src, size_t bytes) {
    if (!h || (bytes && (!dst || !src))) return fail(B2B_ERR_INVALID_ARG, "b2b_memcpy_d2d: NULL argument");
    if (!bytes) return B2B_OK;
    DeviceGuard g(h);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "device-to-device copy");
    return B2B_OK;
}

int b2b_memset(b2b_handle *h, void *dptr, int value, size_t bytes) {
    if (!h || (bytes && !dptr)) return fail(B2B_ERR_INVALID_ARG, "b2b_memset: NULL argument");
    if (!bytes) return B2B_OK;
    DeviceGuard g(h);
    cudaError_t e = cudaMemsetAsync(dptr, value, bytes, h->stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync");
    return B2B_OK;
}

int b2b_host_alloc(size_t bytes, void **hptr) {
    if (!hptr) return fail(B2B_ERR_INVALID_ARG, "b2b_host_alloc: NULL argument");
    *hptr = nullptr;
    cudaError_t e = cudaHostAlloc(hptr, bytes ? bytes : 1, cudaHostAllocPortable);
    if (e != cudaSuccess) return fail_cuda(e, "cudaHostAlloc");
    return B2B_OK;
}

int b2b_host_free(void *hptr) {
    if (!hptr) return B2B_OK;
    cudaError_t e = cudaFreeHost(hptr);
    if (e != cudaSuccess) return fail_cuda(e, "cudaFreeHost");
    return B2B_OK;
}

}  // extern "C"
