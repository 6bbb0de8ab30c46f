// timer.cu -- GpuTimer: two CUDA events around work on the handle's stream,
// the timer the reference's bench crate declares (benches/src/timer.rs:6-19,
// a todo! stub there).  The start event is recorded when the timer is made,
// the stop event at stop(), which waits for it and frees the timer.
#include <cuda_runtime.h>

#include <new>

#include "internal.h"

struct b2b_gpu_timer {
    cudaEvent_t start = nullptr;
    cudaEvent_t stop = nullptr;
    cudaStream_t stream = nullptr;
    int device = 0;
};

using namespace b2b;

extern "C" {

int b2b_gpu_timer_start(b2b_handle *h, b2b_gpu_timer **out) {
    if (!h || !out) return fail(B2B_ERR_INVALID_ARG, "b2b_gpu_timer_start: NULL argument");
    *out = nullptr;
    DeviceGuard g(h);
    b2b_gpu_timer *t = new (std::nothrow) b2b_gpu_timer;
    if (!t) return fail(B2B_ERR_ALLOC, "b2b_gpu_timer_start: out of host memory");
    t->stream = h->stream;
    t->device = h->device;
    cudaError_t e = cudaEventCreate(&t->start);
    if (e == cudaSuccess) e = cudaEventCreate(&t->stop);
    if (e == cudaSuccess) e = cudaEventRecord(t->start, t->stream);
    if (e != cudaSuccess) {
        if (t->start) cudaEventDestroy(t->start);
        if (t->stop) cudaEventDestroy(t->stop);
        delete t;
        return fail_cuda(e, "b2b_gpu_timer_start");
    }
    *out = t;
    return B2B_OK;
}

int b2b_gpu_timer_stop(b2b_gpu_timer *t, double *ms) {
    if (!t) return fail(B2B_ERR_INVALID_ARG, "b2b_gpu_timer_stop: NULL timer");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(t->device);
    cudaError_t e = cudaEventRecord(t->stop, t->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(t->stop);
    float f = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&f, t->start, t->stop);
    cudaEventDestroy(t->start);
    cudaEventDestroy(t->stop);
    delete t;
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fail_cuda(e, "b2b_gpu_timer_stop");
    if (ms) *ms = static_cast<double>(f);
    return B2B_OK;
}

}  // extern "C"
