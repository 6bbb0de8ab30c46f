// selftest.cu -- exercises the bounded device waits used by the tensor-core
// kernels: one CTA waits on an mbarrier that nothing ever arrives at, gives
// up after `limit_ns`, records the timeout in the handle's device status
// word and returns normally.  The context stays usable; b2b_synchronize then
// reports B2B_ERR_DEVICE_TIMEOUT.
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"
#include "sm100.cuh"

namespace {

__global__ void bounded_wait_selftest_kernel(int *status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        abort_flag = 0;
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // Phase 0 never completes: the wait must time out.
        sm100::mbar_wait(&bar, 0, &abort_flag, status, B2B_DEVSTAT_TIMEOUT | 0x7f, limit_ns);
    }
    __syncthreads();
}

}  // namespace

extern "C" int b2b_selftest_bounded_wait(b2b_handle *h, uint64_t limit_ns) {
    if (!h) return b2b::fail(B2B_ERR_INVALID_ARG, "b2b_selftest_bounded_wait: NULL handle");
    if (limit_ns == 0 || limit_ns > 5000000000ull)
        return b2b::fail(B2B_ERR_INVALID_ARG, "b2b_selftest_bounded_wait: limit must be in (0, 5 s]");
    b2b::DeviceGuard g(h);
    bounded_wait_selftest_kernel<<<1, 32, 0, h->stream>>>(h->d_status, limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return b2b::fail_cuda(e, "bounded-wait self-test launch");
    return B2B_OK;
}
