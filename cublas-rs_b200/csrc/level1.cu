// level1.cu -- SAXPY and the panel re-layout used after a column-sharded
// GEMM's all-gather.
//
// SAXPY: y <- alpha * x + y (crates/cublas-l1/src/saxpy.rs:13-20), one 16-byte
// vector per thread per step over a grid-stride loop sized to the SM count
// (the reference launches one thread per element, saxpy.rs:36).
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace {

__global__ void __launch_bounds__(256) saxpy_vec_kernel(int64_t n4, float alpha, const float4 *__restrict__ x,
                                                        float4 *__restrict__ y) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float4 a = x[i], b = y[i];
        b.x = fmaf(alpha, a.x, b.x);
        b.y = fmaf(alpha, a.y, b.y);
        b.z = fmaf(alpha, a.z, b.z);
        b.w = fmaf(alpha, a.w, b.w);
        y[i] = b;
    }
}

__global__ void __launch_bounds__(256) saxpy_kernel(int64_t start, int64_t n, float alpha, const float *__restrict__ x,
                                                    float *__restrict__ y) {
    for (int64_t i = start + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = fmaf(alpha, x[i], y[i]);
}

constexpr int kMaxPanels = 64;
struct PanelTable {
    int64_t off[kMaxPanels + 1];  // column offset of each panel, off[g] = n
    int g;
};

// C[i, j] = panel_p[i, j - off[p]] for the panel p holding column j.
template <typename T>
__global__ void __launch_bounds__(256) panels_kernel(const T *__restrict__ panels, T *__restrict__ C, int64_t m,
                                                     int64_t n, PanelTable tab) {
    const int64_t total = m * n;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = idx / n, j = idx - i * n;
        int p = 0;
        while (p + 1 < tab.g && j >= tab.off[p + 1]) ++p;
        const int64_t w = tab.off[p + 1] - tab.off[p];
        C[idx] = panels[m * tab.off[p] + i * w + (j - tab.off[p])];
    }
}

unsigned grid_for(const b2b_handle *h, int64_t work) {
    int64_t g = (work + 255) / 256;
    int64_t cap = static_cast<int64_t>(h->sm_count) * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<unsigned>(g);
}

}  // namespace

namespace b2b {

int launch_saxpy(b2b_handle *h, size_t n_, float alpha, const float *x, float *y) {
    const int64_t n = static_cast<int64_t>(n_);
    cudaError_t e;
    if (aligned16(x) && aligned16(y)) {
        const int64_t n4 = n / 4;
        if (n4 > 0) {
            saxpy_vec_kernel<<<grid_for(h, n4), 256, 0, h->stream>>>(n4, alpha, reinterpret_cast<const float4 *>(x),
                                                                    reinterpret_cast<float4 *>(y));
            e = cudaGetLastError();
            if (e != cudaSuccess) return fail_cuda(e, "saxpy launch");
        }
        if (n4 * 4 < n) {
            saxpy_kernel<<<1, 256, 0, h->stream>>>(n4 * 4, n, alpha, x, y);
            e = cudaGetLastError();
            if (e != cudaSuccess) return fail_cuda(e, "saxpy tail launch");
        }
        return B2B_OK;
    }
    saxpy_kernel<<<grid_for(h, n), 256, 0, h->stream>>>(0, n, alpha, x, y);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "saxpy launch");
    return B2B_OK;
}

int launch_panels_to_rowmajor(b2b_handle *h, size_t elem_bytes, size_t m, size_t g, const size_t *widths,
                              const void *panels, void *C) {
    if (g < 1 || g > static_cast<size_t>(kMaxPanels))
        return fail(B2B_ERR_INVALID_ARG, "panels_to_rowmajor: panel count must be 1.." + std::to_string(kMaxPanels));
    PanelTable tab;
    tab.g = static_cast<int>(g);
    tab.off[0] = 0;
    for (size_t p = 0; p < g; ++p) tab.off[p + 1] = tab.off[p] + static_cast<int64_t>(widths[p]);
    const int64_t n = tab.off[g];
    const int64_t total = static_cast<int64_t>(m) * n;
    if (total == 0) return B2B_OK;
    const unsigned grid = grid_for(h, total);
    switch (elem_bytes) {
        case 2:
            panels_kernel<uint16_t><<<grid, 256, 0, h->stream>>>(static_cast<const uint16_t *>(panels),
                                                                static_cast<uint16_t *>(C), (int64_t)m, n, tab);
            break;
        case 4:
            panels_kernel<uint32_t><<<grid, 256, 0, h->stream>>>(static_cast<const uint32_t *>(panels),
                                                                static_cast<uint32_t *>(C), (int64_t)m, n, tab);
            break;
        case 8:
            panels_kernel<uint64_t><<<grid, 256, 0, h->stream>>>(static_cast<const uint64_t *>(panels),
                                                                static_cast<uint64_t *>(C), (int64_t)m, n, tab);
            break;
        default:
            return fail(B2B_ERR_INVALID_ARG, "panels_to_rowmajor: elem_bytes must be 2, 4 or 8");
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "panels_to_rowmajor launch");
    return B2B_OK;
}

}  // namespace b2b
