// tma_host.cu -- host-side creation of TMA tensor maps (cuTensorMapEncodeTiled,
// resolved from the driver at run time so the library does not link
// libcuda directly).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "internal.h"

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

}  // namespace

namespace b2b {

int encode_tma_2d(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base, uint64_t rows,
                  uint64_t cols, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto enc = encode_fn();
    if (!enc) return fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * elem_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
    return B2B_OK;
}

int encode_tma_3d(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base, uint64_t dim0,
                  uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                  uint32_t box1, CUtensorMapSwizzle swizzle) {
    auto enc = encode_fn();
    if (!enc) return fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {dim0, dim1, dim2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2B_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (" + std::to_string(r) + ")");
    return B2B_OK;
}

}  // namespace b2b
