// sgemm_3xtf32.cu -- opt-in split-precision SGEMM on the tensor cores.
#include "internal.h"

namespace b2b {

int launch_sgemm_3xtf32(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A, const float *B,
                        float beta, float *C) {
    (void)h; (void)m; (void)n; (void)k; (void)alpha; (void)A; (void)B; (void)beta; (void)C;
    return fail(B2B_ERR_NOT_SUPPORTED, "b2b_sgemm: B2B_ALGO_3XTF32 is not available in this build");
}

}  // namespace b2b
