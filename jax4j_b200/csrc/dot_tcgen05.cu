// dot_tcgen05.cu -- FP32 GEMM on the 5th-generation tensor cores (placeholder
// until the tcgen05 kernel lands: reports no supported shapes).
#include "common.cuh"

namespace j4c {
bool tc_gemm_supported(int64_t, int64_t, int64_t) { return false; }
int tc_gemm_workspace(int64_t, int64_t, int64_t, size_t *bytes) {
    *bytes = 0;
    return J4C_OK;
}
int tc_gemm_f32(const float *, const float *, float *, int64_t, int64_t, int64_t, int, int, void *,
                size_t, cudaStream_t) {
    return set_error(J4C_E_UNSUPPORTED, "tensor-core GEMM not built");
}
}  // namespace j4c
