#include "common.cuh"
#include "gemm_i8_tc.cuh"

namespace qvl {
bool gemm_tc_supported(size_t, size_t, size_t, size_t) { return false; }
cudaError_t launch_gemm_i8_tc(const int16_t *, const float *, const int8_t *, const float *, float *,
                              int, int, int, int, cudaStream_t) {
    return cudaErrorNotSupported;
}
}  // namespace qvl
