#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace qvl {
// Tensor-core (tcgen05 kind::i8) INT8 GEMM with TILED summation semantics.
bool gemm_tc_supported(size_t M, size_t N, size_t K, size_t g);
cudaError_t launch_gemm_i8_tc(const int16_t *q, const float *qs, const int8_t *W, const float *ws,
                              float *C, int M, int N, int K, int g, cudaStream_t stream);
}  // namespace qvl
