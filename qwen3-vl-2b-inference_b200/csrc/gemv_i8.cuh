#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace qvl {

struct GemvArgs {
    const int16_t *q;   // [M, K] quantised activations
    const float *qs;    // [M, K/g] activation scales
    const int8_t *W;    // [N, K]
    const float *ws;    // [N * K/g]
    float *y;           // [M, ldy]
    int M, N, K, g;
    long ldy;
    int acc;            // 1: y += result (fused residual add), 0: y = result
};

bool gemv_shape_supported(int K, int g);
bool gemv_fast_eligible(int M, int K, int g);
size_t gemv_smem_bytes(int M, int K, int g);
// M <= 8 rows; lane8 selects the M=1 decode summation order.
cudaError_t launch_gemv_i8(const GemvArgs &a, bool lane8, cudaStream_t stream);

}  // namespace qvl
