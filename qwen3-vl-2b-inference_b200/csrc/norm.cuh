#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace qvl {
cudaError_t launch_rmsnorm_quant(const float *x, const int8_t *wq, const float *ws, float *out,
                                 int16_t *q, float *qs, int rows, int H, int ngs, float eps,
                                 bool inplace_form, int qg, cudaStream_t st, int8_t *hi = nullptr,
                                 uint8_t *lo = nullptr);
cudaError_t launch_embedding_i8(const int8_t *table, const float *scales, const int32_t *ids, float *out,
                                int n, int H, int vocab, cudaStream_t st);
}  // namespace qvl
