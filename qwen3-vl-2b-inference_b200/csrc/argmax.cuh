#pragma once
#include <cuda_runtime.h>
#include <cstdint>
namespace qvl {
cudaError_t launch_argmax_rows(const float *logits, int32_t *idx, long rows, long n,
                               cudaStream_t stream);
}
