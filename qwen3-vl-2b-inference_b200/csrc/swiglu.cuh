#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace qvl {
cudaError_t launch_swiglu(float *gate, const float *up, long n, cudaStream_t stream);
// q/s = quantize_rows(swiglu(gate, up)) for M rows of I values, group g.
cudaError_t launch_swiglu_quant(const float *gate, const float *up, int16_t *q, float *s, int M,
                                int I, int g, cudaStream_t stream);
// y = expf_host(x): the device restatement of the host expf, for its tests
cudaError_t launch_expf_host(const float *x, float *y, long n, cudaStream_t stream);
}  // namespace qvl
