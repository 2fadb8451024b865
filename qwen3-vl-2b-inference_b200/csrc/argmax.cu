// Greedy decode on device, tokenizer/src/utils.cpp:34-44: the first index of
// the maximum (strict >, starting from -FLT_MAX, so NaN and -FLT_MAX never
// win and an all-losing row yields 0).  One CTA per row; returns 4 bytes per
// row instead of the 600 KB logits row.
#include <cfloat>
#include <climits>
#include "common.cuh"
#include "argmax.cuh"

namespace qvl {

__device__ __forceinline__ void better(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float *__restrict logits,
                                                           int32_t *__restrict idx, long n) {
    pdl_launch_dependents();
    pdl_wait();
    const float *row = logits + (long)blockIdx.x * n;
    float v = -FLT_MAX;
    int bi = INT_MAX;
    for (long j = threadIdx.x; j < n; j += blockDim.x) {
        const float x = row[j];
        if (x > v) { v = x; bi = (int)j; }   // ascending j: strict > keeps the first
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        better(v, bi, v2, i2);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv[w] = v; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        v = (threadIdx.x < nw) ? sv[threadIdx.x] : -FLT_MAX;
        bi = (threadIdx.x < nw) ? si[threadIdx.x] : INT_MAX;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            better(v, bi, v2, i2);
        }
        if (threadIdx.x == 0) idx[blockIdx.x] = (bi == INT_MAX) ? 0 : bi;
    }
}

cudaError_t launch_argmax_rows(const float *logits, int32_t *idx, long rows, long n,
                               cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)rows);
    cfg.blockDim = dim3(1024);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, argmax_rows_kernel, logits, idx, n);
}

}  // namespace qvl
