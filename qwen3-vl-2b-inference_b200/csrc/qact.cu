// Activation quantisation fp32 -> int16 per K-group, bit-exact with the
// reference's inlined prologue (matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:
// 135-177; identical at :348-390 and :488-530).
//
// One half-warp per group: thread t (0..15) owns elements kk + 16j + t, which
// are exactly the reference's two 8-lane accumulators (t < 8: first vector,
// t >= 8: second).  The fused x*x chain runs over j in the reference order,
// then the 8+8 -> 8 -> 4 -> 1 combination is done with shuffles in the order
// of _mm256_add_ps + add_reduce_mm_256.
#include "common.cuh"
#include "qact.cuh"

namespace qvl {

// grid: (ceil(G / 8), M); block: 128 threads = 8 half-warps, one group each.
__global__ void __launch_bounds__(128) quantize_rows_kernel(const float *__restrict x,
                                                            int16_t *__restrict q,
                                                            float *__restrict s, int K, int g) {
    pdl_launch_dependents();
    pdl_wait();
    const int G = K / g;
    int gi = blockIdx.x * 8 + (threadIdx.x >> 4);
    const int row = blockIdx.y;
    const bool active = gi < G;   // whole half-warps only: keep them in the shuffles
    if (!active) gi = G - 1;
    const size_t off = (size_t)row * K + (size_t)gi * g;
    quantize_group(x + off, q + off, s + (size_t)row * G + gi, g, threadIdx.x & 15, active);
}

cudaError_t launch_quantize_rows(const float *x, int16_t *q, float *s, int M, int K, int g,
                                 cudaStream_t stream) {
    const int G = K / g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((G + 7) / 8, M);
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quantize_rows_kernel, x, q, s, K, g);
}

}  // namespace qvl
