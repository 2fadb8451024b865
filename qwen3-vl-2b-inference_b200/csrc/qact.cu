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

// grid: (ceil(G / gpb), M); block 256; gpb = groups per block (<= 16, at
// most 8192 values).  The block's slice of x is staged in shared memory, then
// each half-warp computes the scale of one group (the reference's sequential
// fused chain cannot be split) and all 256 threads quantise the slice.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float *__restrict x,
                                                            int16_t *__restrict q,
                                                            float *__restrict s, int K, int g,
                                                            int gpb, int8_t *__restrict hi,
                                                            uint8_t *__restrict lo) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float inv_s[16];
    pdl_launch_dependents();
    pdl_wait();
    const int G = K / g;
    const int g0 = blockIdx.x * gpb;
    const int ng = min(gpb, G - g0);
    const int row = blockIdx.y;
    const size_t base = (size_t)row * K + (size_t)g0 * g;
    const int n = ng * g;
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(x + base)[i];
    __syncthreads();
    quantize_slice(xs, g, ng, q + base, s + (size_t)row * G + g0, hi ? hi + base : nullptr,
                   lo ? lo + base : nullptr, inv_s);
}

cudaError_t launch_quantize_rows(const float *x, int16_t *q, float *s, int M, int K, int g,
                                 cudaStream_t stream, int8_t *hi, uint8_t *lo) {
    const int G = K / g;
    int gpb = 8192 / g;
    gpb = gpb < 1 ? 1 : (gpb > 16 ? 16 : gpb);
    const size_t smem = (size_t)gpb * g * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(quantize_rows_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((G + gpb - 1) / gpb, M);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quantize_rows_kernel, x, q, s, K, g, gpb, hi, lo);
}

}  // namespace qvl
