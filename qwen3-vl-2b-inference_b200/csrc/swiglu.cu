// SwiGLU, layers/src/text_layer.cpp:420-434:
//   gate[i] = (gate[i] / (1 + expf(-gate[i]))) * up[i]
// and its fusion with the down projection's activation quantisation
// (the down linear re-quantises the SwiGLU output,
// matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:135-177).
//
// exp is expf_host (common.cuh): the host C library's expf, bit for bit; the
// add, divide and multiply are IEEE single-precision round-to-nearest like
// the CPU's.
#include "common.cuh"
#include "qact.cuh"
#include "swiglu.cuh"

namespace qvl {


__global__ void swiglu_kernel(float *__restrict gate, const float *__restrict up, long n) {
    pdl_launch_dependents();
    pdl_wait();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        gate[i] = swiglu_one(gate[i], up[i]);
}

// grid: (ceil(G / gpb), M); block 256; gpb groups per block (<= 16, at most
// 8192 values).  All threads compute the block's SwiGLU values into shared
// memory, then each half-warp computes one group's scale (the reference's
// sequential fused chain) and all threads quantise -- the arithmetic of
// quantize_rows_kernel applied to swiglu(gate, up).
__global__ void __launch_bounds__(256)
swiglu_quant_kernel(const float *__restrict gate, const float *__restrict up,
                    int16_t *__restrict q, float *__restrict s, int I, int g, int gpb) {
    extern __shared__ __align__(16) float hs[];
    __shared__ float inv_s[16];
    pdl_launch_dependents();
    pdl_wait();
    const int G = I / g;
    const int g0 = blockIdx.x * gpb;
    const int ng = min(gpb, G - g0);
    const int row = blockIdx.y;
    const size_t base = (size_t)row * I + (size_t)g0 * g;
    const int n = ng * g;
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        const float4 a = reinterpret_cast<const float4 *>(gate + base)[i];
        const float4 b = reinterpret_cast<const float4 *>(up + base)[i];
        reinterpret_cast<float4 *>(hs)[i] = make_float4(swiglu_one(a.x, b.x), swiglu_one(a.y, b.y),
                                                        swiglu_one(a.z, b.z), swiglu_one(a.w, b.w));
    }
    __syncthreads();
    quantize_slice(hs, g, ng, q + base, s + (size_t)row * G + g0, nullptr, nullptr, inv_s);
}

__global__ void expf_host_kernel(const float *__restrict x, float *__restrict y, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        y[i] = expf_host(x[i]);
}

static void pdl_cfg(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *attr, cudaStream_t stream) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = stream;
}

cudaError_t launch_swiglu(float *gate, const float *up, long n, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_cfg(cfg, attr, stream);
    long blocks = (n + 255) / 256;
    cfg.gridDim = dim3((unsigned)(blocks < 148 * 16 ? blocks : 148 * 16));
    cfg.blockDim = dim3(256);
    return cudaLaunchKernelEx(&cfg, swiglu_kernel, gate, up, n);
}

cudaError_t launch_swiglu_quant(const float *gate, const float *up, int16_t *q, float *s, int M,
                                int I, int g, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_cfg(cfg, attr, stream);
    int gpb = 8192 / g;
    gpb = gpb < 1 ? 1 : (gpb > 16 ? 16 : gpb);
    cfg.dynamicSmemBytes = (size_t)gpb * g * sizeof(float);
    if (cfg.dynamicSmemBytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(swiglu_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)cfg.dynamicSmemBytes);
        if (e != cudaSuccess) return e;
    }
    cfg.gridDim = dim3((I / g + gpb - 1) / gpb, M);
    cfg.blockDim = dim3(256);
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, q, s, I, g, gpb);
}

cudaError_t launch_expf_host(const float *x, float *y, long n, cudaStream_t stream) {
    long blocks = (n + 255) / 256;
    expf_host_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, stream>>>(x, y, n);
    return cudaGetLastError();
}

}  // namespace qvl
