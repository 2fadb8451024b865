// SwiGLU, layers/src/text_layer.cpp:420-434:
//   gate[i] = (gate[i] / (1 + expf(-gate[i]))) * up[i]
// and its fusion with the down projection's activation quantisation
// (the down linear re-quantises the SwiGLU output,
// matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:135-177).
//
// exp is evaluated in double precision and rounded once to fp32, which gives
// the correctly rounded expf value (glibc's expf, used by the reference, is
// correctly rounded for all but a vanishing set of inputs); the add, divide
// and multiply are IEEE single-precision round-to-nearest like the CPU's.
#include "common.cuh"
#include "qact.cuh"
#include "swiglu.cuh"

namespace qvl {

__device__ __forceinline__ float swiglu_one(float x, float u) {
    float e = (float)exp(-(double)x);
    float silu = __fdiv_rn(x, add_rn(1.0f, e));
    return mul_rn(silu, u);
}

__global__ void swiglu_kernel(float *__restrict gate, const float *__restrict up, long n) {
    pdl_launch_dependents();
    pdl_wait();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        gate[i] = swiglu_one(gate[i], up[i]);
}

// One half-warp per K-group of the SwiGLU output row, as in
// quantize_rows_kernel, with the SwiGLU value recomputed on the fly (it is
// needed twice: for the sum of squares and for the quantisation).
// grid: (ceil(G / 8), M); block 128.
__global__ void __launch_bounds__(128)
swiglu_quant_kernel(const float *__restrict gate, const float *__restrict up,
                    int16_t *__restrict q, float *__restrict s, int I, int g) {
    pdl_launch_dependents();
    pdl_wait();
    const int G = I / g;
    int gi = blockIdx.x * 8 + (threadIdx.x >> 4);
    const int row = blockIdx.y;
    const bool active = gi < G;
    if (!active) gi = G - 1;
    const int t16 = threadIdx.x & 15;
    const size_t off = (size_t)row * I + (size_t)gi * g;
    const float *gg = gate + off;
    const float *uu = up + off;
    const unsigned full = 0xffffffffu;
    float acc = 0.0f;
    for (int j = 0; j < g; j += 16) {
        float v = swiglu_one(gg[j + t16], uu[j + t16]);
        acc = fma_rn(v, v, acc);
    }
    float o = __shfl_down_sync(full, acc, 8, 16);
    float v = add_rn(acc, o);
    o = __shfl_down_sync(full, v, 4, 16);
    float u = add_rn(v, o);
    o = __shfl_down_sync(full, u, 1, 16);
    float p = add_rn(u, o);
    o = __shfl_down_sync(full, p, 2, 16);
    float ss = __shfl_sync(full, add_rn(p, o), 0, 16);
    float inv_g = __fdiv_rn(1.0f, (float)g);
    float rms = __fsqrt_rn(fma_rn(ss, inv_g, 1e-6f));
    float sc = mul_rn(rms, inv127());
    if (!active) return;
    if (t16 == 0) s[(size_t)row * G + gi] = sc;
    float inv = __fdiv_rn(1.0f, sc);
    for (int j = t16; j < g; j += 16) q[off + j] = quant_one(swiglu_one(gg[j], uu[j]), inv);
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
    cfg.gridDim = dim3((I / g + 7) / 8, M);
    cfg.blockDim = dim3(128);
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, q, s, I, g);
}

}  // namespace qvl
