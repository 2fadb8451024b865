// RMSNorm with an INT8 group-quantised weight (the exporter always
// group-quantises norm weights, export_bin/export_qwen_bin.py:325), fused with
// the activation quantisation of the linear that consumes its output, and the
// INT8 embedding lookup.
//
// Reference arithmetic (layers/src/text_layer.cpp:111-147 rms_norm,
// :234-272 rms_norm_inplace), pinned against the compiled reference: the sum
// of squares is 8 float lanes (lane l accumulates x[8i+l]^2, multiply and add
// rounded separately) added in lane order; a = ss * (1/H) + eps (fused);
// inv_rms = (float)(1.0 / (double)sqrtf(a)) for rms_norm and 1.0f / sqrtf(a)
// for rms_norm_inplace; out[j] = (float)wq[j] * ((ws[j/gs] * inv_rms) * x[j]).
#include "common.cuh"
#include "tail.cuh"
#include "norm.cuh"

namespace qvl {

// grid: rows; block 256; dynamic smem 2*H floats (+ H + H/ngs with stage_w).
// out (nullable) receives the normalised row; q/qs (nullable) its
// quantisation with group qg (bit-exact with quantize_rows on `out`).
// The norm weight does not depend on the previous kernel: it is staged in
// shared memory (as floats) before the programmatic-dependent-launch wait.
__global__ void __launch_bounds__(256)
rmsnorm_quant_kernel(const float *x, const int8_t *__restrict wq,
                     const float *__restrict ws, float *out, int16_t *__restrict q,
                     float *__restrict qs, int H, int ngs, float eps, int inplace_form, int qg,
                     int8_t *__restrict hi, uint8_t *__restrict lo, int stage_w) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float scratch[65];
    pdl_launch_dependents();
    float *wqf = stage_w ? sm + 2 * H : nullptr, *wsg = stage_w ? sm + 3 * H : nullptr;
    if (stage_w) {
        for (int j = threadIdx.x; j < H; j += blockDim.x) wqf[j] = (float)wq[j];
        for (int j = threadIdx.x; j < H / ngs; j += blockDim.x) wsg[j] = ws[j];
    }
    pdl_wait();
    const int row = blockIdx.x;
    const int G = q ? H / qg : 0;
    cta_norm_quant_row(x + (size_t)row * H, wq, ws, ngs, eps, inplace_form != 0,
                       out ? out + (size_t)row * H : nullptr, q ? q + (size_t)row * H : nullptr,
                       q ? qs + (size_t)row * G : nullptr, qg, H, sm, sm + H, scratch,
                       hi ? hi + (size_t)row * H : nullptr, lo ? lo + (size_t)row * H : nullptr, wqf, wsg);
}

// grid: n_tokens; block 256.  out[t] = (float)table[id] * scale[id]
// (embedding_lookup, per-row scales, layers/src/text_layer.cpp:41-48).
__global__ void embedding_i8_kernel(const int8_t *__restrict table, const float *__restrict scales,
                                    const int32_t *__restrict ids, float *__restrict out, int H,
                                    int vocab) {
    pdl_launch_dependents();
    pdl_wait();
    int id = ids[blockIdx.x];
    if (id < 0 || id >= vocab) id = 0;
    const int8_t *r = table + (size_t)id * H;
    const float s = scales[id];
    for (int j = threadIdx.x; j < H; j += blockDim.x)
        out[(size_t)blockIdx.x * H + j] = mul_rn((float)r[j], s);
}

static void pdl_attr(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *attr, cudaStream_t st) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = st;
}

cudaError_t launch_rmsnorm_quant(const float *x, const int8_t *wq, const float *ws, float *out,
                                 int16_t *q, float *qs, int rows, int H, int ngs, float eps,
                                 bool inplace_form, int qg, cudaStream_t st, int8_t *hi, uint8_t *lo) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_attr(cfg, attr, st);
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(256);
    const size_t staged = ((size_t)3 * H + (size_t)H / ngs) * sizeof(float);
    const int stage_w = (wq != nullptr && staged <= 160 * 1024) ? 1 : 0;
    cfg.dynamicSmemBytes = stage_w ? staged : (size_t)2 * H * sizeof(float);
    if (cfg.dynamicSmemBytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)cfg.dynamicSmemBytes);
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, x, wq, ws, out, q, qs, H, ngs, eps,
                              inplace_form ? 1 : 0, qg, hi, lo, stage_w);
}

cudaError_t launch_embedding_i8(const int8_t *table, const float *scales, const int32_t *ids, float *out,
                                int n, int H, int vocab, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    pdl_attr(cfg, attr, st);
    cfg.gridDim = dim3(n);
    cfg.blockDim = dim3(256);
    return cudaLaunchKernelEx(&cfg, embedding_i8_kernel, table, scales, ids, out, H, vocab);
}

}  // namespace qvl
