#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include "common.cuh"

namespace qvl {
// hi/lo (optional, both or neither): the tensor-core GEMM's activation
// planes q >> 8 (int8) and q & 255 (uint8), [M, K] each, written alongside q.
cudaError_t launch_quantize_rows(const float *x, int16_t *q, float *s, int M, int K, int g,
                                 cudaStream_t stream, int8_t *hi = nullptr, uint8_t *lo = nullptr);

__device__ __forceinline__ float inv127() { return __int_as_float(0x3c010204); }  // (float)1/127

// Sum of squares of one group in the reference order; valid in lane t16 == 0
// of the half-warp, broadcast to all 16.
// The reference's reduction of the 16 lane sums of a group (lane order of
// _mm256 pairs, then (u0+u1)+(u2+u3)); the result is broadcast to all 16.
__device__ __forceinline__ float group_reduce16_ref(float acc) {
    const unsigned full = 0xffffffffu;
    float o = __shfl_down_sync(full, acc, 8, 16);
    float v = add_rn(acc, o);                     // lane l<8: v_l = a0_l + a1_l
    o = __shfl_down_sync(full, v, 4, 16);
    float u = add_rn(v, o);                       // l<4: u_l = v_l + v_{l+4}
    o = __shfl_down_sync(full, u, 1, 16);
    float p = add_rn(u, o);                       // l=0: u0+u1 ; l=2: u2+u3
    o = __shfl_down_sync(full, p, 2, 16);
    float r = add_rn(p, o);                       // l=0: (u0+u1)+(u2+u3)
    return __shfl_sync(full, r, 0, 16);
}

__device__ __forceinline__ float group_sumsq_ref(const float *xg, int g, int t16) {
    float acc = 0.0f;
    // values of a batch are loaded ahead of the (serial) fma chain
    for (int j0 = 0; j0 < g; j0 += 16 * 16) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = j0 + 16 * k < g ? xg[j0 + 16 * k + t16] : 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (j0 + 16 * k < g) acc = fma_rn(v[k], v[k], acc);
    }
    return group_reduce16_ref(acc);
}

__device__ __forceinline__ int16_t quant_one(float x, float inv) {
    float p = mul_rn(x, inv);
    int r;
    if (!(p > -2147483648.0f && p < 2147483648.0f)) r = INT32_MIN;  // cvtps_epi32 overflow/NaN
    else r = __float2int_rn(p);
    r = max(-32768, min(32767, r));                                  // packs_epi32
    return (int16_t)r;
}

// Quantise group `gi` of row x (length g) into q/s; called by one half-warp.
__device__ __forceinline__ void quantize_group(const float *xg, int16_t *qg, float *sg,
                                               int g, int t16, bool write = true) {
    float ss = group_sumsq_ref(xg, g, t16);
    float inv_g = __fdiv_rn(1.0f, (float)g);
    float rms = __fsqrt_rn(fma_rn(ss, inv_g, 1e-6f));
    float s = mul_rn(rms, inv127());
    if (write && t16 == 0) *sg = s;
    float inv = __fdiv_rn(1.0f, s);
    if (write)
        for (int j = t16; j < g; j += 16) qg[j] = quant_one(xg[j], inv);
}


// Scale of one group: s = sqrtf(sum(x^2) * (1/g) + 1e-6) * (1/127), the sum in
// the reference order (group_sumsq_ref).  Called by a whole half-warp.
__device__ __forceinline__ float group_scale_ref(const float *xg, int g, int t16) {
    float ss = group_sumsq_ref(xg, g, t16);
    float inv_g = __fdiv_rn(1.0f, (float)g);
    return mul_rn(__fsqrt_rn(fma_rn(ss, inv_g, 1e-6f)), inv127());
}

// Scales and quantisation of a block's slice xs[0, ng * g) of one row, held in
// shared memory (ng <= 16 groups, block of 256 threads): half-warp h < ng runs
// group h's scale chain -- warps with no live group skip it -- then all
// threads quantise four elements at a time.  s, q, hi, lo point at the
// slice's first scale / element; hi and lo may be null.
__device__ __forceinline__ void quantize_slice(const float *xs, int g, int ng, int16_t *q, float *s,
                                               int8_t *hi, uint8_t *lo, float *inv_s) {
    const int hw = threadIdx.x >> 4;
    if ((threadIdx.x >> 5) * 2 < ng) {
        const int gl = hw < ng ? hw : 0;   // a dead half of a live warp repeats group 0 (shuffle partners)
        const float sc = group_scale_ref(xs + (size_t)gl * g, g, threadIdx.x & 15);
        if (hw < ng && (threadIdx.x & 15) == 0) {
            s[gl] = sc;
            inv_s[gl] = __fdiv_rn(1.0f, sc);
        }
    }
    __syncthreads();
    const int n4 = ng * g / 4;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(xs)[i];
        const float inv = inv_s[ng == 1 ? 0 : (4 * i) / g];
        const uint32_t a = (uint16_t)quant_one(v.x, inv), b = (uint16_t)quant_one(v.y, inv);
        const uint32_t c = (uint16_t)quant_one(v.z, inv), d = (uint16_t)quant_one(v.w, inv);
        reinterpret_cast<uint2 *>(q)[i] = make_uint2(a | (b << 16), c | (d << 16));
        if (hi) {
            reinterpret_cast<uint32_t *>(hi)[i] = (a >> 8) | ((b >> 8) << 8) | ((c >> 8) << 16) | ((d >> 8) << 24);
            reinterpret_cast<uint32_t *>(lo)[i] = (a & 255u) | ((b & 255u) << 8) | ((c & 255u) << 16) | (d << 24);
        }
    }
}

}  // namespace qvl
