// CTA-wide row operations shared by the standalone kernels and the fused
// GEMV tails: RMSNorm with an INT8 group-quantised weight (+ quantisation of
// the result) and plain activation quantisation, with the reference's
// arithmetic (see norm.cu and qact.cu for the citations).  Every function is
// called by all threads of a CTA and synchronises it.
#pragma once
#include "common.cuh"
#include "qact.cuh"

namespace qvl {

// Sum of squares of xs[0..H) in the reference's rms_norm order (8 lanes,
// multiply and add rounded separately, lanes added in order); valid in every
// lane of warp 0.
__device__ __forceinline__ float rms_sumsq_ref(const float *xs, int H) {
    const int l = threadIdx.x & 7;
    float acc = 0.0f;
    // squares of a batch are loaded and formed ahead of the (serial) sum
    for (int i0 = 0; i0 < H; i0 += 8 * 32) {
        float sq[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            const int i = i0 + 8 * k;
            const float v = i < H ? xs[i + l] : 0.0f;
            sq[k] = mul_rn(v, v);
        }
#pragma unroll
        for (int k = 0; k < 32; ++k)
            if (i0 + 8 * k < H) acc = add_rn(acc, sq[k]);
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = add_rn(ss, __shfl_sync(0xffffffffu, acc, k));
    return ss;
}

__device__ __forceinline__ float rms_inv(float ss, int H, float eps, bool inplace_form) {
    const float inv_hs = __fdiv_rn(1.0f, (float)H);
    const float a = fma_rn(ss, inv_hs, eps);
    const float r = __fsqrt_rn(a);
    return inplace_form ? __fdiv_rn(1.0f, r) : __double2float_rn(1.0 / (double)r);
}

// Group scales of ts[0..H) (group g, G = H/g <= 64) and quantisation into q
// (and, when hi is given, the tensor-core planes hi = q >> 8, lo = q & 255).
// scratch: >= 64 floats of shared memory.
__device__ __forceinline__ void cta_quantize_smem_row(const float *ts, int H, int g, int16_t *q, float *qs,
                                                      float *scratch, int8_t *hi = nullptr,
                                                      uint8_t *lo = nullptr) {
    const int G = H / g;
    const int hw = threadIdx.x >> 4, nhw = blockDim.x >> 4, t16 = threadIdx.x & 15;
    // both half-warps of a warp take the same trip count (full-mask shuffles)
    for (int e0 = hw & ~1; e0 < G; e0 += nhw) {
        const int e_raw = e0 + (hw & 1);
        const bool active = e_raw < G;
        const int e = active ? e_raw : e0;
        const float s = group_scale_ref(ts + (size_t)e * g, g, t16);
        if (active && t16 == 0) {
            qs[e] = s;
            scratch[e] = __fdiv_rn(1.0f, s);
        }
    }
    __syncthreads();
    if (hi) {
        for (int j4 = threadIdx.x; j4 < H / 4; j4 += blockDim.x) {
            const float4 v = reinterpret_cast<const float4 *>(ts)[j4];
            const float inv = scratch[(4 * j4) / g];
            const uint32_t a = (uint16_t)quant_one(v.x, inv), b = (uint16_t)quant_one(v.y, inv);
            const uint32_t c = (uint16_t)quant_one(v.z, inv), d = (uint16_t)quant_one(v.w, inv);
            reinterpret_cast<uint2 *>(q)[j4] = make_uint2(a | (b << 16), c | (d << 16));
            reinterpret_cast<uint32_t *>(hi)[j4] = (a >> 8) | ((b >> 8) << 8) | ((c >> 8) << 16) | ((d >> 8) << 24);
            reinterpret_cast<uint32_t *>(lo)[j4] = (a & 255u) | ((b & 255u) << 8) | ((c & 255u) << 16) | (d << 24);
        }
    } else {
        for (int j = threadIdx.x; j < H; j += blockDim.x) q[j] = quant_one(ts[j], scratch[j / g]);
    }
    __syncthreads();
}

// One row: optional RMSNorm (wq != nullptr), then optional quantisation
// (q != nullptr).  xs/ts: shared memory of H floats each; scratch >= 65 floats.
// Reads x with L2-coherent loads (it may have been written by other CTAs).
// wqf/wsg (optional): the norm weight already staged in shared memory as
// floats ((float)wq[j], and ws[g]), read instead of wq/ws.
__device__ __forceinline__ void cta_norm_quant_row(const float *x, const int8_t *wq, const float *ws, int ngs,
                                                   float eps, bool inplace_form, float *out, int16_t *q,
                                                   float *qs, int qg, int H, float *xs, float *ts,
                                                   float *scratch, int8_t *hi = nullptr, uint8_t *lo = nullptr,
                                                   const float *wqf = nullptr, const float *wsg = nullptr) {
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(x) + i);
    __syncthreads();
    const float *src = xs;
    if (wq) {
        if (threadIdx.x < 32) {
            const float ss = rms_sumsq_ref(xs, H);
            if (threadIdx.x == 0) scratch[64] = rms_inv(ss, H, eps, inplace_form);
        }
        __syncthreads();
        const float inv = scratch[64];
        for (int j = threadIdx.x; j < H; j += blockDim.x) {
            const float w = wqf ? wqf[j] : (float)wq[j];
            const float g = wsg ? wsg[j / ngs] : ws[j / ngs];
            const float t = mul_rn(w, mul_rn(mul_rn(g, inv), xs[j]));
            ts[j] = t;
            if (out) out[j] = t;
        }
        __syncthreads();
        src = ts;
    }
    if (q) cta_quantize_smem_row(src, H, qg, q, qs, scratch, hi, lo);
}

// Fused tail of a producer kernel: the last CTA of the grid to finish runs
// cta_norm_quant_row over `rows` rows of x.  `counter` is a device int that
// is zero before the launch; the last CTA sets it back to zero.
struct RowTail {
    int *counter;              // nullptr: no tail
    const float *x;            // [rows, H]
    const int8_t *wq;          // norm weight (nullptr: quantise only)
    const float *ws;
    int ngs;
    float eps;
    int inplace_form;
    float *out;                // [rows, H] normalised copy (nullable; may alias x)
    int16_t *q;                // [rows, H]
    float *qs;                 // [rows, H / qg]
    int qg;
    int H;
    int rows;
    int participants;          // CTAs that call run_row_tail (0: the whole grid)
};

// Bytes of dynamic shared memory the tail needs (the normalised row needs a
// second buffer only when there is a norm).
__host__ __device__ inline size_t row_tail_smem(int H, bool norm) { return (size_t)(norm ? 2 : 1) * H * sizeof(float); }

// Called by all threads of every CTA at the very end of the producer kernel.
// smem: >= row_tail_smem(H) bytes, free for reuse at this point.
__device__ __forceinline__ void run_row_tail(const RowTail &t, unsigned char *smem) {
    __shared__ int is_last;
    __shared__ float scratch[65];
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();   // this CTA's outputs are visible before it is counted
        const unsigned total = t.participants > 0 ? (unsigned)t.participants : gridDim.x * gridDim.y * gridDim.z;
        is_last = (atomicAdd(t.counter, 1) == (int)total - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float *xs = reinterpret_cast<float *>(smem);
    float *ts = xs + t.H;
    for (int r = 0; r < t.rows; ++r)
        cta_norm_quant_row(t.x + (size_t)r * t.H, t.wq, t.ws, t.ngs, t.eps, t.inplace_form != 0,
                           t.out ? t.out + (size_t)r * t.H : nullptr, t.q + (size_t)r * t.H,
                           t.qs + (size_t)r * (t.H / t.qg), t.qg, t.H, xs, ts, scratch);
    if (threadIdx.x == 0) *t.counter = 0;
}

}  // namespace qvl
