// GQA decode attention in the reference's own summation order, bit for bit
// (given the same fp16-valued cache): attn_scores_all_heads, softmax and
// attn_weighted_sum_all_heads, layers/src/text_layer.cpp:436-710.
//
//   scores   t < 8*(pos/8): 8 fused lanes over d = l, l+8, ... (:590-633),
//            then add_reduce_mm_256_layer ((v_i + v_{i+4}), two hadds);
//            the 0-7 tail (:636-645): 8 unfused lanes added 0..7 in order
//            (what g++ makes of `#pragma omp simd reduction(+:score)`);
//            times 1/sqrtf(D).
//   softmax  max; for t < 8*(n/8): exp256_ps(s - max), masked where s is
//            -inf, summed into 8 float lanes t-ascending, the lanes added in
//            double 0..7; then the tail, each term added in double; p = e *
//            (float)(1/sum) (:436-535).
//   P.V      out[h][d] = one fma chain over t ascending (:677-689).
//
// Two launches: scores (one thread per token and KV head, every score of the
// KV head's query heads) into a caller workspace, then one CTA per (query,
// head) for the softmax and the 128 P.V chains (one thread per d).  The
// chains are sequential by construction -- this path trades the split
// context of qvl_attention_decode for exact agreement with the reference.
#include <cuda_fp16.h>
#include "common.cuh"
#include "attention_ordered.cuh"

namespace qvl {

namespace {
constexpr int kD = 128;
constexpr int kThreads = 128;

__device__ __forceinline__ size_t kv_index(const int32_t *pt_row, int t, int kvh, int NKV, int P) {
    const int pg = t / P;
    return (((size_t)pt_row[pg] * NKV + kvh) * P + (t - pg * P)) * kD;
}
}  // namespace

// grid (ceil(max_ctx / 128), NKV, nq); block 128; smem kv_mul * 128 floats.
__global__ void __launch_bounds__(kThreads)
attn_ordered_scores_kernel(const float *__restrict q, const uint16_t *__restrict k_pages,
                           const int32_t *__restrict page_table, const int32_t *__restrict seq_ids,
                           const int32_t *__restrict positions, float *__restrict scores, int max_ctx, int NH,
                           int NKV, int P, int maxp) {
    extern __shared__ float qs[];
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.z, kvh = blockIdx.y;
    const int kvm = NH / NKV;
    const int pos = positions[i];
    for (int e = threadIdx.x; e < kvm * kD; e += blockDim.x) qs[e] = q[((size_t)i * NH + kvh * kvm) * kD + e];
    __syncthreads();
    const int t = blockIdx.x * kThreads + threadIdx.x;
    if (pos < 0 || pos >= max_ctx || t > pos) return;
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * maxp;
    const uint4 *kr = reinterpret_cast<const uint4 *>(k_pages + kv_index(pt_row, t, kvh, NKV, P));
    float k[kD];
#pragma unroll
    for (int c = 0; c < kD / 8; ++c) {
        const uint4 v = __ldg(kr + c);
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            k[8 * c + 2 * j] = f.x;
            k[8 * c + 2 * j + 1] = f.y;
        }
    }
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)kD));
    const bool tail = t >= (pos / 8) * 8;
    for (int hh = 0; hh < kvm; ++hh) {
        const float *qh = qs + hh * kD;
        float l8[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) l8[l] = 0.0f;
        float r;
        if (!tail) {
#pragma unroll
            for (int c = 0; c < kD; c += 8)
#pragma unroll
                for (int l = 0; l < 8; ++l) l8[l] = fma_rn(qh[c + l], k[c + l], l8[l]);
            r = reduce8_ref(l8);
        } else {
#pragma unroll
            for (int c = 0; c < kD; c += 8)
#pragma unroll
                for (int l = 0; l < 8; ++l) l8[l] = add_rn(l8[l], mul_rn(qh[c + l], k[c + l]));
            r = l8[0];
#pragma unroll
            for (int l = 1; l < 8; ++l) r = add_rn(r, l8[l]);
            r = add_rn(0.0f, r);
        }
        scores[((size_t)i * NH + kvh * kvm + hh) * max_ctx + t] = mul_rn(r, inv_sqrt_d);
    }
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kSumChunk = 2048;    // exponentials staged per pass of the lane sums
constexpr int kPvChunk = 64;       // V rows staged per P.V step (16 KB), double-buffered

// grid (NH, nq); block 128 (thread = output dimension d).  `scores` rows are
// overwritten with the exponentials.  Everything read sequentially (the lane
// sums, the P.V chains) comes from shared memory: the exponentials in chunks
// of 2048, the V rows in double-buffered chunks of 64 fetched with cp.async.
__global__ void __launch_bounds__(kThreads)
attn_ordered_softmax_pv_kernel(const uint16_t *__restrict v_pages, const int32_t *__restrict page_table,
                               const int32_t *__restrict seq_ids, const int32_t *__restrict positions,
                               float *__restrict scores, float *__restrict out, int max_ctx, int NH, int NKV,
                               int P, int maxp) {
    __shared__ float red[kThreads / 32];
    __shared__ float lane_sum[8];
    __shared__ float inv_sh;
    __shared__ int zero_sh;
    __shared__ __align__(16) float ebuf[kSumChunk];
    __shared__ __align__(16) uint4 vbuf[2][kPvChunk * kD / 8];
    __shared__ float pbuf[2][kPvChunk];
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, i = blockIdx.y, d = threadIdx.x;
    const int pos = positions[i];
    float *o = out + ((size_t)i * NH + h) * kD;
    if (pos < 0 || pos >= max_ctx) return;
    const int n = pos + 1, n8 = (n / 8) * 8;
    float *s = scores + ((size_t)i * NH + h) * max_ctx;
    // 1. maximum (order-free)
    float m = -__int_as_float(0x7f800000);
    for (int t = d; t < n; t += kThreads) m = fmaxf(m, s[t]);
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((d & 31) == 0) red[d >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    if (!isfinite(m)) {          // every score -inf or NaN: the row is zeros
        o[d] = 0.0f;
        return;
    }
    // 2. exponentials in place (-inf scores give 0)
    const float ninf = -__int_as_float(0x7f800000);
    for (int t = d; t < n; t += kThreads) {
        const float x = s[t];
        s[t] = x > ninf ? exp_ref(add_rn(x, -m)) : 0.0f;
    }
    __syncthreads();
    // 3. the sum: 8 float lanes t-ascending, the lanes in double, the tail in double
    float acc8 = 0.0f;
    for (int c0 = 0; c0 < n8; c0 += kSumChunk) {
        const int cn = min(kSumChunk, n8 - c0);
        for (int t = d; t < cn; t += kThreads) ebuf[t] = s[c0 + t];
        __syncthreads();
        if (d < 8)
            for (int k = d; k < cn; k += 8) acc8 = add_rn(acc8, ebuf[k]);
        __syncthreads();
    }
    if (d < 8) lane_sum[d] = acc8;
    __syncthreads();
    if (d == 0) {
        double sum = 0.0;
        for (int l = 0; l < 8; ++l) sum = __dadd_rn(sum, (double)lane_sum[l]);
        for (int t = n8; t < n; ++t) sum = __dadd_rn(sum, (double)s[t]);
        zero_sh = !(sum > 0.0) || !isfinite(sum);
        inv_sh = __double2float_rn(__ddiv_rn(1.0, sum));
    }
    __syncthreads();
    if (zero_sh) {
        o[d] = 0.0f;
        return;
    }
    const float inv = inv_sh;
    // 4. P.V: one fma chain per d over t ascending, V staged by cp.async
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * maxp;
    const int kvh = h / (NH / NKV);
    const int nch = (n + kPvChunk - 1) / kPvChunk;
    auto issue = [&](int c) {
        const int c0 = c * kPvChunk, cn = min(kPvChunk, n - c0);
        uint4 *vb = vbuf[c & 1];
        for (int e = d; e < cn * (kD / 8); e += kThreads) {
            const int r = e / (kD / 8), q = e - r * (kD / 8);
            cp_async16(vb + e, reinterpret_cast<const uint4 *>(v_pages + kv_index(pt_row, c0 + r, kvh, NKV, P)) + q);
        }
        if (d < cn) pbuf[c & 1][d] = mul_rn(s[c0 + d], inv);
        cp_async_commit();
    };
    issue(0);
    float acc = 0.0f;
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            issue(c + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int cn = min(kPvChunk, n - c * kPvChunk);
        const __half *vb = reinterpret_cast<const __half *>(vbuf[c & 1]) + d;
        const float *pb = pbuf[c & 1];
        int k = 0;
        for (; k + 8 <= cn; k += 8) {
            float pv[8], vv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                pv[j] = pb[k + j];
                vv[j] = __half2float(vb[(k + j) * kD]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fma_rn(pv[j], vv[j], acc);
        }
        for (; k < cn; ++k) acc = fma_rn(pb[k], __half2float(vb[k * kD]), acc);
        __syncthreads();
    }
    o[d] = acc;
}

size_t attn_ordered_workspace_bytes(size_t nq, int max_ctx, int NH) {
    return ((nq * (size_t)NH * (size_t)max_ctx * sizeof(float)) + 255) & ~(size_t)255;
}

cudaError_t launch_attention_ordered(const AttnArgs &a, void *workspace, cudaStream_t stream) {
    float *scores = static_cast<float *>(workspace);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = stream;
    cfg.gridDim = dim3((a.max_ctx + kThreads - 1) / kThreads, a.NKV, (unsigned)a.nq);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)(a.NH / a.NKV) * kD * sizeof(float);
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_ordered_scores_kernel, a.q, a.k_pages, a.page_table, a.seq_ids,
                                       a.positions, scores, a.max_ctx, a.NH, a.NKV, a.P, a.maxp);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(a.NH, (unsigned)a.nq);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, attn_ordered_softmax_pv_kernel, a.v_pages, a.page_table, a.seq_ids,
                              a.positions, scores, a.out, a.max_ctx, a.NH, a.NKV, a.P, a.maxp);
}

}  // namespace qvl
