// GQA attention over a paged FP16 KV cache (decode and causal prefill).
//
// Reference path (per token, per layer): apply_rotary on q, apply_rotary_cache
// on k writing the cache row, memcpy of v into the cache
// (layers/src/text_layer.cpp:712-824, model/src/forward.cpp:545-562), then
// attn_scores_all_heads -> softmax -> attn_weighted_sum_all_heads
// (layers/src/text_layer.cpp:436-710).
//
// The reference softmax is two-pass (max first, then exp), evaluated with its
// own polynomial exp (exp256_ps) and a double-precision sum.  To keep those
// semantics -- including the polynomial's error and its "all-zero row" rules
// -- without a second read of K, the GPU path is split-K over the context
// with the raw scores kept in a small fp32 scratch (4 bytes per token per
// head, 1/64 of the K+V bytes it replaces re-reading):
//   1. scores:  s[t] = (q . k_t) / sqrt(D) for a chunk of tokens, chunk max
//   2. pv:      global max from the chunk maxima, p_t = exp_ref(s_t - max),
//               chunk partial sum and partial sum_t p_t v_t
//   3. combine: sum over chunks (double), out = acc / sum
// Each K and V byte is read exactly once with 16-byte loads: a token row
// (D = 128 halves = 256 B) is covered by 16 threads.
#include <cuda_fp16.h>
#include <cfloat>
#include "common.cuh"
#include "attention.cuh"
#include "tail.cuh"
#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace qvl {

namespace {
constexpr int kD = 128;
constexpr int kAttnThreads = 128;
constexpr int kMaxChunk = 256;

struct Dims {
    int NH, NKV, P, maxp, max_pos;
};

__device__ __forceinline__ const uint4 *kv_row(const uint16_t *pages, const int32_t *pt_row, int t,
                                               int kvh, const Dims &d) {
    const int page = pt_row[t / d.P];
    const int slot = t - (t / d.P) * d.P;
    const size_t off = (((size_t)page * d.NKV + kvh) * d.P + slot) * kD;
    return reinterpret_cast<const uint4 *>(pages + off);
}

__device__ __forceinline__ void h8_to_f8(const uint4 &v, float f[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 x = __half22float2(h[i]);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
    }
}
}  // namespace

// ---------------------------------------------------------------- RoPE + append
// grid: nq; block 256; dynamic smem (NH + NKV) * D floats.
// Optional QK-norm first (rms_norm_inplace with the per-layer INT8 q_norm /
// k_norm weights, model/src/forward.cpp:531-538, arithmetic of
// layers/src/text_layer.cpp:234-272), then RoPE on pairs (i, i + D/2):
// y1 = x1*c - (x2*s) fused, y2 = x1*s + (x2*c) fused, exactly as
// apply_rotary's fmsub/fmadd.  q is rotated in place; k (rotated) and v are
// rounded to fp16 and written at the query's position.
__global__ void rope_append_kernel(float *__restrict q, const float *__restrict k_new,
                                   const float *__restrict v_new, uint16_t *__restrict k_pages,
                                   uint16_t *__restrict v_pages, const int32_t *__restrict page_table,
                                   const int32_t *__restrict seq_ids, const int32_t *__restrict positions,
                                   const float *__restrict rope_cos, const float *__restrict rope_sin,
                                   QkNorm nrm, Dims d) {
    extern __shared__ __align__(16) float hs[];
    __shared__ float red[64 * 8];
    __shared__ float invh[64];
    // constant operands first (QK-norm weights): into L2 before the wait
    if (nrm.q_w && threadIdx.x < 4) {
        const void *p[4] = {nrm.q_w, nrm.q_s, nrm.k_w, nrm.k_s};
        prefetch_l2(p[threadIdx.x]);
    }
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x;
    const int pos = positions[i];
    if (pos < 0 || pos >= d.max_pos) return;
    constexpr int half = kD / 2;
    const bool has_k = k_new != nullptr;
    const int nh = d.NH + (has_k ? d.NKV : 0);
    float *qi = q + (size_t)i * d.NH * kD;
    const float *ki = has_k ? k_new + (size_t)i * d.NKV * kD : nullptr;
    for (int e = threadIdx.x; e < nh * kD; e += blockDim.x)
        hs[e] = (e < d.NH * kD) ? qi[e] : ki[e - d.NH * kD];
    __syncthreads();
    if (nrm.q_w) {
        for (int t = threadIdx.x; t < nh * 8; t += blockDim.x) {
            const int h = t >> 3, l = t & 7;
            const float *xh = hs + h * kD;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < kD; j += 8) acc = add_rn(acc, mul_rn(xh[j + l], xh[j + l]));
            red[t] = acc;
        }
        __syncthreads();
        for (int h = threadIdx.x; h < nh; h += blockDim.x) {
            float ss = 0.0f;
#pragma unroll
            for (int l = 0; l < 8; ++l) ss = add_rn(ss, red[h * 8 + l]);
            const float a = fma_rn(ss, __fdiv_rn(1.0f, (float)kD), nrm.eps);
            invh[h] = __fdiv_rn(1.0f, __fsqrt_rn(a));
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nh * kD; e += blockDim.x) {
            const int h = e / kD, j = e - h * kD;
            const bool isq = h < d.NH;
            const int8_t *w = isq ? nrm.q_w : nrm.k_w;
            const float *ws = isq ? nrm.q_s : nrm.k_s;
            hs[e] = mul_rn((float)w[j], mul_rn(mul_rn(ws[j / nrm.gs], invh[h]), hs[e]));
        }
        __syncthreads();
    }
    const float *c = rope_cos + (size_t)pos * half;
    const float *s = rope_sin + (size_t)pos * half;
    for (int e = threadIdx.x; e < d.NH * half; e += blockDim.x) {
        const int h = e / half, j = e - h * half;
        const float *x = hs + h * kD;
        const float x1 = x[j], x2 = x[j + half];
        qi[h * kD + j] = fma_rn(x1, c[j], -mul_rn(x2, s[j]));
        qi[h * kD + j + half] = fma_rn(x1, s[j], mul_rn(x2, c[j]));
    }
    if (!has_k) return;
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * d.maxp;
    const int page = pt_row[pos / d.P];
    const int slot = pos % d.P;
    const float *vi = v_new + (size_t)i * d.NKV * kD;
    for (int e = threadIdx.x; e < d.NKV * half; e += blockDim.x) {
        const int h = e / half, j = e - h * half;
        const float *x = hs + (d.NH + h) * kD;
        const float x1 = x[j], x2 = x[j + half];
        const float y1 = fma_rn(x1, c[j], -mul_rn(x2, s[j]));
        const float y2 = fma_rn(x1, s[j], mul_rn(x2, c[j]));
        const size_t off = (((size_t)page * d.NKV + h) * d.P + slot) * kD;
        k_pages[off + j] = __half_as_ushort(__float2half_rn(y1));
        k_pages[off + j + half] = __half_as_ushort(__float2half_rn(y2));
    }
    for (int e = threadIdx.x; e < d.NKV * kD; e += blockDim.x) {
        const int h = e / kD, j = e - h * kD;
        const size_t off = (((size_t)page * d.NKV + h) * d.P + slot) * kD;
        v_pages[off + j] = __half_as_ushort(__float2half_rn(vi[(size_t)h * kD + j]));
    }
}

// ---------------------------------------------------------------- scores
// grid: (nq, NKV, nchunk); block 128 = 8 half-warps.  Half-warp w takes tokens
// chunk_start + w + 8j; thread t16 covers dims 8*t16..8*t16+7 with one
// 16-byte load.  KVM = NH / NKV query heads share each K row.
// Scratch: scores [nq, NH, ctx_pad], cmax [nq, NH, nchunk].
template <int KVM>
__global__ void __launch_bounds__(kAttnThreads)
attn_scores_kernel(const float *__restrict q, const uint16_t *__restrict k_pages,
                   const int32_t *__restrict page_table, const int32_t *__restrict seq_ids,
                   const int32_t *__restrict positions, int max_ctx, int chunk, int nchunk,
                   float *__restrict scores, float *__restrict cmax, Dims d) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x, kvh = blockIdx.y, c = blockIdx.z;
    const int ctx = min(positions[i] + 1, max_ctx);
    const int t0 = c * chunk;
    if (t0 >= ctx) return;
    const int t1 = min(t0 + chunk, ctx);
    const int t16 = threadIdx.x & 15, hw = threadIdx.x >> 4;
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * d.maxp;
    const int ctx_pad = nchunk * chunk;

    float qv[KVM][8];
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        const float4 *qp = reinterpret_cast<const float4 *>(q + ((size_t)i * d.NH + kvh * KVM + h) * kD + t16 * 8);
        float4 a = qp[0], b = qp[1];
        qv[h][0] = a.x; qv[h][1] = a.y; qv[h][2] = a.z; qv[h][3] = a.w;
        qv[h][4] = b.x; qv[h][5] = b.y; qv[h][6] = b.z; qv[h][7] = b.w;
    }
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)kD));
    float mx[KVM];
#pragma unroll
    for (int h = 0; h < KVM; ++h) mx[h] = -INFINITY;

    // Half-warps of one warp may run different trip counts: shuffle within the
    // own half only.
    const unsigned hmask = 0xffffu << (threadIdx.x & 16);
    constexpr int U = 4;
    for (int tb = t0 + hw; tb < t1; tb += 8 * U) {
        uint4 kr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) kr[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 8 * u;
            if (t < t1) kr[u] = ld_stream_v4(kv_row(k_pages, pt_row, t, kvh, d) + t16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 8 * u;
            float kf[8];
            h8_to_f8(kr[u], kf);
#pragma unroll
            for (int h = 0; h < KVM; ++h) {
                float acc = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc = fma_rn(qv[h][e], kf[e], acc);
#pragma unroll
                for (int o = 8; o >= 1; o >>= 1) acc += __shfl_xor_sync(hmask, acc, o, 16);
                const float sc = mul_rn(acc, inv_sqrt_d);
                if (t < t1) {
                    mx[h] = fmaxf(mx[h], sc);
                    if (t16 == 0) scores[((size_t)i * d.NH + kvh * KVM + h) * ctx_pad + t] = sc;
                }
            }
        }
    }
    __shared__ float red[KVM][kAttnThreads / 32];
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        float m = mx[h];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31) == 0) red[h][threadIdx.x >> 5] = m;
    }
    __syncthreads();
    if (threadIdx.x < KVM) {
        float m = red[threadIdx.x][0];
        for (int w = 1; w < kAttnThreads / 32; ++w) m = fmaxf(m, red[threadIdx.x][w]);
        cmax[((size_t)i * d.NH + kvh * KVM + threadIdx.x) * nchunk + c] = m;
    }
}

// ---------------------------------------------------------------- p . V
// grid: (nq, NKV, nchunk); block 128.  p_t = exp_ref(s_t - max) for the KVM
// heads of this KV head (masked -inf scores give 0, text_layer.cpp:481-488);
// thread (tl = tid/16, dg = tid%16) accumulates dims 8*dg..8*dg+7 over tokens
// t = tl + 8j of the chunk.
// Scratch out: psum [nq, NH, nchunk], pacc [nq, NH, nchunk, D].
template <int KVM>
__global__ void __launch_bounds__(kAttnThreads)
attn_pv_kernel(const uint16_t *__restrict v_pages, const int32_t *__restrict page_table,
               const int32_t *__restrict seq_ids, const int32_t *__restrict positions, int max_ctx,
               int chunk, int nchunk, const float *__restrict scores, const float *__restrict cmax,
               float *__restrict psum, float *__restrict pacc, Dims d) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x, kvh = blockIdx.y, c = blockIdx.z;
    const int ctx = min(positions[i] + 1, max_ctx);
    const int t0 = c * chunk;
    if (t0 >= ctx) return;
    const int len = min(chunk, ctx - t0);
    const int nch_q = (ctx + chunk - 1) / chunk;
    const int ctx_pad = nchunk * chunk;
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * d.maxp;

    __shared__ float p_s[KVM][kMaxChunk];
    __shared__ float gmax[KVM];
    __shared__ float red[KVM][kAttnThreads / 32];
    __shared__ float acc_s[8][KVM][kD + 4];

    // global max over this query's chunk maxima
    if (threadIdx.x < 32) {
#pragma unroll
        for (int h = 0; h < KVM; ++h) {
            const float *cm = cmax + ((size_t)i * d.NH + kvh * KVM + h) * nchunk;
            float m = -INFINITY;
            for (int j = threadIdx.x; j < nch_q; j += 32) m = fmaxf(m, cm[j]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (threadIdx.x == 0) gmax[h] = m;
        }
    }
    __syncthreads();
    // probabilities of this chunk (unnormalised) and their partial sum
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        const float M = gmax[h];
        const float *sp = scores + ((size_t)i * d.NH + kvh * KVM + h) * ctx_pad + t0;
        float part = 0.0f;
        for (int t = threadIdx.x; t < len; t += kAttnThreads) {
            const float sv = sp[t];
            const float p = (sv > -INFINITY) ? exp_ref(sv - M) : 0.0f;
            p_s[h][t] = p;
            part += p;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((threadIdx.x & 31) == 0) red[h][threadIdx.x >> 5] = part;
    }
    __syncthreads();
    if (threadIdx.x < KVM) {
        float sum = 0.0f;
        for (int w = 0; w < kAttnThreads / 32; ++w) sum += red[threadIdx.x][w];
        psum[((size_t)i * d.NH + kvh * KVM + threadIdx.x) * nchunk + c] = sum;
    }

    const int dg = threadIdx.x & 15, tl = threadIdx.x >> 4;
    float acc[KVM][8];
#pragma unroll
    for (int h = 0; h < KVM; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[h][e] = 0.0f;
    constexpr int U = 4;
    for (int tb = tl; tb < len; tb += 8 * U) {
        uint4 vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) vr[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 8 * u;
            if (t < len) vr[u] = ld_stream_v4(kv_row(v_pages, pt_row, t0 + t, kvh, d) + dg);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 8 * u;
            if (t < len) {
                float vf[8];
                h8_to_f8(vr[u], vf);
#pragma unroll
                for (int h = 0; h < KVM; ++h) {
                    const float p = p_s[h][t];
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[h][e] = fma_rn(p, vf[e], acc[h][e]);
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < KVM; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc_s[tl][h][dg * 8 + e] = acc[h][e];
    __syncthreads();
    for (int e = threadIdx.x; e < KVM * kD; e += kAttnThreads) {
        const int h = e / kD, dd = e - h * kD;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += acc_s[w][h][dd];
        pacc[(((size_t)i * d.NH + kvh * KVM + h) * nchunk + c) * kD + dd] = s;
    }
}

// ---------------------------------------------------------------- combine
// grid: (nq, NH); block 128 (one thread per dim).  The reference zeroes the
// row when the max is not finite or the sum is not a positive finite number
// (text_layer.cpp:466-469, :514-517); the same rules apply here.
__global__ void __launch_bounds__(kAttnThreads)
attn_combine_kernel(const int32_t *__restrict positions, int max_ctx, int chunk, int nchunk,
                    const float *__restrict cmax, const float *__restrict psum,
                    const float *__restrict pacc, float *__restrict out, Dims d) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x, h = blockIdx.y;
    const int ctx = min(positions[i] + 1, max_ctx);
    const int nch_q = (ctx + chunk - 1) / chunk;
    const size_t base = ((size_t)i * d.NH + h) * nchunk;
    float M = -INFINITY;
    double sum = 0.0;
    for (int j = 0; j < nch_q; ++j) {
        M = fmaxf(M, cmax[base + j]);
        sum += (double)psum[base + j];
    }
    float *o = out + ((size_t)i * d.NH + h) * kD;
    const int dd = threadIdx.x;
    if (ctx <= 0 || !isfinite(M) || !(sum > 0.0) || !isfinite(sum)) {
        o[dd] = 0.0f;
        return;
    }
    const float inv = (float)(1.0 / sum);
    float a = 0.0f;
    for (int j = 0; j < nch_q; ++j) a += pacc[(base + j) * kD + dd];
    o[dd] = mul_rn(a, inv);
}

// ---------------------------------------------------------------- cluster (one launch)
// grid: (kClusterCtas, nq, NKV), cluster (kClusterCtas, 1, 1); block 256.
// The kClusterCtas CTAs of a cluster own one (query, KV head) pair and split
// its context into contiguous slices.  Each CTA keeps its raw scores in shared
// memory; the CTAs exchange slice maxima, then slice sums and partial weighted
// V sums, through distributed shared memory, and rank 0 writes the output.
// The arithmetic is that of the split-K kernels (global max first, reference
// exp polynomial, double-precision sum, zeroing rules) in a single launch
// with no global scratch.
constexpr int kClusterCtas = 8;
constexpr int kSliceMax = 4096;          // tokens per CTA slice
constexpr int kClusterThreads = 256;

template <int KVM>
__global__ void __launch_bounds__(kClusterThreads)
attn_cluster_kernel(const float *__restrict q, const uint16_t *__restrict k_pages,
                    const uint16_t *__restrict v_pages, const int32_t *__restrict page_table,
                    const int32_t *__restrict seq_ids, const int32_t *__restrict positions, int max_ctx,
                    float *__restrict out, Dims d, RowTail tail) {
    extern __shared__ __align__(16) float sp[];          // [KVM][kSliceMax] scores / probabilities
    __shared__ float accs[16][KVM][kD + 4];              // per token-lane partials, then [0] = CTA partial
    __shared__ float redf[KVM][kClusterThreads / 32];
    __shared__ double redd[KVM][kClusterThreads / 32];
    __shared__ float lmax[KVM];
    __shared__ double lsum[KVM];
    __shared__ float gmax[KVM];
    cg::cluster_group cluster = cg::this_cluster();
    pdl_launch_dependents();
    pdl_wait();
    const int rank = (int)cluster.block_rank();
    const int i = blockIdx.y, kvh = blockIdx.z;
    const int ctx = min(positions[i] + 1, max_ctx);
    const int per = (ctx + kClusterCtas - 1) / kClusterCtas;
    const int t0 = min(ctx, rank * per), t1 = min(ctx, t0 + per);
    const int len = t1 - t0;
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * d.maxp;
    const int t16 = threadIdx.x & 15, hw = threadIdx.x >> 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    float qv[KVM][8];
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        const float4 *qp = reinterpret_cast<const float4 *>(q + ((size_t)i * d.NH + kvh * KVM + h) * kD + t16 * 8);
        float4 a = qp[0], b = qp[1];
        qv[h][0] = a.x; qv[h][1] = a.y; qv[h][2] = a.z; qv[h][3] = a.w;
        qv[h][4] = b.x; qv[h][5] = b.y; qv[h][6] = b.z; qv[h][7] = b.w;
    }
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)kD));
    const unsigned hmask = 0xffffu << (threadIdx.x & 16);
    float mx[KVM];
#pragma unroll
    for (int h = 0; h < KVM; ++h) mx[h] = -INFINITY;
    constexpr int U = 4;
    for (int tb = hw; tb < len; tb += 16 * U) {
        uint4 kr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 16 * u;
            kr[u] = (t < len) ? ld_stream_v4(kv_row(k_pages, pt_row, t0 + t, kvh, d) + t16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 16 * u;
            float kf[8];
            h8_to_f8(kr[u], kf);
#pragma unroll
            for (int h = 0; h < KVM; ++h) {
                float acc = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc = fma_rn(qv[h][e], kf[e], acc);
#pragma unroll
                for (int o = 8; o >= 1; o >>= 1) acc += __shfl_xor_sync(hmask, acc, o, 16);
                const float sc = mul_rn(acc, inv_sqrt_d);
                if (t < len) {
                    mx[h] = fmaxf(mx[h], sc);
                    if (t16 == 0) sp[h * kSliceMax + t] = sc;
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        float m = mx[h];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) redf[h][warp] = m;
    }
    __syncthreads();
    if (threadIdx.x < KVM) {
        float m = redf[threadIdx.x][0];
        for (int w = 1; w < kClusterThreads / 32; ++w) m = fmaxf(m, redf[threadIdx.x][w]);
        lmax[threadIdx.x] = m;
    }
    cluster.sync();                                       // slice maxima visible cluster-wide
    if (threadIdx.x < KVM) {
        float m = -INFINITY;
        for (int r = 0; r < kClusterCtas; ++r) m = fmaxf(m, cluster.map_shared_rank(lmax, r)[threadIdx.x]);
        gmax[threadIdx.x] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < KVM; ++h) {
        const float M = gmax[h];
        double part = 0.0;
        for (int t = threadIdx.x; t < len; t += kClusterThreads) {
            const float sv = sp[h * kSliceMax + t];
            const float p = (sv > -INFINITY) ? exp_ref(sv - M) : 0.0f;
            sp[h * kSliceMax + t] = p;
            part += (double)p;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) redd[h][warp] = part;
    }
    __syncthreads();
    if (threadIdx.x < KVM) {
        double sum = 0.0;
        for (int w = 0; w < kClusterThreads / 32; ++w) sum += redd[threadIdx.x][w];
        lsum[threadIdx.x] = sum;
    }
    const int dg = t16, tl = hw;
    float acc[KVM][8];
#pragma unroll
    for (int h = 0; h < KVM; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[h][e] = 0.0f;
    for (int tb = tl; tb < len; tb += 16 * U) {
        uint4 vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 16 * u;
            vr[u] = (t < len) ? ld_stream_v4(kv_row(v_pages, pt_row, t0 + t, kvh, d) + dg) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int t = tb + 16 * u;
            if (t < len) {
                float vf[8];
                h8_to_f8(vr[u], vf);
#pragma unroll
                for (int h = 0; h < KVM; ++h) {
                    const float p = sp[h * kSliceMax + t];
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[h][e] = fma_rn(p, vf[e], acc[h][e]);
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < KVM; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) accs[tl][h][dg * 8 + e] = acc[h][e];
    __syncthreads();
    float cpart[KVM];   // this CTA's partial for (h, dd) handled by this thread
    for (int e = threadIdx.x; e < KVM * kD; e += kClusterThreads) {
        const int h = e / kD, dd = e - h * kD;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < 16; ++w) sum += accs[w][h][dd];
        cpart[h] = sum;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < KVM * kD; e += kClusterThreads) {
        const int h = e / kD, dd = e - h * kD;
        accs[0][h][dd] = cpart[h];
    }
    cluster.sync();                                       // partial sums visible cluster-wide
    if (rank == 0) {
        for (int e = threadIdx.x; e < KVM * kD; e += kClusterThreads) {
            const int h = e / kD, dd = e - h * kD;
            double sum = 0.0;
            float a = 0.0f;
            for (int r = 0; r < kClusterCtas; ++r) {
                sum += cluster.map_shared_rank(lsum, r)[h];
                a += cluster.map_shared_rank(&accs[0][0][0], r)[h * (kD + 4) + dd];
            }
            const float M = gmax[h];
            // the reference zeroes the row when the max is not finite or the
            // sum is not a positive finite number (text_layer.cpp:466-469, :514-517)
            const bool zero = ctx <= 0 || !isfinite(M) || !(sum > 0.0) || !isfinite(sum);
            out[((size_t)i * d.NH + kvh * KVM + h) * kD + dd] = zero ? 0.0f : mul_rn(a, (float)(1.0 / sum));
        }
    }
    cluster.sync();                                       // keep shared memory alive for rank 0's reads
    // Optional fused quantisation of the attention output rows (the o_proj
    // input): the last rank-0 CTA to finish quantises every row.
    if (tail.counter && rank == 0) run_row_tail(tail, reinterpret_cast<unsigned char *>(sp));
}

// ---------------------------------------------------------------- host side
// One cluster per (query, KV head) when every slice fits in shared memory
// and the context is short enough that the cluster's CTAs are not starved,
// or there are enough clusters to fill the GPU; split-K over the context
// (three launches, global scratch) otherwise.
bool attn_use_cluster(size_t nq, int max_ctx, int nkv) {
    if (max_ctx > kClusterCtas * kSliceMax) return false;
    return max_ctx <= 8192 || nq * (size_t)nkv * kClusterCtas >= 2 * 148;
}

int attn_chunk_tokens(size_t nq, int max_ctx, int nkv) {
    int chunk = kMaxChunk;
    while (chunk > 32 && (double)nq * nkv * ((max_ctx + chunk - 1) / chunk) < 2.0 * 148) chunk /= 2;
    return chunk;
}

AttnScratch attn_scratch_layout(size_t nq, int max_ctx, int NH, int nkv) {
    AttnScratch s;
    s.chunk = attn_chunk_tokens(nq, max_ctx, nkv);
    s.nchunk = (max_ctx + s.chunk - 1) / s.chunk;
    const size_t rows = nq * (size_t)NH;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    s.scores_off = 0;
    s.cmax_off = al(rows * (size_t)s.nchunk * s.chunk * 4);
    s.psum_off = s.cmax_off + al(rows * s.nchunk * 4);
    s.pacc_off = s.psum_off + al(rows * s.nchunk * 4);
    s.total = s.pacc_off + al(rows * s.nchunk * (size_t)kD * 4);
    return s;
}

namespace {
template <typename K, typename... Args>
cudaError_t launch_pdl(K kern, dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int KVM>
cudaError_t launch_attn_t(const AttnArgs &a, const AttnScratch &s, char *ws, cudaStream_t st) {
    Dims d{a.NH, a.NKV, a.P, a.maxp, a.max_pos};
    if (attn_use_cluster(a.nq, a.max_ctx, a.NKV)) {
        auto kern = attn_cluster_kernel<KVM>;
        const size_t smem = (size_t)KVM * kSliceMax * sizeof(float);
        // static + dynamic shared memory exceeds the 48 KB default: opt in
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kClusterCtas, (unsigned)a.nq, a.NKV);
        cfg.blockDim = dim3(kClusterThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = kClusterCtas;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        RowTail tail = {};
        if (a.q_out) {
            tail.counter = a.counter; tail.x = a.out; tail.q = a.q_out; tail.qs = a.q_out_scales;
            tail.qg = a.NH * kD; tail.H = a.NH * kD; tail.rows = (int)a.nq;
            tail.participants = (int)a.nq * a.NKV;   // rank-0 CTAs of every cluster
        }
        return cudaLaunchKernelEx(&cfg, kern, a.q, a.k_pages, a.v_pages, a.page_table, a.seq_ids, a.positions,
                                  a.max_ctx, a.out, d, tail);
    }
    float *scores = reinterpret_cast<float *>(ws + s.scores_off);
    float *cmax = reinterpret_cast<float *>(ws + s.cmax_off);
    float *psum = reinterpret_cast<float *>(ws + s.psum_off);
    float *pacc = reinterpret_cast<float *>(ws + s.pacc_off);
    dim3 g3((unsigned)a.nq, a.NKV, s.nchunk);
    cudaError_t e = launch_pdl(attn_scores_kernel<KVM>, g3, dim3(kAttnThreads), st, a.q, a.k_pages,
                               a.page_table, a.seq_ids, a.positions, a.max_ctx, s.chunk, s.nchunk,
                               scores, cmax, d);
    if (e != cudaSuccess) return e;
    e = launch_pdl(attn_pv_kernel<KVM>, g3, dim3(kAttnThreads), st, a.v_pages, a.page_table, a.seq_ids,
                   a.positions, a.max_ctx, s.chunk, s.nchunk, (const float *)scores,
                   (const float *)cmax, psum, pacc, d);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_combine_kernel, dim3((unsigned)a.nq, a.NH), dim3(kD), st, a.positions,
                      a.max_ctx, s.chunk, s.nchunk, (const float *)cmax, (const float *)psum,
                      (const float *)pacc, a.out, d);
}
}  // namespace

cudaError_t launch_attention(const AttnArgs &a, void *workspace, cudaStream_t stream) {
    AttnScratch s = attn_scratch_layout(a.nq, a.max_ctx, a.NH, a.NKV);
    char *ws = static_cast<char *>(workspace);
    switch (a.NH / a.NKV) {
        case 1: return launch_attn_t<1>(a, s, ws, stream);
        case 2: return launch_attn_t<2>(a, s, ws, stream);
        case 4: return launch_attn_t<4>(a, s, ws, stream);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_rope_append(const RopeArgs &a, cudaStream_t stream) {
    Dims d{a.NH, a.NKV, a.P, a.maxp, a.max_pos};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.nq);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t)(a.NH + a.NKV) * kD * sizeof(float);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rope_append_kernel, a.q, a.k_new, a.v_new, a.k_pages, a.v_pages,
                              a.page_table, a.seq_ids, a.positions, a.rope_cos, a.rope_sin, a.norm, d);
}

}  // namespace qvl
