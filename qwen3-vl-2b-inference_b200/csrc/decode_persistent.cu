// One decode token of the whole Qwen3-VL-2B text decoder (28 layers, LM head,
// greedy decode) in ONE persistent, cooperatively launched kernel, for a
// single request with per-output-row INT8 weights.
//
// Why: at batch 1 the step is a chain of small dependent operations (see
// forward_text, model/src/forward.cpp:458-720); as separate launches each
// costs >= 2.3 us of hand-off plus its own latency.  Here every CTA stays
// resident and the phases are separated by a grid-wide barrier.  Small
// row operations (RMSNorm + quantisation, attention combine + quantisation)
// are computed redundantly by every CTA from L2 instead of by one CTA plus a
// barrier; matrix rows are spread over all warps of the grid.
//
// Arithmetic is the multi-kernel path's, operation by operation (M=1 GEMV
// lane order, reference RMSNorm / quantisation / SwiGLU / RoPE / softmax
// rules); only the attention's split of the context (16 slices per KV head)
// changes fp32 summation order there.
//
// Safety: every barrier wait is bounded by the global timer; a timeout sets
// the abort flag, after which every CTA leaves at its next barrier.  The
// launch is cooperative, so all CTAs are co-resident (the launch fails
// instead of deadlocking if they cannot be).
#include <cfloat>
#include <climits>
#include <cuda_fp16.h>
#include "gemv_common.cuh"
#include "tail.cuh"
#include "decode_persistent.cuh"

namespace qvl {

namespace {
constexpr int kPThreads = 512;
constexpr int kPWarps = kPThreads / 32;
constexpr int H = 2048, I = 6144, NH = 16, NKV = 8, D = 128;
constexpr int kSlices = 16;                    // attention context slices per KV head
constexpr int kSliceMax = 512;                 // tokens per slice (context <= 8192)
constexpr unsigned long long kBarrierLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned ld_volatile(const unsigned *p) {
    return *reinterpret_cast<const volatile unsigned *>(p);
}

// Grid barrier with a bounded wait.  Returns false once any CTA has aborted.
__device__ __forceinline__ bool grid_sync(const PersistState &S, unsigned &gen) {
    __syncthreads();
    __shared__ int ok;
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned arrived = atomicAdd(S.bar_count, 1u) + 1u;
        if (arrived == gridDim.x) {
            atomicExch(S.bar_count, 0u);
            __threadfence();
            atomicExch(S.bar_gen, gen + 1u);
        } else {
            unsigned long long t0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            while (ld_volatile(S.bar_gen) == gen) {
                if (ld_volatile(reinterpret_cast<const unsigned *>(S.abort_flag))) break;
                unsigned long long t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t - t0 > kBarrierLimitNs) {
                    atomicExch(S.abort_flag, 1);
                    break;
                }
            }
        }
        __threadfence();
        ok = ld_volatile(reinterpret_cast<const unsigned *>(S.abort_flag)) == 0;
    }
    ++gen;
    __syncthreads();
    return ok;
}

__device__ __forceinline__ void h8f(const uint4 &v, float f[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 x = __half22float2(h[i]);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
    }
}

__device__ __forceinline__ size_t kv_off(const PersistState &S, int layer, int t, int kvh) {
    const int page = S.page_table[t / S.page_size];
    const int slot = t - (t / S.page_size) * S.page_size;
    return (size_t)layer * S.kv_layer_stride + (((size_t)page * NKV + kvh) * S.page_size + slot) * D;
}

// smem layout (bytes): q16 [I] int16 | xs [I] f32 | ts [I] f32 | sp [2][kSliceMax] f32
struct PSmem {
    int16_t *q16;
    float *xs, *ts, *sp;
};

}  // namespace

namespace {

template <int IT>
__device__ __forceinline__ void load_row(const int8_t *__restrict wrow, int lane, uint4 (&w)[IT]) {
#pragma unroll
    for (int it = 0; it < IT; ++it) w[it] = ld_stream_v4(wrow + (size_t)(it * 32 + lane) * 16);
}

// One output row of an M=1 GEMV with per-row weight scale, in the reference's
// 8-lane order (cpu_f32a_i8f32sb_f32c_avx2.cpp:181-223), from weights already
// loaded by load_row.  q_s: the int16 activations in shared memory as int4
// pairs.  Valid in all lanes.
template <int IT>
__device__ __forceinline__ float dot_row(const uint4 (&w)[IT], const int4 *q_s, float a_s, float w_s, int lane) {
    int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int it = 0; it < IT; ++it) {
        const int c = it * 32 + lane;
        madd_chunk(w[it], q_s[2 * c], q_s[2 * c + 1], p);
    }
    const unsigned full = 0xffffffffu;
    bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int send = up ? p[i] : p[i + 4];
        int keep = up ? p[i + 4] : p[i];
        p[i] = keep + __shfl_xor_sync(full, send, 16);
    }
    up = lane & 8;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        int send = up ? p[i] : p[i + 2];
        int keep = up ? p[i + 2] : p[i];
        p[i] = keep + __shfl_xor_sync(full, send, 8);
    }
    up = lane & 4;
    int r = (up ? p[1] : p[0]) + __shfl_xor_sync(full, up ? p[0] : p[1], 4);
    r += __shfl_xor_sync(full, r, 2);
    r += __shfl_xor_sync(full, r, 1);
    const float cf = fma_rn(__int2float_rn(r), mul_rn(a_s, w_s), 0.0f);
    const float u = add_rn(cf, __shfl_xor_sync(full, cf, 16));
    const float pp = add_rn(u, __shfl_xor_sync(full, u, 4));
    return add_rn(pp, __shfl_xor_sync(full, pp, 8));
}

// Rows k = 0 .. count-1 of this warp's share of an M=1 GEMV with K = 512*IT,
// the next row's loads issued before the current row is reduced.
// row(k, &wrow, &ws) selects the weight row; emit(k, out) consumes the
// result (valid in all lanes).
template <int IT, typename RowFn, typename EmitFn>
__device__ __forceinline__ void gemv_rows(int count, const int4 *q_s, float a_s, int lane, RowFn row, EmitFn emit) {
    if (count <= 0) return;
    if constexpr (IT > 4) {            // long rows: no second register set
        for (int k = 0; k < count; ++k) {
            uint4 w[IT];
            const int8_t *wr;
            float ws;
            row(k, wr, ws);
            load_row<IT>(wr, lane, w);
            emit(k, dot_row<IT>(w, q_s, a_s, ws, lane));
        }
        return;
    }
    uint4 w[IT], nx[IT];
    const int8_t *wr;
    float ws, nws = 0.0f;
    row(0, wr, ws);
    load_row<IT>(wr, lane, w);
    for (int k = 0; k < count; ++k) {
        if (k + 1 < count) {
            const int8_t *nwr;
            row(k + 1, nwr, nws);
            load_row<IT>(nwr, lane, nx);
        }
        emit(k, dot_row<IT>(w, q_s, a_s, ws, lane));
#pragma unroll
        for (int i = 0; i < IT; ++i) w[i] = nx[i];
        ws = nws;
    }
}

// Rows first, first + stride, ... below n_rows.
__device__ __forceinline__ int strided_count(int first, int stride, int n_rows) {
    return first < n_rows ? (n_rows - first + stride - 1) / stride : 0;
}

}  // namespace

__global__ void __launch_bounds__(kPThreads, 1)
decode_persistent_kernel(PersistWeights W, PersistState S) {
    extern __shared__ __align__(16) unsigned char smraw[];
    int16_t *q16 = reinterpret_cast<int16_t *>(smraw);
    float *xs = reinterpret_cast<float *>(smraw + (size_t)I * sizeof(int16_t));
    float *ts = xs + I;
    float *sp = ts + I;
    const int4 *q_s = reinterpret_cast<const int4 *>(q16);
    __shared__ float scratch[65];
    __shared__ float a_s_sh;
    __shared__ unsigned gen0;
    __shared__ float head_m[NH], head_inv[NH];
    __shared__ float redf[2][kPWarps];
    __shared__ double redd[2][kPWarps];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = blockIdx.x * kPWarps + warp, nw = gridDim.x * kPWarps;
    const int ng = W.norm_group;
    const float eps = W.eps;
    if (threadIdx.x == 0) gen0 = ld_volatile(S.bar_gen);
    __syncthreads();
    unsigned gen = gen0;
    const int token = S.token[0];
    const int pos = S.pos[0];
    const int ctx = min(pos + 1, S.max_ctx);

    // embedding_lookup (per-row scale) of the input token into the residual stream
    if (blockIdx.x == 0) {
        const int id = (token >= 0 && token < W.vocab) ? token : 0;
        const float sc = W.embed_s[id];
        for (int j = threadIdx.x; j < H; j += kPThreads) S.x[j] = mul_rn((float)W.embed[(size_t)id * H + j], sc);
    }
    if (!grid_sync(S, gen)) return;

    for (int l = 0; l < W.layers; ++l) {
        // ---- input rms_norm + quantisation (every CTA), q/k/v rows over all warps
        cta_norm_quant_row(S.x, W.in_norm + (size_t)l * H, W.in_norm_s + (size_t)l * (H / ng), ng, eps, false,
                           nullptr, q16, &a_s_sh, H, H, xs, ts, scratch);
        gemv_rows<4>(strided_count(gw, nw, NH * D + 2 * NKV * D), q_s, a_s_sh, lane,
            [&](int k, const int8_t *&wr, float &ws) {
                const int n = gw + k * nw;
                if (n < NH * D) {
                    wr = W.wq + ((size_t)l * NH * D + n) * H; ws = __ldg(W.sq + (size_t)l * NH * D + n);
                } else if (n < NH * D + NKV * D) {
                    const int r = n - NH * D;
                    wr = W.wk + ((size_t)l * NKV * D + r) * H; ws = __ldg(W.sk + (size_t)l * NKV * D + r);
                } else {
                    const int r = n - NH * D - NKV * D;
                    wr = W.wv + ((size_t)l * NKV * D + r) * H; ws = __ldg(W.sv + (size_t)l * NKV * D + r);
                }
            },
            [&](int k, float out) { if (lane == 0) S.qkv[gw + k * nw] = out; });
        if (!grid_sync(S, gen)) return;

        // ---- QK rms_norm_inplace + RoPE (q written back; k, v appended as fp16)
        // (a position past the cache is not appended; the host keeps pos < max_ctx)
        if (blockIdx.x < NH + (pos < S.max_ctx ? NKV : 0)) {
            const bool isq = blockIdx.x < NH;
            const int hh = isq ? blockIdx.x : blockIdx.x - NH;
            const float *src = S.qkv + (isq ? hh * D : NH * D + hh * D);
            if (threadIdx.x < D) xs[threadIdx.x] = __ldcg(src + threadIdx.x);
            __syncthreads();
            if (threadIdx.x < 32) {
                const float ss = rms_sumsq_ref(xs, D);
                if (threadIdx.x == 0) scratch[64] = rms_inv(ss, D, eps, true);
            }
            __syncthreads();
            const int8_t *nwq = (isq ? W.q_norm : W.k_norm) + (size_t)l * D;
            const float *nws = (isq ? W.q_norm_s : W.k_norm_s) + (size_t)l * (D / ng);
            if (threadIdx.x < D)
                ts[threadIdx.x] = mul_rn((float)nwq[threadIdx.x],
                                         mul_rn(mul_rn(nws[threadIdx.x / ng], scratch[64]), xs[threadIdx.x]));
            __syncthreads();
            const float *c = S.rope_cos + (size_t)pos * (D / 2);
            const float *s = S.rope_sin + (size_t)pos * (D / 2);
            if (threadIdx.x < D / 2) {
                const int j = threadIdx.x;
                const float x1 = ts[j], x2 = ts[j + D / 2];
                const float y1 = fma_rn(x1, c[j], -mul_rn(x2, s[j]));
                const float y2 = fma_rn(x1, s[j], mul_rn(x2, c[j]));
                if (isq) {
                    S.qkv[hh * D + j] = y1;
                    S.qkv[hh * D + j + D / 2] = y2;
                } else {
                    const size_t off = kv_off(S, l, pos, hh);
                    S.k_pages[off + j] = __half_as_ushort(__float2half_rn(y1));
                    S.k_pages[off + j + D / 2] = __half_as_ushort(__float2half_rn(y2));
                }
            }
            if (!isq && threadIdx.x < D) {
                const size_t off = kv_off(S, l, pos, hh);
                S.v_pages[off + threadIdx.x] =
                    __half_as_ushort(__float2half_rn(__ldcg(S.qkv + NH * D + NKV * D + hh * D + threadIdx.x)));
            }
        }
        if (!grid_sync(S, gen)) return;

        // ---- attention, phase 1: scores of one context slice and its maximum
        const int per = (ctx + kSlices - 1) / kSlices;
        const bool attn_cta = blockIdx.x < NKV * kSlices;
        const int kvh = blockIdx.x / kSlices, sl = blockIdx.x % kSlices;
        const int t0 = min(ctx, sl * per), t1 = min(ctx, t0 + per), len = t1 - t0;
        const int t16 = threadIdx.x & 15, hw = threadIdx.x >> 4;
        if (attn_cta) {
            float qv[2][8];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) qv[h][e] = __ldcg(S.qkv + (kvh * 2 + h) * D + t16 * 8 + e);
            const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
            const unsigned hmask = 0xffffu << (threadIdx.x & 16);
            float mx[2] = {-INFINITY, -INFINITY};
            for (int tb = hw; tb < len; tb += 32 * 4) {
                uint4 kr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    kr[u] = (t < len) ? __ldcg(reinterpret_cast<const uint4 *>(S.k_pages + kv_off(S, l, t0 + t, kvh)) + t16)
                                      : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    float kf[8];
                    h8f(kr[u], kf);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
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
            for (int h = 0; h < 2; ++h) {
                float m = mx[h];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (lane == 0) redf[h][warp] = m;
            }
            __syncthreads();
            if (threadIdx.x < 2) {
                float m = redf[threadIdx.x][0];
                for (int w = 1; w < kPWarps; ++w) m = fmaxf(m, redf[threadIdx.x][w]);
                S.att_lmax[(kvh * 2 + threadIdx.x) * kSlices + sl] = m;
            }
        }
        if (!grid_sync(S, gen)) return;

        // ---- attention, phase 2: probabilities (global max), slice sum, partial P.V
        if (attn_cta) {
            __shared__ float gm[2];
            if (threadIdx.x < 2) {
                float m = -INFINITY;
                for (int s2 = 0; s2 < kSlices; ++s2) m = fmaxf(m, __ldcg(S.att_lmax + (kvh * 2 + threadIdx.x) * kSlices + s2));
                gm[threadIdx.x] = m;
            }
            __syncthreads();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                double part = 0.0;
                for (int t = threadIdx.x; t < len; t += kPThreads) {
                    const float sv = sp[h * kSliceMax + t];
                    const float p = (sv > -INFINITY) ? exp_ref(sv - gm[h]) : 0.0f;
                    sp[h * kSliceMax + t] = p;
                    part += (double)p;
                }
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
                if (lane == 0) redd[h][warp] = part;
            }
            __syncthreads();
            if (threadIdx.x < 2) {
                double sum = 0.0;
                for (int w = 0; w < kPWarps; ++w) sum += redd[threadIdx.x][w];
                S.att_lsum[(kvh * 2 + threadIdx.x) * kSlices + sl] = sum;
            }
            float acc[2][8];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[h][e] = 0.0f;
            for (int tb = hw; tb < len; tb += 32 * 4) {
                uint4 vr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    vr[u] = (t < len) ? __ldcg(reinterpret_cast<const uint4 *>(S.v_pages + kv_off(S, l, t0 + t, kvh)) + t16)
                                      : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    if (t < len) {
                        float vf[8];
                        h8f(vr[u], vf);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float p = sp[h * kSliceMax + t];
#pragma unroll
                            for (int e = 0; e < 8; ++e) acc[h][e] = fma_rn(p, vf[e], acc[h][e]);
                        }
                    }
                }
            }
            float *red = xs;   // [32 token lanes][2][D]
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) red[(hw * 2 + h) * D + t16 * 8 + e] = acc[h][e];
            __syncthreads();
            for (int e = threadIdx.x; e < 2 * D; e += kPThreads) {
                const int h = e / D, dd = e - h * D;
                float s2 = 0.0f;
                for (int w = 0; w < 32; ++w) s2 += red[(w * 2 + h) * D + dd];
                S.att_pacc[((kvh * 2 + h) * kSlices + sl) * D + dd] = s2;
            }
        }
        if (!grid_sync(S, gen)) return;

        // ---- attention combine (every CTA) -> quantisation -> o_proj + residual
        if (threadIdx.x < NH) {
            const int h = threadIdx.x;
            float m = -INFINITY;
            double sum = 0.0;
            for (int s2 = 0; s2 < kSlices; ++s2) {
                m = fmaxf(m, __ldcg(S.att_lmax + h * kSlices + s2));
                sum += __ldcg(S.att_lsum + h * kSlices + s2);
            }
            // the reference zeroes the row when the max is not finite or the
            // sum is not a positive finite number (text_layer.cpp:466-469, :514-517)
            const bool zero = ctx <= 0 || !isfinite(m) || !(sum > 0.0) || !isfinite(sum);
            head_inv[h] = zero ? 0.0f : (float)(1.0 / sum);
            head_m[h] = zero ? 0.0f : 1.0f;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < H; e += kPThreads) {
            const int h = e / D, dd = e - h * D;
            float a = 0.0f;
            for (int s2 = 0; s2 < kSlices; ++s2) a += __ldcg(S.att_pacc + (h * kSlices + s2) * D + dd);
            xs[e] = head_m[h] != 0.0f ? mul_rn(a, head_inv[h]) : 0.0f;
        }
        __syncthreads();
        cta_quantize_smem_row(xs, H, H, q16, &a_s_sh, scratch);
        gemv_rows<4>(strided_count(gw, nw, H), q_s, a_s_sh, lane,
            [&](int k, const int8_t *&wr, float &ws) {
                const int n = gw + k * nw;
                wr = W.wo + ((size_t)l * H + n) * H; ws = __ldg(W.so + (size_t)l * H + n);
            },
            [&](int k, float out) {
                const int n = gw + k * nw;
                if (lane == 0) S.x[n] = add_rn(__ldcg(S.x + n), out);
            });
        if (!grid_sync(S, gen)) return;

        // ---- post-attention rms_norm + quantisation (every CTA), gate/up + SwiGLU
        cta_norm_quant_row(S.x, W.post_norm + (size_t)l * H, W.post_norm_s + (size_t)l * (H / ng), ng, eps, false,
                           nullptr, q16, &a_s_sh, H, H, xs, ts, scratch);
        {
            float gate_v = 0.0f;
            // the warp's k-th row: gate (k even) or up (k odd) row p = gw + (k/2)*nw
            gemv_rows<4>(2 * strided_count(gw, nw, I), q_s, a_s_sh, lane,
                [&](int k, const int8_t *&wr, float &ws) {
                    const int p = gw + (k >> 1) * nw;
                    if ((k & 1) == 0) { wr = W.wg + ((size_t)l * I + p) * H; ws = __ldg(W.sg + (size_t)l * I + p); }
                    else { wr = W.wu + ((size_t)l * I + p) * H; ws = __ldg(W.su + (size_t)l * I + p); }
                },
                [&](int k, float out) {
                    if ((k & 1) == 0) gate_v = out;
                    else if (lane == 0) S.h[gw + (k >> 1) * nw] = swiglu_one(gate_v, out);
                });
        }
        if (!grid_sync(S, gen)) return;

        // ---- quantisation of the SwiGLU row (every CTA), down + residual
        for (int i = threadIdx.x; i < I / 4; i += kPThreads)
            reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(S.h) + i);
        __syncthreads();
        cta_quantize_smem_row(xs, I, I, q16, &a_s_sh, scratch);
        gemv_rows<12>(strided_count(gw, nw, H), q_s, a_s_sh, lane,
            [&](int k, const int8_t *&wr, float &ws) {
                const int n = gw + k * nw;
                wr = W.wd + ((size_t)l * H + n) * I; ws = __ldg(W.sd + (size_t)l * H + n);
            },
            [&](int k, float out) {
                const int n = gw + k * nw;
                if (lane == 0) S.x[n] = add_rn(__ldcg(S.x + n), out);
            });
        if (!grid_sync(S, gen)) return;
    }

    // ---- final rms_norm_inplace + quantisation (every CTA), LM head + greedy
    cta_norm_quant_row(S.x, W.final_norm, W.final_norm_s, ng, eps, true, nullptr, q16, &a_s_sh, H, H, xs, ts,
                       scratch);
    {
        float best_v = -FLT_MAX;
        int best_i = INT_MAX;
        gemv_rows<4>(strided_count(gw, nw, W.vocab), q_s, a_s_sh, lane,
            [&](int k, const int8_t *&wr, float &ws) {
                const int n = gw + k * nw;
                wr = W.embed + (size_t)n * H; ws = __ldg(W.embed_s + n);
            },
            [&](int k, float out) {
                const int n = gw + k * nw;
                if (lane == 0) S.logits[n] = out;
                if (out > best_v) { best_v = out; best_i = n; }   // ascending n: strict > keeps the first
            });
        if (lane == 0) {
            S.warp_best_v[gw] = best_v;
            S.warp_best_i[gw] = best_i;
        }
    }
    if (!grid_sync(S, gen)) return;
    if (blockIdx.x == 0) {
        float v = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = threadIdx.x; w < nw; w += kPThreads) {
            const float v2 = __ldcg(S.warp_best_v + w);
            const int i2 = __ldcg(S.warp_best_i + w);
            if (v2 > v || (v2 == v && i2 < bi)) { v = v2; bi = i2; }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (v2 > v || (v2 == v && i2 < bi)) { v = v2; bi = i2; }
        }
        if (lane == 0) { redf[0][warp] = v; reinterpret_cast<int *>(scratch)[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            float fv = -FLT_MAX;
            int fi = INT_MAX;
            for (int w = 0; w < kPWarps; ++w) {
                const float v2 = redf[0][w];
                const int i2 = reinterpret_cast<int *>(scratch)[w];
                if (v2 > fv || (v2 == fv && i2 < fi)) { fv = v2; fi = i2; }
            }
            S.token[0] = (fi == INT_MAX) ? 0 : fi;
            S.pos[0] = pos + 1;
        }
    }
}

size_t persist_smem_bytes() {
    return (size_t)I * sizeof(int16_t) + 2 * (size_t)I * sizeof(float) + 2 * (size_t)kSliceMax * sizeof(float);
}

int persist_grid_ctas() {
    static int cached[64] = {};                 // per device, computed on first use
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev < 64 && cached[dev] > 0) return cached[dev];
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)persist_smem_bytes()) != cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, kPThreads,
                                                      persist_smem_bytes()) != cudaSuccess)
        return 0;
    // every attention (KV head, slice) pair and QK row needs a CTA of its own
    const int ctas = sms * (per_sm > 1 ? 1 : per_sm);
    if (ctas < NKV * kSlices) return 0;
    if (dev < 64) cached[dev] = ctas;
    return ctas;
}

bool persist_supported(int hidden, int intermediate, int heads, int kv_heads, int head_dim, int max_ctx) {
    return hidden == H && intermediate == I && heads == NH && kv_heads == NKV && head_dim == D && max_ctx >= 1 &&
           max_ctx <= kSlices * kSliceMax;
}

cudaError_t launch_decode_persistent(const PersistWeights &w, const PersistState &s, int ctas, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = persist_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, w, s);
}

}  // namespace qvl
