/* Test infrastructure only -- see oracle.h.  A scalar restatement of the
 * reference's CPU arithmetic, operation by operation, with every fused
 * multiply-add the reference's AVX2/FMA code performs written as fmaf()
 * (this file is compiled with -ffp-contract=off so nothing else fuses). */
#include "oracle.h"
#include <math.h>
#include <float.h>
#include <string.h>

/* Horizontal sum of an 8-lane fp32 vector in the order of add_reduce_mm_256
 * (matmul/include/simd_utils.hpp:5-19, layers/include/simd_utils.hpp:148):
 * u_i = v_i + v_{i+4}; then two hadd steps -> (u0+u1)+(u2+u3). */
static float reduce8(const float v[8]) {
    float u0 = v[0] + v[4], u1 = v[1] + v[5], u2 = v[2] + v[6], u3 = v[3] + v[7];
    return (u0 + u1) + (u2 + u3);
}

/* Activation quantization, matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:135-177.
 * Per group of g values: two 8-lane fma accumulators of x^2 (elements
 * kk+16j+l and kk+16j+8+l), summed lane-wise, reduced by reduce8;
 * s = sqrtf(ss * (1/g) + 1e-6) / 127 (the compiler fuses the multiply-add);
 * q = saturate_int16(round_half_even(x * (1/s))). */
void orc_quantize_row(const float *x, size_t K, size_t g, int16_t *q, float *s) {
    const float inv_g = 1.0f / (float)g;
    const float inv_127 = 1.0f / 127.0f;
    for (size_t kk = 0; kk < K; kk += g) {
        float a0[8] = {0}, a1[8] = {0}, v[8];
        for (size_t k = kk; k < kk + g; k += 16)
            for (int l = 0; l < 8; ++l) {
                a0[l] = fmaf(x[k + l], x[k + l], a0[l]);
                a1[l] = fmaf(x[k + 8 + l], x[k + 8 + l], a1[l]);
            }
        for (int l = 0; l < 8; ++l) v[l] = a0[l] + a1[l];
        float ss = reduce8(v);
        float rms = sqrtf(fmaf(ss, inv_g, 1e-6f));
        float sv = rms * inv_127;
        s[kk / g] = sv;
        float inv = 1.0f / sv;
        for (size_t k = kk; k < kk + g; ++k) {
            float p = x[k] * inv;
            /* cvtps_epi32: round-half-even; NaN/overflow -> INT32_MIN */
            long r;
            if (!(p > -2147483648.0f && p < 2147483648.0f)) r = INT32_MIN;
            else r = (long)nearbyintf(p);
            if (r > 32767) r = 32767;
            if (r < -32768) r = -32768;
            q[k] = (int16_t)r;
        }
    }
}

/* Exact integer dot product of group `gi` of quantized row q with weight
 * row w (the madd_epi16 lanes summed; integer addition is associative). */
static int32_t group_dot(const int16_t *q, const int8_t *w, size_t k0, size_t g) {
    int32_t acc = 0;
    for (size_t k = k0; k < k0 + g; ++k) acc += (int32_t)q[k] * (int32_t)w[k];
    return acc;
}

void orc_group_sums(const int16_t *q, const int8_t *w, int32_t *out,
                    size_t M, size_t N, size_t K, size_t g) {
    const size_t G = K / g;
    for (size_t i = 0; i < M; ++i)
        for (size_t j = 0; j < N; ++j)
            for (size_t gi = 0; gi < G; ++gi)
                out[(i * N + j) * G + gi] = group_dot(q + i * K, w + j * K, gi * g, g);
}

/* M=1 GEMV semantics, cpu_f32a_i8f32sb_f32c_avx2.cpp:181-223 (and the
 * identical arithmetic of the LM-head variant :405-452): per output row, 8
 * int32 lanes per group (lane l holds columns with k mod 16 in {2l, 2l+1});
 * each lane is converted to fp32 and fused into a per-lane fp32 accumulator
 * with the scale a_s*w_s; the 8 lanes are reduced by reduce8. */
static void row_lane8(const int16_t *q, const float *as, const int8_t *w, const float *ws,
                      size_t N, size_t K, size_t g, float *y) {
    const size_t G = K / g;
    for (size_t j = 0; j < N; ++j) {
        const int8_t *wr = w + j * K;
        float cf[8] = {0};
        for (size_t gi = 0; gi < G; ++gi) {
            int32_t c[8] = {0};
            for (size_t k = gi * g; k < gi * g + g; k += 16)
                for (int l = 0; l < 8; ++l)
                    c[l] += (int32_t)q[k + 2 * l] * wr[k + 2 * l] +
                            (int32_t)q[k + 2 * l + 1] * wr[k + 2 * l + 1];
            const float sc = as[gi] * ws[j * G + gi];
            for (int l = 0; l < 8; ++l) cf[l] = fmaf((float)c[l], sc, cf[l]);
        }
        y[j] = reduce8(cf);
    }
}

/* M>1 tiled semantics, cpu_f32a_i8f32sb_f32c_avx2.cpp:538-653: per group the
 * full integer sum is converted to fp32 and accumulated as
 * acc = fma(float(S) * a_s, w_s, acc), groups in ascending order. */
static void row_tiled(const int16_t *q, const float *as, const int8_t *w, const float *ws,
                      size_t N, size_t K, size_t g, float *y) {
    const size_t G = K / g;
    for (size_t j = 0; j < N; ++j) {
        float acc = 0.0f;
        for (size_t gi = 0; gi < G; ++gi) {
            int32_t S = group_dot(q, w + j * K, gi * g, g);
            acc = fmaf((float)S * as[gi], ws[j * G + gi], acc);
        }
        y[j] = acc;
    }
}

void orc_linear_i8(const float *x, const int8_t *w, const float *ws, float *y,
                   size_t M, size_t N, size_t K, size_t g, int mode) {
    int16_t *q = (int16_t *)__builtin_alloca(K * sizeof(int16_t));
    float *as = (float *)__builtin_alloca((K / g) * sizeof(float));
    int lane8 = (mode == ORC_LANE8) ||
                (mode == ORC_DISPATCH && M == 1 && N >= 1024 && K >= 1024);
    for (size_t i = 0; i < M; ++i) {
        orc_quantize_row(x + i * K, K, g, q, as);
        if (lane8) row_lane8(q, as, w, ws, N, K, g, y + i * N);
        else row_tiled(q, as, w, ws, N, K, g, y + i * N);
    }
}

/* layers/src/text_layer.cpp:420-434 */
void orc_swiglu(float *gate, const float *up, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float x = gate[i];
        float silu = x / (1.0f + expf(-x));
        gate[i] = silu * up[i];
    }
}

/* The host C library's expf, elementwise over a buffer: what the reference's
 * swiglu calls (layers/src/text_layer.cpp:430, scalar expf; the object file
 * of text_layer.cpp references the libm symbol expf). */
void orc_expf(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = expf(x[i]);
}

/* exp256_ps, layers/include/simd_utils.hpp:7-47, one lane: clamp to
 * +-88.3762626647949, n = floor(x*log2e), g = x - n*ln2 (fused),
 * y = 1 + g + g^2/2 + g^3/6 + g^4/24 (Horner-free, fused adds),
 * result = y * float_from_bits((n+127) << 23). */
float orc_exp_ref(float x) {
    const float max_x = 88.3762626647949f;
    x = (x < max_x) ? x : max_x;          /* _mm256_min_ps(x, max) */
    x = (x > -max_x) ? x : -max_x;        /* _mm256_max_ps(x, min) */
    const float ln2 = 0.69314718056f, inv_ln2 = 1.44269504089f;
    float fx = floorf(x * inv_ln2);
    int32_t e = (int32_t)fx;
    float g = fmaf(-fx, ln2, x);
    float y = fmaf(g, 1.0f, 1.0f);
    float g2 = g * g;
    y = fmaf(g2, 0.5f, y);
    float g3 = g2 * g;
    y = fmaf(g3, 1.0f / 6.0f, y);
    float g4 = g3 * g;
    y = fmaf(g4, 1.0f / 24.0f, y);
    uint32_t bits = (uint32_t)(e + 127) << 23;
    float p;
    memcpy(&p, &bits, 4);
    return y * p;
}

/* softmax, layers/src/text_layer.cpp:437-535 (AVX2 branch). */
void orc_softmax(float *x, size_t n) {
    if (n == 0) return;
    size_t i = 0;
    float vmax[8];
    for (int l = 0; l < 8; ++l) vmax[l] = -INFINITY;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) vmax[l] = (vmax[l] > x[i + l]) ? vmax[l] : x[i + l];
    float mx = vmax[0];
    for (int l = 1; l < 8; ++l) mx = fmaxf(mx, vmax[l]);
    for (; i < n; ++i) mx = fmaxf(mx, x[i]);
    if (!isfinite(mx)) { memset(x, 0, n * sizeof(float)); return; }
    float vsum[8] = {0};
    i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) {
            float v = x[i + l];
            float e = (v > -INFINITY) ? orc_exp_ref(v - mx) : 0.0f;
            x[i + l] = e;
            vsum[l] += e;
        }
    double sum = 0.0;
    for (int l = 0; l < 8; ++l) sum += vsum[l];
    for (; i < n; ++i) {
        if (x[i] == -INFINITY) { x[i] = 0.0f; continue; }
        x[i] = orc_exp_ref(x[i] - mx);
        sum += x[i];
    }
    if (!(sum > 0.0) || !isfinite(sum)) { memset(x, 0, n * sizeof(float)); return; }
    float inv = (float)(1.0 / sum);
    for (i = 0; i < n; ++i) x[i] *= inv;
}

/* apply_rotary / apply_rotary_cache, layers/src/text_layer.cpp:712-824:
 * y1 = x1*c - (x2*s) (fused), y2 = x1*s + (x2*c) (fused), pairs (i, i+D/2). */
void orc_rope_inplace(float *x, const float *c, const float *s, int n_heads, int D) {
    const int half = D / 2;
    for (int h = 0; h < n_heads; ++h) {
        float *x1 = x + h * D, *x2 = x1 + half;
        for (int i = 0; i < half; ++i) {
            float a = x1[i], b = x2[i];
            x1[i] = fmaf(a, c[i], -(b * s[i]));
            x2[i] = fmaf(a, s[i], b * c[i]);
        }
    }
}

/* attn_scores_all_heads + softmax + attn_weighted_sum_all_heads,
 * layers/src/text_layer.cpp:575-710.  Scores: 8-lane fused dot over
 * head_dim, reduce8, times 1/sqrtf(D).  The reference's 0-7 position tail
 * uses a compiler-vectorised reduction whose order is not pinned; the same
 * 8-lane order is used here (agreement is to fp32 rounding, not bits).
 * Weighted sum: out[d] = fma(att[t], v[t][d], out[d]) for t ascending. */
void orc_attention(const float *key_cache, const float *value_cache, const float *q,
                   float *att, float *out, int NH, int NKV, int D, size_t S, int pos) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    const int kv_mul = NH / NKV;
    for (int h = 0; h < NH; ++h) {
        const float *qh = q + (size_t)h * D;
        const float *kh = key_cache + (size_t)(h / kv_mul) * S * D;
        float *ah = att + (size_t)h * S;
        /* positions [0, 8*(pos/8)): the 8-position unrolled loop (:590-633),
         * 8 fused lanes then add_reduce_mm_256_layer; the 0-7 tail (:636-645):
         * `#pragma omp simd reduction(+:score)` over `score += q*k`, which g++
         * (-std=c++17 -O3 -fopenmp -mavx2 -mfma, no FP contraction in ISO
         * mode) vectorises as 8 lanes of unfused multiply-adds whose partial
         * sums are then added lane 0..7 in order onto the initial 0. */
        const int tail0 = (pos / 8) * 8;
        for (int t = 0; t <= pos; ++t) {
            float l8[8] = {0};
            const float *kt = kh + (size_t)t * D;
            if (t < tail0) {
                for (int i = 0; i < D; i += 8)
                    for (int l = 0; l < 8; ++l) l8[l] = fmaf(qh[i + l], kt[i + l], l8[l]);
                ah[t] = reduce8(l8) * inv_sqrt_d;
            } else {
                for (int i = 0; i < D; i += 8)
                    for (int l = 0; l < 8; ++l) l8[l] = l8[l] + qh[i + l] * kt[i + l];
                float r = l8[0];
                for (int l = 1; l < 8; ++l) r = r + l8[l];
                ah[t] = (0.0f + r) * inv_sqrt_d;
            }
        }
        orc_softmax(ah, (size_t)pos + 1);
    }
    for (int h = 0; h < NH; ++h) {
        const float *vh = value_cache + (size_t)(h / kv_mul) * S * D;
        const float *ah = att + (size_t)h * S;
        for (int d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int t = 0; t <= pos; ++t) acc = fmaf(ah[t], vh[(size_t)t * D + d], acc);
            out[(size_t)h * D + d] = acc;
        }
    }
}

/* greedy_decode, tokenizer/src/utils.cpp:34-44: first index of the maximum
 * (strict >), starting from -FLT_MAX. */
int orc_argmax(const float *x, size_t n) {
    float mv = -FLT_MAX;
    int mi = 0;
    for (size_t i = 0; i < n; ++i)
        if (x[i] > mv) { mv = x[i]; mi = (int)i; }
    return mi;
}

/* Text-position section of qwen_rope_precompute, model/src/load_model.cpp:
 * 428-472: inv_freq[i] = 1/powf(theta, 2i/D); cos/sin of (pos*inv_freq[i]).
 * For text tokens the three M-RoPE sections carry the same position, so the
 * interleave (:450-463) leaves section 0 equal to the plain table. */
void orc_rope_table(float *cos_tab, float *sin_tab, size_t S, int D, float theta) {
    const int half = D / 2;
    for (int i = 0; i < half; ++i) {
        float inv_freq = 1.0f / powf(theta, (2.0f * i) / (float)D);
        for (size_t p = 0; p < S; ++p) {
            float f = (float)p * inv_freq;
            cos_tab[p * half + i] = cosf(f);
            sin_tab[p * half + i] = sinf(f);
        }
    }
}

/* rms_norm / rms_norm_inplace with an INT8 group-quantised weight,
 * layers/src/text_layer.cpp:111-147 and :234-272.  The reference's
 * `#pragma omp simd reduction(+:ss)` compiles (g++ 13, AVX2) to 8 float lanes
 * (lane l: x[8i+l]^2 added in i order, multiply and add rounded separately)
 * whose lanes are then added in lane order; this was pinned against the
 * compiled reference.  inv_rms: out-of-place (float)(1.0 / (double)sqrtf(a)),
 * in place 1.0f / sqrtf(a), a = ss * (1/hidden) + eps (fused).
 * out[j] = (float)wq[j] * ((ws[j/gs] * inv_rms) * x[j]). */
void orc_rms_norm_i8(const float *x, const int8_t *wq, const float *ws, float *out,
                     size_t hidden, size_t gs, float eps, size_t batches, int inplace) {
    const float inv_hs = 1.0f / (float)hidden;
    for (size_t b = 0; b < batches; ++b) {
        const float *xr = x + b * hidden;
        float *o = out + b * hidden;
        float lane[8] = {0};
        for (size_t i = 0; i < hidden; i += 8)
            for (int l = 0; l < 8; ++l) {
                float p = xr[i + l] * xr[i + l];
                lane[l] = lane[l] + p;
            }
        float ss = 0.0f;
        for (int l = 0; l < 8; ++l) ss = ss + lane[l];
        float a = fmaf(ss, inv_hs, eps);
        float inv = inplace ? 1.0f / sqrtf(a) : (float)(1.0 / (double)sqrtf(a));
        for (size_t j = 0; j < hidden; ++j) {
            float comb = ws[j / gs] * inv;
            o[j] = (float)wq[j] * (comb * xr[j]);
        }
    }
}

/* embedding_lookup, layers/src/text_layer.cpp:41-48 (per-row scale). */
void orc_embedding_i8(const int8_t *table, const float *scales, float *out, size_t hidden,
                      size_t token) {
    const int8_t *r = table + token * hidden;
    const float s = scales[token];
    for (size_t i = 0; i < hidden; ++i) out[i] = (float)r[i] * s;
}
