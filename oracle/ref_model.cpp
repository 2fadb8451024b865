// Test infrastructure only (not shipped, not on any product path).
//
// The reference engine's own text decoder, end to end: init_model_weights
// reads a model file in the exporter's .bin layout
// (model/src/load_model.cpp:50-246), init_model_run_state builds the RoPE
// tables with qwen_rope_precompute (:413-490), and forward_text
// (model/src/forward.cpp:458-720) runs one token.  This file adds a C ABI for
// ctypes and two link-time interpositions (-Wl,--wrap), nothing else:
//
//  * linear() with INT8 weights and group_quantized == false routes to the
//    reference's own INT8 kernel with group = K
//    (f32a_i8f32sb_f32c_avx2_kernel, matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:
//    665).  The reference's row-quantised branch (matmul/src/cpu_wrapper.cpp:
//    172-215) reads the exported [N, K] weight as [K, N], and forward_text
//    passes the embedding's group (H) even for the down projection; the
//    interposition gives the intended per-output-row product.
//  * attn_scores_all_heads(), optionally (fp16_kv): before the real function
//    runs, the key and value rows just written at `pos` for that layer are
//    rounded to fp16 values, so that the cache holds what an FP16 cache holds
//    (the reference keeps FP32, load_model.cpp:348-349; the B200 path keeps
//    FP16 as BASELINE asks).  Everything else is the reference's arithmetic.
//
// Built a second time with REF_MODEL_DROPIN (libqwen_ref_b200.so): no linear()
// interposition; instead the product's host shim (host/linear_shim.cpp, which
// defines the reference's own `linear` symbol) is linked ahead of a weakened
// copy of the reference's, so the reference's forward_text runs every INT8
// product on the B200 kernels -- the drop-in as the reference host would
// link it.
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <unistd.h>
#include "model/include/load_model.hpp"
#include "model/include/forward.hpp"
#include "matmul/module.hpp"
#include "utils/include/half.hpp"

#define LINEAR_SYM _Z6linearPKvS0_S0_S0_S0_PvmmmbN5DType4TypeES3_S3_S3_bm
#define SCORES_SYM _Z21attn_scores_all_headsPKfPK6TensorPS1_miiimi
#define CAT_(a, b) a##b
#define CAT(a, b) CAT_(a, b)

#ifndef REF_MODEL_DROPIN
extern "C" void CAT(__real_, LINEAR_SYM)(const void *, const void *, const void *, const void *, const void *,
                                         void *, size_t, size_t, size_t, bool, DType::Type, DType::Type,
                                         DType::Type, DType::Type, bool, size_t);
#endif
extern "C" void CAT(__real_, SCORES_SYM)(const float *, const Tensor *, Tensor *, size_t, int, int, int, size_t,
                                         int);

namespace {
QwenConfig g_cfg;
QwenWeight g_w;
QwenRunState g_st;
bool g_loaded = false;
bool g_fp16_kv = false;

struct QuietStdout {
    int saved = -1;
    QuietStdout() {
        fflush(stdout);
        saved = dup(1);
        FILE *null = fopen("/dev/null", "w");
        if (null) { dup2(fileno(null), 1); fclose(null); }
    }
    ~QuietStdout() {
        fflush(stdout);
        if (saved >= 0) { dup2(saved, 1); close(saved); }
    }
};

inline float to_f16(float x) { return (float)half_float::half(x); }
}  // namespace

extern "C" {

#ifndef REF_MODEL_DROPIN
void CAT(__wrap_, LINEAR_SYM)(const void *A, const void *B, const void *Bs, const void *bias, const void *bias_s,
                              void *C, size_t M, size_t N, size_t K, bool transpose, DType::Type ta,
                              DType::Type tb, DType::Type tbs, DType::Type tc, bool gq, size_t g) {
    if (tb == DType::INT8 && !gq && transpose && ta == DType::FP32 && tc == DType::FP32 && !bias) {
        f32a_i8f32sb_f32c_avx2_kernel((const float *)A, (const int8_t *)B, (const float *)Bs, (float *)C, M, N, K,
                                      true, K);
        return;
    }
    CAT(__real_, LINEAR_SYM)(A, B, Bs, bias, bias_s, C, M, N, K, transpose, ta, tb, tbs, tc, gq, g);
}
#endif

void CAT(__wrap_, SCORES_SYM)(const float *key_cache, const Tensor *q, Tensor *att, size_t heads, int kv_mul,
                              int head_dim, int kv_dim, size_t sh_offset, int pos) {
    if (g_fp16_kv && g_loaded) {
        // key_cache is this layer's base inside state->key_cache [1, L, NKV, S, D]
        const float *k0 = (const float *)g_st.key_cache->ptr();
        const size_t layer_elems = (size_t)g_cfg.num_key_value_heads * sh_offset;
        const size_t l = (size_t)(key_cache - k0) / layer_elems;
        float *kl = (float *)g_st.key_cache->ptr() + l * layer_elems;
        float *vl = (float *)g_st.value_cache->ptr() + l * layer_elems;
        for (int h = 0; h < g_cfg.num_key_value_heads; ++h) {
            float *kr = kl + h * sh_offset + (size_t)pos * head_dim;
            float *vr = vl + h * sh_offset + (size_t)pos * head_dim;
            for (int d = 0; d < head_dim; ++d) {
                kr[d] = to_f16(kr[d]);
                vr[d] = to_f16(vr[d]);
            }
        }
    }
    CAT(__real_, SCORES_SYM)(key_cache, q, att, heads, kv_mul, head_dim, kv_dim, sh_offset, pos);
}

// Loads `path` (exporter .bin layout) and builds the run state.  fp16_kv: see
// the file comment.  Returns 0, or -1 if the file could not be read.
int refm_load(const char *path, int fp16_kv) {
    if (g_loaded) return -1;
    QuietStdout quiet;
    memset(&g_cfg, 0, sizeof(g_cfg));
    memset(&g_w, 0, sizeof(g_w));
    memset(&g_st, 0, sizeof(g_st));
    init_model_weights(path, &g_cfg, &g_w);
    if (!g_w.token_embedding_table || !g_w.rms_out_w) return -1;
    init_model_run_state(&g_st, &g_cfg);
    g_fp16_kv = fp16_kv != 0;
    g_loaded = true;
    return 0;
}

// vocab, hidden, intermediate, layers, heads, kv_heads, seq_len, rope_theta,
// text_bits, group_size, group_quantized, eps (float bits)
void refm_config(int32_t *out) {
    out[0] = g_cfg.vocab_size; out[1] = g_cfg.hidden_size; out[2] = g_cfg.intermediate_size;
    out[3] = g_cfg.num_hidden_layers; out[4] = g_cfg.num_attention_heads; out[5] = g_cfg.num_key_value_heads;
    out[6] = g_cfg.seq_len; out[7] = g_cfg.rope_theta; out[8] = g_cfg.text_bits; out[9] = g_cfg.group_size;
    out[10] = g_cfg.group_quantized;
    memcpy(out + 11, &g_cfg.rms_norm_eps, 4);
}

// forward_text for `token` at `pos`; returns the logits [vocab].
const float *refm_forward(int token, int pos) {
    QuietStdout quiet;
    return forward_text(&g_cfg, &g_st, &g_w, token, (size_t)pos);
}

// The text-position section of the RoPE tables [rows, D/2] (cos_tensor,
// sin_tensor section 0, model/src/load_model.cpp:413-490).
void refm_rope(float *cos_out, float *sin_out, int rows) {
    const size_t half = (size_t)g_cfg.hidden_size / g_cfg.num_attention_heads / 2;
    memcpy(cos_out, g_st.cos_tensor->ptr(), (size_t)rows * half * sizeof(float));
    memcpy(sin_out, g_st.sin_tensor->ptr(), (size_t)rows * half * sizeof(float));
}

// forward_img (model/src/forward.cpp:3-456) on preprocessed patches
// [n_patches, C*T*P*P] (copied: forward_img frees its input); then the merged
// image embeddings [d_tokens, out_hidden] (vision_x, fp32) into out_x and the
// three deep-stack rows [3][d_tokens][hidden] (fp16 in the reference) as
// float into out_deep.  Returns d_tokens, or -1.
int refm_forward_img(const float *patches, int n_patches, int grid_h, int grid_w, float *out_x, float *out_deep) {
    if (!g_loaded) return -1;
    const size_t kp = (size_t)g_cfg.vision_num_channels * g_cfg.vision_temporal_patch_size *
                      g_cfg.vision_patch_size * g_cfg.vision_patch_size;
    float *img = (float *)malloc((size_t)n_patches * kp * sizeof(float));
    if (!img) return -1;
    memcpy(img, patches, (size_t)n_patches * kp * sizeof(float));
    {
        QuietStdout quiet;
        forward_img(&g_cfg, &g_st, &g_w, img, n_patches, (int)kp, grid_h, grid_w);
    }
    const int m = g_cfg.vision_spatial_merge_size;
    const int d_tokens = n_patches / (m * m);
    const size_t oh = (size_t)g_cfg.out_hidden_size, H = (size_t)g_cfg.hidden_size;
    memcpy(out_x, g_st.vision_x->ptr(), (size_t)d_tokens * oh * sizeof(float));
    const size_t vnp_max = g_st.vision_deep_stack->shape[1];
    const half_float::half *ds = (const half_float::half *)g_st.vision_deep_stack->ptr();
    for (int d = 0; d < g_cfg.vision_deep_stack_depth; ++d)
        for (int i = 0; i < d_tokens; ++i)
            for (size_t j = 0; j < H; ++j)
                out_deep[((size_t)d * d_tokens + i) * H + j] = (float)ds[((size_t)d * vnp_max + i) * H + j];
    return d_tokens;
}

// Puts given image embeddings [d_tokens, out_hidden] (fp32) and deep-stack
// rows [3][d_tokens][hidden] (rounded to the reference's fp16) where
// forward_img leaves its results, and restarts the image-token counter, so
// that forward_text on a prompt with image tokens reads them
// (model/src/forward.cpp:476-485, 665-673).
void refm_set_vision(const float *x, const float *deep, int d_tokens) {
    const size_t oh = (size_t)g_cfg.out_hidden_size, H = (size_t)g_cfg.hidden_size;
    memcpy(g_st.vision_x->ptr(), x, (size_t)d_tokens * oh * sizeof(float));
    const size_t vnp_max = g_st.vision_deep_stack->shape[1];
    half_float::half *ds = (half_float::half *)g_st.vision_deep_stack->ptr();
    for (int d = 0; d < g_cfg.vision_deep_stack_depth; ++d)
        for (int i = 0; i < d_tokens; ++i)
            for (size_t j = 0; j < H; ++j)
                ds[((size_t)d * vnp_max + i) * H + j] = half_float::half(deep[((size_t)d * d_tokens + i) * H + j]);
    g_st.vision_embed_tokens = d_tokens;
    g_st.cur_img_token_id = 0;
}

// Releases the model so that another file can be loaded (the mapped weight
// files stay mapped: the reference's destructor unmaps an unaligned address).
void refm_free(void) {
    if (!g_loaded) return;
    QuietStdout quiet;
    free_model_run_state(&g_st);
    free_model_weights(&g_w);
    free_model_config(&g_cfg);
    g_loaded = false;
}

// key_cache / value_cache [L, NKV, S, D] fp32 (which = 0 keys, 1 values).
float *refm_kv(int which) { return (float *)(which ? g_st.value_cache : g_st.key_cache)->ptr(); }

}  // extern "C"
