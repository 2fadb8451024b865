#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace qvl {

// Weights of the text decoder, reference layout, stacked over layers.
struct PersistWeights {
    const int8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;        // [L, N, K]
    const float *sq, *sk, *sv, *so, *sg, *su, *sd;         // [L, N] per-row scales
    const int8_t *in_norm, *post_norm, *q_norm, *k_norm;   // [L, n]
    const float *in_norm_s, *post_norm_s, *q_norm_s, *k_norm_s;   // [L, n / norm_group]
    const int8_t *final_norm;
    const float *final_norm_s;
    const int8_t *embed;                                    // [V, H] tied embedding / LM head
    const float *embed_s;                                   // [V]
    int layers, vocab, norm_group;
    float eps;
};

struct PersistState {
    float *x;              // [H] residual stream
    float *qkv;            // [NH*D + 2*NKV*D]
    float *h;              // [I] SwiGLU output
    float *logits;         // [V]
    float *att_lmax;       // [NH][16] slice maxima
    double *att_lsum;      // [NH][16] slice sums
    float *att_pacc;       // [NH][16][D] slice partial outputs
    float *att_e;          // [NH][16 * 512] exponentials (reference-order mode)
    int ordered;           // attention in the reference's summation order
    int *att_cnt;          // [NKV] slices finished (zero between layers)
    float *att_out;        // [NH * D] attention output
    float *warp_best_v;    // [grid * 16]
    int *warp_best_i;      // [grid * 16]
    int32_t *token;        // [1] input token, replaced by the greedy token
    int32_t *pos;          // [1] position of the input token, advanced by one
    uint16_t *k_pages, *v_pages;    // [L] x [pages, NKV, page, D] fp16
    long kv_layer_stride;           // elements per layer
    const int32_t *page_table;      // [max_pages]
    int page_size;
    const float *rope_cos, *rope_sin;   // [max_pos, D/2]
    int max_ctx;
    unsigned long long *bar_count;      // grid barrier: arrivals since the workspace was zeroed
    unsigned long long *head_bar;       // [NKV] barriers of the 16 slice CTAs of each KV head
    int *abort_flag;                    // set to 1 if a barrier wait timed out
    unsigned long long *trace;          // [kPersistTraceSlots] kernel start + barrier opening times (ns)
};

// Dimensions the kernel is compiled for (Qwen3-VL-2B text decoder).
bool persist_supported(int hidden, int intermediate, int heads, int kv_heads, int head_dim, int max_ctx);
// CTAs of the cooperative grid on the current device (one per SM), 0 if the
// kernel cannot be made resident.  warp_best_* need ctas * 16 entries.
int persist_grid_ctas();
constexpr int kPersistWarpsPerCta = 16;
constexpr int kPersistSlices = 16;
constexpr unsigned kPersistTraceSlots = 1024;
cudaError_t launch_decode_persistent(const PersistWeights &w, const PersistState &s, int ctas, cudaStream_t stream);

}  // namespace qvl
