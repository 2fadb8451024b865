// C ABI of the one-launch decode token (decode_persistent.cu).
#include "common.cuh"
#include "decode_persistent.cuh"

namespace {

constexpr int kMaxCtas = 1024;
constexpr size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

// Workspace layout; the barrier words come first so that they keep their
// place whatever the device's SM count.
struct DecodeWs {
    size_t bar, trace, x_qkv, h, lmax, lsum, pacc, cnt, att, best_v, best_i, e, total;
};
constexpr DecodeWs decode_ws() {
    DecodeWs w{};
    w.bar = 0;                                             // bar_count (u64), abort (int at +8), head_bar [8] u64 at +64
    w.trace = 256;
    w.x_qkv = w.trace + qvl::kPersistTraceSlots * 8;
    w.h = w.x_qkv + al256((16 * 128 + 2 * 8 * 128) * 4);
    w.lmax = w.h + al256(6144 * 4);
    w.lsum = w.lmax + al256(16 * qvl::kPersistSlices * 4);
    w.pacc = w.lsum + al256(16 * qvl::kPersistSlices * 8);
    w.cnt = w.pacc + al256(16 * qvl::kPersistSlices * 128 * 4);
    w.att = w.cnt + 256;
    w.best_v = w.att + al256(16 * 128 * 4);
    w.best_i = w.best_v + al256(kMaxCtas * qvl::kPersistWarpsPerCta * 4);
    w.e = w.best_i + al256(kMaxCtas * qvl::kPersistWarpsPerCta * 4);
    w.total = w.e + al256(16 * qvl::kPersistSlices * 512 * 4);
    return w;
}

}  // namespace

extern "C" {

size_t qvl_text_decode_workspace_bytes(void) { return decode_ws().total; }

int *qvl_text_decode_abort_flag(void *workspace) {
    return workspace ? reinterpret_cast<int *>(static_cast<unsigned char *>(workspace) + 8) : nullptr;
}

const uint64_t *qvl_text_decode_trace(const void *workspace) {
    return workspace ? reinterpret_cast<const uint64_t *>(static_cast<const unsigned char *>(workspace) +
                                                          decode_ws().trace)
                     : nullptr;
}

int qvl_text_decode_step(const qvl_text_weights *w, float *x, float *logits, int32_t *token, int32_t *pos,
                         uint16_t *k_pages, uint16_t *v_pages, long kv_layer_stride, const int32_t *page_table,
                         int page_size, const float *rope_cos, const float *rope_sin, int max_ctx, void *workspace,
                         size_t workspace_bytes, void *stream) {
    return qvl_text_decode_step_ex(w, x, logits, token, pos, k_pages, v_pages, kv_layer_stride, page_table,
                                   page_size, rope_cos, rope_sin, max_ctx, workspace, workspace_bytes, 0, stream);
}

int qvl_text_decode_step_ex(const qvl_text_weights *w, float *x, float *logits, int32_t *token, int32_t *pos,
                            uint16_t *k_pages, uint16_t *v_pages, long kv_layer_stride, const int32_t *page_table,
                            int page_size, const float *rope_cos, const float *rope_sin, int max_ctx,
                            void *workspace, size_t workspace_bytes, int flags, void *stream) {
    if (flags & ~QVL_DECODE_REFERENCE_ORDER) return QVL_ERR_INVALID;
    if (!w || !x || !logits || !token || !pos || !k_pages || !v_pages || !page_table || !rope_cos || !rope_sin)
        return QVL_ERR_INVALID;
    const void *ptrs[] = {w->w_q, w->w_k, w->w_v, w->w_o, w->w_gate, w->w_up, w->w_down, w->s_q, w->s_k,
                          w->s_v, w->s_o, w->s_gate, w->s_up, w->s_down, w->in_norm, w->post_norm, w->q_norm,
                          w->k_norm, w->in_norm_s, w->post_norm_s, w->q_norm_s, w->k_norm_s, w->final_norm,
                          w->final_norm_s, w->embed, w->embed_s};
    for (const void *p : ptrs)
        if (!p) return QVL_ERR_INVALID;
    if (w->layers <= 0 || w->vocab <= 0 || w->vocab % 16 || page_size < 16 || page_size % 16 || kv_layer_stride <= 0 || !(w->eps >= 0.0f))
        return QVL_ERR_INVALID;
    if (w->norm_group < 16 || w->head_dim % w->norm_group || w->hidden % w->norm_group) return QVL_ERR_INVALID;
    if (!qvl::persist_supported(w->hidden, w->intermediate, w->heads, w->kv_heads, w->head_dim, max_ctx))
        return QVL_ERR_UNSUPPORTED;
    // 16-byte copies of weight rows and their scales, 16-byte KV rows and activations
    const void *aligned[] = {w->w_q, w->w_k, w->w_v, w->w_o, w->w_gate, w->w_up, w->w_down, w->embed,
                             w->s_q, w->s_k, w->s_v, w->s_o, w->s_gate, w->s_up, w->s_down, w->embed_s,
                             k_pages, v_pages, x};
    for (const void *p : aligned)
        if (reinterpret_cast<uintptr_t>(p) & 15) return QVL_ERR_INVALID;
    if (kv_layer_stride % 8) return QVL_ERR_INVALID;
    const DecodeWs L = decode_ws();
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return QVL_ERR_WORKSPACE;
    const int ctas = qvl::persist_grid_ctas();
    if (ctas <= 0 || ctas > kMaxCtas) return QVL_ERR_UNSUPPORTED;

    unsigned char *ws = static_cast<unsigned char *>(workspace);
    qvl::PersistWeights pw{};
    pw.wq = w->w_q; pw.wk = w->w_k; pw.wv = w->w_v; pw.wo = w->w_o;
    pw.wg = w->w_gate; pw.wu = w->w_up; pw.wd = w->w_down;
    pw.sq = w->s_q; pw.sk = w->s_k; pw.sv = w->s_v; pw.so = w->s_o;
    pw.sg = w->s_gate; pw.su = w->s_up; pw.sd = w->s_down;
    pw.in_norm = w->in_norm; pw.post_norm = w->post_norm; pw.q_norm = w->q_norm; pw.k_norm = w->k_norm;
    pw.in_norm_s = w->in_norm_s; pw.post_norm_s = w->post_norm_s;
    pw.q_norm_s = w->q_norm_s; pw.k_norm_s = w->k_norm_s;
    pw.final_norm = w->final_norm; pw.final_norm_s = w->final_norm_s;
    pw.embed = w->embed; pw.embed_s = w->embed_s;
    pw.layers = w->layers; pw.vocab = w->vocab; pw.norm_group = w->norm_group; pw.eps = w->eps;

    qvl::PersistState ps{};
    ps.x = x;
    ps.qkv = reinterpret_cast<float *>(ws + L.x_qkv);
    ps.h = reinterpret_cast<float *>(ws + L.h);
    ps.logits = logits;
    ps.att_lmax = reinterpret_cast<float *>(ws + L.lmax);
    ps.att_lsum = reinterpret_cast<double *>(ws + L.lsum);
    ps.att_pacc = reinterpret_cast<float *>(ws + L.pacc);
    ps.att_e = reinterpret_cast<float *>(ws + L.e);
    ps.ordered = (flags & QVL_DECODE_REFERENCE_ORDER) ? 1 : 0;
    ps.att_cnt = reinterpret_cast<int *>(ws + L.cnt);
    ps.att_out = reinterpret_cast<float *>(ws + L.att);
    ps.warp_best_v = reinterpret_cast<float *>(ws + L.best_v);
    ps.warp_best_i = reinterpret_cast<int *>(ws + L.best_i);
    ps.token = token;
    ps.pos = pos;
    ps.k_pages = k_pages;
    ps.v_pages = v_pages;
    ps.kv_layer_stride = kv_layer_stride;
    ps.page_table = page_table;
    ps.page_size = page_size;
    ps.rope_cos = rope_cos;
    ps.rope_sin = rope_sin;
    ps.max_ctx = max_ctx;
    ps.bar_count = reinterpret_cast<unsigned long long *>(ws);
    ps.head_bar = reinterpret_cast<unsigned long long *>(ws + 64);
    ps.abort_flag = reinterpret_cast<int *>(ws + 8);
    ps.trace = reinterpret_cast<unsigned long long *>(ws + L.trace);
    QVL_CUDA_TRY(qvl::launch_decode_persistent(pw, ps, ctas, (cudaStream_t)stream));
    return QVL_OK;
}

}  // extern "C"
