#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace qvl {

struct AttnArgs {
    const float *q;
    const uint16_t *k_pages, *v_pages;
    const int32_t *page_table, *seq_ids, *positions;
    size_t nq;
    int max_ctx;
    float *out;
    int NH, NKV, P, maxp, max_pos;
    // optional quantisation of `out` rows (per-row group) for the next linear;
    // honoured by the single-launch cluster path, otherwise done separately
    int16_t *q_out;
    float *q_out_scales;
    int *counter;
};

// Optional per-layer QK-norm: INT8 weights [D] with fp32 group scales.
struct QkNorm {
    const int8_t *q_w;   // nullptr: no QK-norm
    const float *q_s;
    const int8_t *k_w;
    const float *k_s;
    int gs;
    float eps;
};

struct RopeArgs {
    float *q;
    const float *k_new, *v_new;
    uint16_t *k_pages, *v_pages;
    const int32_t *page_table, *seq_ids, *positions;
    size_t nq;
    const float *rope_cos, *rope_sin;
    int NH, NKV, P, maxp, max_pos;
    QkNorm norm;
};

// Split-K scratch: raw scores, chunk maxima, chunk sums, chunk partial outputs.
struct AttnScratch {
    int chunk, nchunk;
    size_t scores_off, cmax_off, psum_off, pacc_off, total;
};

bool attn_use_cluster(size_t nq, int max_ctx, int nkv);
int attn_chunk_tokens(size_t nq, int max_ctx, int nkv);
AttnScratch attn_scratch_layout(size_t nq, int max_ctx, int NH, int nkv);
cudaError_t launch_attention(const AttnArgs &a, void *workspace, cudaStream_t stream);
cudaError_t launch_rope_append(const RopeArgs &a, cudaStream_t stream);

}  // namespace qvl
