#pragma once
#include "attention.cuh"

namespace qvl {
// Decode attention in the reference's summation order (attention_ordered.cu).
// Workspace: fp32 scores [nq, NH, max_ctx].
size_t attn_ordered_workspace_bytes(size_t nq, int max_ctx, int NH);
// The raw projections of a decode step for the fused QK-norm + RoPE + append
// (launch_attention_ordered's `rope`; AttnArgs::q is then the raw q).  Each
// query must belong to a different sequence.
struct OrdRope {
    const float *k_new, *v_new;           // [nq, NKV, D]
    uint16_t *k_pages, *v_pages;          // the cache pages, written at each query's position
    const float *rope_cos, *rope_sin;     // [max_ctx, D/2]
    QkNorm norm;                          // q_w == nullptr: no QK-norm
};
cudaError_t launch_attention_ordered(const AttnArgs &a, void *workspace, cudaStream_t stream,
                                     const OrdRope *rope = nullptr);
}  // namespace qvl
