#pragma once
#include "attention.cuh"

namespace qvl {
// Decode attention in the reference's summation order (attention_ordered.cu).
// Workspace: fp32 scores [nq, NH, max_ctx].
size_t attn_ordered_workspace_bytes(size_t nq, int max_ctx, int NH);
cudaError_t launch_attention_ordered(const AttnArgs &a, void *workspace, cudaStream_t stream);
}  // namespace qvl
