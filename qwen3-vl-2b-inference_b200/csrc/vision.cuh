#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace qvl {
// Vision-tower operators (vision.cu); fp16 tensors are passed as uint16_t.
cudaError_t launch_patch_embed(const float *img, const uint16_t *w, const uint16_t *b, float *out, int T, int N, int K,
                               cudaStream_t st);
cudaError_t launch_pos_add(float *x, const uint16_t *pos, const int32_t *idx, const float *wt, int T, int H,
                           cudaStream_t st);
cudaError_t launch_layer_norm(const void *x, bool x_f16, const uint16_t *g, const uint16_t *b, void *out, bool out_f16,
                              int rows, int H, float eps, cudaStream_t st);
cudaError_t launch_vision_rotary(uint16_t *x, const uint16_t *cs, const uint16_t *sn, int T, int NH, int HD,
                                 cudaStream_t st);
cudaError_t launch_vision_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int T,
                                    int NH, float scale, cudaStream_t st);
int vision_max_tokens();
}  // namespace qvl
