// C ABI of the vision tower (vision.cu, gemm_f16_tc.cu) and its host tables.
#include <cmath>
#include <vector>
#include <cuda_fp16.h>
#include "common.cuh"
#include "vision.cuh"
#include "gemm_f16_tc.cuh"

namespace {
bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
uint16_t host_f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
}  // namespace

extern "C" {

int qvl_vision_rot_table(float theta, int head_dim, int grid_h, int grid_w, int merge, uint16_t *cos_out,
                         uint16_t *sin_out) {
    if (!cos_out || !sin_out || head_dim <= 0 || head_dim % 4 || grid_h <= 0 || grid_w <= 0 || merge <= 0 ||
        grid_h % merge || grid_w % merge)
        return QVL_ERR_INVALID;
    const int dim = head_dim / 2, half_dim = dim / 2, q = head_dim / 4;
    const int rows = grid_h > grid_w ? grid_h : grid_w;
    std::vector<float> inv(half_dim);
    for (int i = 0; i < half_dim; ++i) {
        const volatile float e = (float)(2 * i) / (float)dim;
        inv[i] = 1.0f / powf(theta, e);
    }
    std::vector<uint16_t> c((size_t)rows * half_dim), s((size_t)rows * half_dim);
    for (int p = 0; p < rows; ++p)
        for (int i = 0; i < half_dim; ++i) {
            const volatile float f = (float)p * inv[i];
            c[(size_t)p * half_dim + i] = host_f2h(cosf(f));
            s[(size_t)p * half_dim + i] = host_f2h(sinf(f));
        }
    int k = 0;
    for (int br = 0; br < grid_h / merge; ++br)
        for (int bc = 0; bc < grid_w / merge; ++bc)
            for (int ir = 0; ir < merge; ++ir)
                for (int ic = 0; ic < merge; ++ic, ++k) {
                    const int r = br * merge + ir, col = bc * merge + ic;
                    for (int part = 0; part < 4; ++part) {
                        const int src = (part % 2 == 0) ? r : col;     // row, col, row, col
                        for (int i = 0; i < q; ++i) {
                            cos_out[(size_t)k * head_dim + part * q + i] = c[(size_t)src * half_dim + i];
                            sin_out[(size_t)k * head_dim + part * q + i] = s[(size_t)src * half_dim + i];
                        }
                    }
                }
    return QVL_OK;
}

int qvl_vision_pos_interp(int grid_h, int grid_w, int num_grid_per_side, int merge, int32_t *idx_out,
                          float *w_out) {
    if (!idx_out || !w_out || grid_h <= 0 || grid_w <= 0 || num_grid_per_side <= 0 || merge <= 0 ||
        grid_h % merge || grid_w % merge)
        return QVL_ERR_INVALID;
    const float max_idx = (float)(num_grid_per_side - 1);
    const long clip = (long)num_grid_per_side - 1;
    auto axis = [&](int g, std::vector<long> &fl, std::vector<long> &ce, std::vector<float> &d) {
        fl.resize(g); ce.resize(g); d.resize(g);
        const float step = g > 1 ? max_idx / (float)(g - 1) : 0.0f;
        for (int i = 0; i < g; ++i) {
            const volatile float v = g > 1 ? (float)i * step : 0.0f;
            fl[i] = (long)floorf(v);
            ce[i] = fl[i] + 1 < clip ? fl[i] + 1 : clip;
            d[i] = v - (float)fl[i];
        }
    };
    std::vector<long> hf, hc, wf, wc;
    std::vector<float> dh, dw;
    axis(grid_h, hf, hc, dh);
    axis(grid_w, wf, wc, dw);
    int k = 0;
    for (int bh = 0; bh < grid_h / merge; ++bh)
        for (int bw = 0; bw < grid_w / merge; ++bw)
            for (int ih = 0; ih < merge; ++ih)
                for (int iw = 0; iw < merge; ++iw, ++k) {
                    const int h = bh * merge + ih, w = bw * merge + iw;
                    const long bh0 = hf[h] * num_grid_per_side, bh1 = hc[h] * num_grid_per_side;
                    idx_out[k * 4 + 0] = (int32_t)(bh0 + wf[w]);
                    idx_out[k * 4 + 1] = (int32_t)(bh0 + wc[w]);
                    idx_out[k * 4 + 2] = (int32_t)(bh1 + wf[w]);
                    idx_out[k * 4 + 3] = (int32_t)(bh1 + wc[w]);
                    const float omh = 1.0f - dh[h], omw = 1.0f - dw[w];
                    w_out[k * 4 + 0] = omh * omw;
                    w_out[k * 4 + 1] = omh * dw[w];
                    w_out[k * 4 + 2] = dh[h] * omw;
                    w_out[k * 4 + 3] = dh[h] * dw[w];
                }
    return QVL_OK;
}

int qvl_vision_patch_embed(const float *patches, const uint16_t *w, const uint16_t *b, float *x, int T, int VH,
                           int Kp, void *stream) {
    if (!patches || !w || !x || T <= 0 || VH <= 0 || Kp <= 0) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_patch_embed(patches, w, b, x, T, VH, Kp, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_vision_pos_add(float *x, const uint16_t *pos_w, const int32_t *idx, const float *wts, int T, int VH,
                       void *stream) {
    if (!x || !pos_w || !idx || !wts || T <= 0 || VH <= 0) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_pos_add(x, pos_w, idx, wts, T, VH, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_layer_norm(const void *x, int x_f16, const uint16_t *gamma, const uint16_t *beta, void *out, int out_f16,
                   int rows, int H, float eps, void *stream) {
    if (!x || !gamma || !beta || !out || rows <= 0 || H <= 0) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_layer_norm(x, x_f16 != 0, gamma, beta, out, out_f16 != 0, rows, H, eps,
                                        (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_gemm_f16(const uint16_t *A, const uint16_t *W, const uint16_t *bias, void *C, size_t M, size_t N, size_t K,
                 int mode, void *stream) {
    if (!A || !W || !C) return QVL_ERR_INVALID;
    if (mode < 0 || mode > 3) return QVL_ERR_INVALID;
    if (M == 0) return QVL_OK;
    if (!al16(A) || !al16(W) || M > (size_t)INT32_MAX || N > (size_t)INT32_MAX) return QVL_ERR_INVALID;
    if (!qvl::gemm_f16_supported(M, N, K)) return QVL_ERR_UNSUPPORTED;
    QVL_CUDA_TRY(qvl::launch_gemm_f16_tc(reinterpret_cast<const __half *>(A), reinterpret_cast<const __half *>(W),
                                         reinterpret_cast<const __half *>(bias), C, (int)M, (int)N, (int)K, mode,
                                         (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_vision_rotary(uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t, int T, int NH, int HD,
                      void *stream) {
    if (!x || !cos_t || !sin_t || T <= 0 || NH <= 0 || HD <= 0 || HD % 2) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_vision_rotary(x, cos_t, sin_t, T, NH, HD, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_vision_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int T, int NH,
                         int HD, float scale, void *stream) {
    if (!q || !k || !v || !out || T <= 0 || NH <= 0) return QVL_ERR_INVALID;
    if (HD != 64 || T > qvl::vision_max_tokens()) return QVL_ERR_UNSUPPORTED;
    if (!al16(q) || !al16(k) || !al16(v) || !al16(out)) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_vision_attention(q, k, v, out, T, NH, scale, (cudaStream_t)stream));
    return QVL_OK;
}

}  // extern "C"
