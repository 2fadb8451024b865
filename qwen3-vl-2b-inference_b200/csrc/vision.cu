// Vision tower of Qwen3-VL (forward_img, model/src/forward.cpp:3-456) on the
// GPU: the operators of layers/src/vision_layer.cpp other than the linear
// layers (which run on gemm_f16_tc.cu), plus the host-side tables.
//
//   patch embed      conv_3d as a product, fp32 image patches x fp16 kernel
//                    (vision_layer.cpp:3-217), fp32 out
//   position embed   bilinear 4-tap interpolation of the 48x48 learned table,
//                    taps and weights from qvl_vision_pos_interp, stored fp16
//                    in merge order and added to the fp32 stream (:219-504,
//                    then add_vector)
//   layer_norm       mean, variance, (x - mean) * inv_std * gamma + beta
//                    (:625-724), fp32 or fp16 in / out
//   rotary           2-D rotary embedding on fp16 q / k rows (:726-776),
//                    tables from qvl_vision_rot_table
//   attention        full (non-causal) attention per head: fp32 scores
//                    times the scale, max, exp256_ps, the sum, P.V times
//                    1/sum, fp16 out (vision_att, :821-867; the softmax is
//                    avx2_max / avx2_sum_exp_max, layers/include/simd_utils.hpp)
//
// Tensors keep the reference's token-major layout [T, heads, head_dim]; the
// reference's transposes to head-major (tensor_transpose) are folded into the
// attention kernel's indexing.  Parity is by tolerance (fp16 intermediates,
// fp32 sums in a different order).
#include <cuda_fp16.h>
#include <cmath>
#include "common.cuh"
#include "vision.cuh"

namespace qvl {

namespace {
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
}  // namespace

// out[t][n] = sum_c img[t][c] * w[n][c] + b[n]; 64x64 output tiles, K in 32s.
__global__ void __launch_bounds__(256)
patch_embed_kernel(const float *__restrict img, const uint16_t *__restrict w, const uint16_t *__restrict b,
                   float *__restrict out, int T, int N, int K) {
    __shared__ float As[32][65];
    __shared__ float Ws[32][65];
    const int t0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int e = threadIdx.x; e < 64 * 32; e += 256) {
            const int r = e >> 5, c = e & 31;
            As[c][r] = (t0 + r < T && k0 + c < K) ? img[(size_t)(t0 + r) * K + k0 + c] : 0.0f;
            Ws[c][r] = (n0 + r < N && k0 + c < K) ? h2f(w[(size_t)(n0 + r) * K + k0 + c]) : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < 32; ++c) {
            float a[4], bw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[c][ty * 4 + i];
                bw[i] = Ws[c][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bw[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = t0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (t < T && n < N) out[(size_t)t * N + n] = __fadd_rn(acc[i][j], b ? h2f(b[n]) : 0.0f);
        }
}

// x[t][j] += float(fp16(sum_k pos[idx[t][k]][j] * wt[t][k]))
__global__ void pos_add_kernel(float *__restrict x, const uint16_t *__restrict pos, const int32_t *__restrict idx,
                               const float *__restrict wt, int T, int H) {
    const int t = blockIdx.x;
    if (t >= T) return;
    const int i0 = idx[t * 4], i1 = idx[t * 4 + 1], i2 = idx[t * 4 + 2], i3 = idx[t * 4 + 3];
    const float w0 = wt[t * 4], w1 = wt[t * 4 + 1], w2 = wt[t * 4 + 2], w3 = wt[t * 4 + 3];
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        float p = 0.0f;
        p = __fadd_rn(p, __fmul_rn(h2f(pos[(size_t)i0 * H + j]), w0));
        p = __fadd_rn(p, __fmul_rn(h2f(pos[(size_t)i1 * H + j]), w1));
        p = __fadd_rn(p, __fmul_rn(h2f(pos[(size_t)i2 * H + j]), w2));
        p = __fadd_rn(p, __fmul_rn(h2f(pos[(size_t)i3 * H + j]), w3));
        float *xp = x + (size_t)t * H + j;
        *xp = __fadd_rn(*xp, h2f(f2h(p)));
    }
}

// One row per block (256 threads).
template <bool XF16, bool OF16>
__global__ void __launch_bounds__(256)
layer_norm_kernel(const void *__restrict xv, const uint16_t *__restrict g, const uint16_t *__restrict bb,
                  void *__restrict ov, int H, float eps) {
    __shared__ float red[8];
    __shared__ float stat[2];
    const int row = blockIdx.x;
    auto ld = [&](int j) -> float {
        return XF16 ? h2f(reinterpret_cast<const uint16_t *>(xv)[(size_t)row * H + j])
                    : reinterpret_cast<const float *>(xv)[(size_t)row * H + j];
    };
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float s = 0.0f;
    for (int j = threadIdx.x; j < H; j += 256) s += ld(j);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < 8; ++w) t += red[w];
        stat[0] = __fmul_rn(t, __fdiv_rn(1.0f, (float)H));
    }
    __syncthreads();
    const float mean = stat[0];
    float v = 0.0f;
    for (int j = threadIdx.x; j < H; j += 256) {
        const float d = __fsub_rn(ld(j), mean);
        v = __fadd_rn(v, __fmul_rn(d, d));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < 8; ++w) t += red[w];
        const float var = __fmul_rn(t, __fdiv_rn(1.0f, (float)H));
        stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const float inv = stat[1];
    for (int j = threadIdx.x; j < H; j += 256) {
        const float y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(ld(j), mean), inv), h2f(g[j])), h2f(bb[j]));
        if (OF16) reinterpret_cast<uint16_t *>(ov)[(size_t)row * H + j] = f2h(y);
        else reinterpret_cast<float *>(ov)[(size_t)row * H + j] = y;
    }
}

// In place on x fp16 [T, NH, HD]; cos/sin fp16 [T, HD].
__global__ void rotary_kernel(uint16_t *__restrict x, const uint16_t *__restrict cs, const uint16_t *__restrict sn,
                              int T, int NH, int HD) {
    const int half = HD / 2;
    const long n = (long)T * NH * half;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
        const int m = (int)(e % half);
        const long th = e / half;
        const int t = (int)(th / NH);
        uint16_t *p = x + th * HD;
        const float x1 = h2f(p[m]), x2 = h2f(p[m + half]);
        const float c1 = h2f(cs[(size_t)t * HD + m]), s1 = h2f(sn[(size_t)t * HD + m]);
        const float c2 = h2f(cs[(size_t)t * HD + m + half]), s2 = h2f(sn[(size_t)t * HD + m + half]);
        p[m] = f2h(__fsub_rn(__fmul_rn(x1, c1), __fmul_rn(x2, s1)));
        p[m + half] = f2h(__fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2)));
    }
}

__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

// One warp per (query, head), kVQ queries of one head per block, so the
// head's K and V rows are staged in shared memory once per block -- chunks of
// kVChunk positions, double-buffered with cp.async so the next chunk loads
// while this one is used -- instead of being read from L2 by every query; the
// scores of each query row stay in shared memory.  q, k, v, out fp16
// [T, NH, HD] (HD = 64).
constexpr int kVQ = 16;
constexpr int kVChunk = 128;
constexpr int kVisMaxT = 2048;
constexpr int kKRow = 72;             // halves per staged key row (64 + 8 pad: 4-way banks)
__global__ void __launch_bounds__(kVQ * 32)
vision_attention_kernel(const uint16_t *__restrict q, const uint16_t *__restrict k, const uint16_t *__restrict v,
                        uint16_t *__restrict out, int T, int NH, float scale) {
    constexpr int HD = 64;
    extern __shared__ __align__(16) unsigned char vsm[];
    __half *Ks = reinterpret_cast<__half *>(vsm);                       // [2][kVChunk][kKRow]
    __half *Vs = Ks + 2 * kVChunk * kKRow;                               // [2][kVChunk][HD]
    float *sc = reinterpret_cast<float *>(Vs + 2 * kVChunk * HD);        // [kVQ][T]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int i = blockIdx.x * kVQ + warp;
    const bool active = i < T;
    float *s = sc + (size_t)warp * T;
    const size_t row = (size_t)NH * HD;
    const int nch = (T + kVChunk - 1) / kVChunk;
    auto issue_k = [&](int c) {
        const int c0 = c * kVChunk, n = min(kVChunk, T - c0);
        __half *dst = Ks + (c & 1) * kVChunk * kKRow;
        for (int e = threadIdx.x; e < n * (HD / 8); e += blockDim.x) {
            const int r = e >> 3, cc = e & 7;
            cp16(dst + r * kKRow + cc * 8, k + (size_t)(c0 + r) * row + (size_t)h * HD + cc * 8);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto issue_v = [&](int c) {
        const int c0 = c * kVChunk, n = min(kVChunk, T - c0);
        __half *dst = Vs + (c & 1) * kVChunk * HD;
        for (int e = threadIdx.x; e < n * (HD / 8); e += blockDim.x) {
            const int r = e >> 3, cc = e & 7;
            cp16(dst + r * HD + cc * 8, v + (size_t)(c0 + r) * row + (size_t)h * HD + cc * 8);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue_k(0);
    float qf[HD];
    if (active) {
        const uint4 *qp = reinterpret_cast<const uint4 *>(q + (size_t)i * row + (size_t)h * HD);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
            const uint4 u = qp[c];
            const __half2 *hh = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(hh[j]);
                qf[8 * c + 2 * j] = f.x;
                qf[8 * c + 2 * j + 1] = f.y;
            }
        }
    }
    float mx = -INFINITY;
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            issue_k(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            issue_v(0);                      // V's first chunk loads during the last scores
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        }
        __syncthreads();
        const int c0 = c * kVChunk, n = min(kVChunk, T - c0);
        const __half *kb = Ks + (c & 1) * kVChunk * kKRow;
        if (active) {
            for (int t = lane; t < n; t += 32) {
                const uint4 *kp = reinterpret_cast<const uint4 *>(kb + t * kKRow);
                float a = 0.0f;
#pragma unroll
                for (int cc = 0; cc < HD / 8; ++cc) {
                    const uint4 u = kp[cc];
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(hh[j]);
                        a = fmaf(qf[8 * cc + 2 * j], f.x, a);
                        a = fmaf(qf[8 * cc + 2 * j + 1], f.y, a);
                    }
                }
                a = __fmul_rn(a, scale);
                s[c0 + t] = a;
                mx = fmaxf(mx, a);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    if (active)
        for (int t = lane; t < T; t += 32) {
            const float e = exp_ref(__fsub_rn(s[t], mx));
            s[t] = e;
            sum += e;
        }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncwarp();
    const float inv = __fdiv_rn(1.0f, sum);
    // P.V: lane owns output dims 2*lane, 2*lane+1
    float o0 = 0.0f, o1 = 0.0f;
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            issue_v(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int c0 = c * kVChunk, n = min(kVChunk, T - c0);
        const __half *vb = Vs + (c & 1) * kVChunk * HD;
        if (active)
            for (int t = 0; t < n; ++t) {
                const float p = s[c0 + t];
                const float2 f = __half22float2(reinterpret_cast<const __half2 *>(vb + t * HD)[lane]);
                o0 = fmaf(p, f.x, o0);
                o1 = fmaf(p, f.y, o1);
            }
        __syncthreads();
    }
    if (active) {
        __half2 r = __floats2half2_rn(__fmul_rn(o0, inv), __fmul_rn(o1, inv));
        reinterpret_cast<__half2 *>(out + (size_t)i * row + (size_t)h * HD)[lane] = r;
    }
}

cudaError_t launch_patch_embed(const float *img, const uint16_t *w, const uint16_t *b, float *out, int T, int N, int K,
                               cudaStream_t st) {
    dim3 grid((N + 63) / 64, (T + 63) / 64);
    patch_embed_kernel<<<grid, 256, 0, st>>>(img, w, b, out, T, N, K);
    return cudaGetLastError();
}

cudaError_t launch_pos_add(float *x, const uint16_t *pos, const int32_t *idx, const float *wt, int T, int H,
                           cudaStream_t st) {
    pos_add_kernel<<<T, 256, 0, st>>>(x, pos, idx, wt, T, H);
    return cudaGetLastError();
}

cudaError_t launch_layer_norm(const void *x, bool x_f16, const uint16_t *g, const uint16_t *b, void *out, bool out_f16,
                              int rows, int H, float eps, cudaStream_t st) {
    if (x_f16 && out_f16) layer_norm_kernel<true, true><<<rows, 256, 0, st>>>(x, g, b, out, H, eps);
    else if (x_f16) layer_norm_kernel<true, false><<<rows, 256, 0, st>>>(x, g, b, out, H, eps);
    else if (out_f16) layer_norm_kernel<false, true><<<rows, 256, 0, st>>>(x, g, b, out, H, eps);
    else layer_norm_kernel<false, false><<<rows, 256, 0, st>>>(x, g, b, out, H, eps);
    return cudaGetLastError();
}

cudaError_t launch_vision_rotary(uint16_t *x, const uint16_t *cs, const uint16_t *sn, int T, int NH, int HD,
                                 cudaStream_t st) {
    const long n = (long)T * NH * (HD / 2);
    const long blocks = (n + 255) / 256;
    rotary_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, st>>>(x, cs, sn, T, NH, HD);
    return cudaGetLastError();
}

cudaError_t launch_vision_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int T,
                                    int NH, float scale, cudaStream_t st) {
    const size_t smem = 2 * ((size_t)kVChunk * kKRow * 2 + (size_t)kVChunk * 64 * 2) + (size_t)kVQ * T * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(vision_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((T + kVQ - 1) / kVQ, NH);
    vision_attention_kernel<<<grid, kVQ * 32, smem, st>>>(q, k, v, out, T, NH, scale);
    return cudaGetLastError();
}

int vision_max_tokens() { return kVisMaxT; }

}  // namespace qvl
