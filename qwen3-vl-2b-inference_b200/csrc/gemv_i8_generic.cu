// Decode-shape INT8 GEMV (M = 1..8 activation rows) on CUDA cores.
//
// Replaces gemv_lg_N_lg_K_transpose / gemv_lg_N_lg_K_transpose_decode
// (matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:122-224, :327-455) and, with
// TILED semantics, the small-M rows of linear_int8_fp32s_int32acc_transpose
// (:458-663).  The kernel is bound by HBM bandwidth: every weight byte is
// read once with a 128-bit streaming load, and activations are staged once
// per CTA in shared memory as int16.
//
// Work mapping.  One warp owns one output row n at a time (rows strided over
// all warps of the grid).  A row is consumed in "steps" of 512 bytes: lane t
// of the warp takes the 16-byte chunk c = 32*it + t.  Chunk c covers columns
// 16c..16c+15, so its 8 dp2a results are exactly the 8 int32 lanes of the
// reference's _mm256_madd_epi16 (lane l <- columns 2l, 2l+1).
//
// Groups.  A K-group of g columns spans g/16 chunks: with g >= 512 a group
// covers g/512 consecutive steps of the whole warp (segment = 32 lanes); with
// g < 512 one step covers 512/g groups, each a segment of g/16 lanes.  At the
// end of a group the per-lane int32 partials of the segment are reduced with a
// transposing butterfly (exact integer adds), after which each thread holds
// one of the 8 lanes.  The fp32 part -- fma(float(lane), a_s*w_s, cf) chained
// over the groups in ascending order, then the (l, l+4) pairwise reduction --
// follows the reference operation by operation, so outputs are bit-exact.
#include "common.cuh"
#include "gemv_common.cuh"
#include "qact.cuh"

// Generic path (any M <= 8, any supported g): stepwise row walk.
namespace qvl {

template <int MR, bool LANE, int SEGLOG>
__global__ void __launch_bounds__(kThreads)
gemv_i8_kernel(const int16_t *__restrict q, const float *__restrict qs,
               const int8_t *__restrict W, const float *__restrict ws, float *__restrict y,
               int M, int N, int K, int g, long ldy, int acc) {
    extern __shared__ __align__(16) unsigned char smem[];
    int16_t *q_s = reinterpret_cast<int16_t *>(smem);
    const int G = K / g;
    float *qs_s = reinterpret_cast<float *>(smem + (size_t)MR * K * sizeof(int16_t));

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const long nwarps = (long)gridDim.x * kWarpsPerBlock;
    const long wid = (long)blockIdx.x * kWarpsPerBlock + warp;
    const int NCH = K / 16;
    const int IT = (NCH + 31) / 32;
    const long nrows_w = (wid < N) ? (N - 1 - wid) / nwarps + 1 : 0;
    const long total = nrows_w * IT;

    constexpr int seg = 1 << SEGLOG;
    const int CPG = g / 16;                // chunks per group
    const int IPG = (CPG >= 32) ? CPG / 32 : 1;
    constexpr int GPI = (SEGLOG >= 5) ? 1 : (32 >> SEGLOG);  // groups per step when g < 512

    auto chunk_ptr = [&](long s) -> const uint4 * {
        long r = s / IT;
        int it = (int)(s - r * IT);
        long n = wid + r * nwarps;
        int c = it * 32 + lane;
        if (c >= NCH) c = NCH - 1;   // clamp (value masked later)
        return reinterpret_cast<const uint4 *>(W + n * (long)K) + c;
    };

    // Prefetch the first steps' weights before waiting on the producer kernel.
    uint4 wbuf[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
        if (u < total) wbuf[u] = ld_stream_v4(chunk_ptr(u));

    pdl_launch_dependents();
    pdl_wait();

    // Stage activations (int16) and their group scales.
    {
        const int nq16 = M * K / 8;   // int4 units (8 x int16)
        const int4 *src = reinterpret_cast<const int4 *>(q);
        int4 *dst = reinterpret_cast<int4 *>(q_s);
        for (int i = threadIdx.x; i < nq16; i += kThreads) dst[i] = src[i];
        for (int i = threadIdx.x; i < M * G; i += kThreads) qs_s[i] = qs[i];
    }
    __syncthreads();

    RowState<MR, LANE, SEGLOG> st;
    auto reset_row = [&]() {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            st.cf[m] = 0.0f;
#pragma unroll
            for (int l = 0; l < 8; ++l) st.part[m][l] = 0;
            if constexpr (SEGLOG < 3) {
#pragma unroll
                for (int l = 0; l < 8; ++l) st.cf8[m][l] = 0.0f;
            }
        }
    };
    reset_row();

    for (long s0 = 0; s0 < total; s0 += kUnroll) {
        uint4 nbuf[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (s0 + kUnroll + u < total) nbuf[u] = ld_stream_v4(chunk_ptr(s0 + kUnroll + u));

#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const long s = s0 + u;
            if (s >= total) break;
            const long r = s / IT;
            const int it = (int)(s - r * IT);
            const long n = wid + r * nwarps;
            const int c = it * 32 + lane;
            const bool valid = c < NCH;
            uint4 w = wbuf[u];
            if (!valid) w = make_uint4(0, 0, 0, 0);
            const int cc = valid ? c : 0;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                if (m < M) {
                    const int4 *ap = reinterpret_cast<const int4 *>(q_s + (size_t)m * K + cc * 16);
                    madd_chunk(w, ap[0], ap[1], st.part[m]);
                }
            }
            // ---- group boundary ----
            const bool group_end = (SEGLOG >= 5) ? ((it + 1) % IPG == 0) : true;
            if (group_end) {
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    if (m >= M) continue;
                    if constexpr (LANE) {
                        if constexpr (SEGLOG >= 3) {
                            int v = seg_transpose_reduce<SEGLOG>(st.part[m], lane);
                            if constexpr (SEGLOG >= 5) {
                                const int gi = it / IPG;
                                const int l8 = seg_lane_id<SEGLOG>(lane);
                                (void)l8;
                                float sc = mul_rn(qs_s[m * G + gi], __ldg(ws + n * (long)G + gi));
                                st.cf[m] = fma_rn(__int2float_rn(v), sc, st.cf[m]);
                            } else {
#pragma unroll
                                for (int sgi = 0; sgi < GPI; ++sgi) {
                                    int vs = __shfl_sync(0xffffffffu, v, sgi * seg + (lane & (seg - 1)));
                                    const int gi = it * GPI + sgi;
                                    if (gi < G) {
                                        float sc = mul_rn(qs_s[m * G + gi], __ldg(ws + n * (long)G + gi));
                                        st.cf[m] = fma_rn(__int2float_rn(vs), sc, st.cf[m]);
                                    }
                                }
                            }
                        } else {
                            // seg < 8: plain butterfly, every thread gets all 8 lanes.
#pragma unroll
                            for (int l = 0; l < 8; ++l)
#pragma unroll
                                for (int d = seg / 2; d >= 1; d >>= 1)
                                    st.part[m][l] += __shfl_xor_sync(0xffffffffu, st.part[m][l], d);
#pragma unroll
                            for (int sgi = 0; sgi < GPI; ++sgi) {
                                const int gi = it * GPI + sgi;
                                float sc = 0.0f;
                                if (gi < G) sc = mul_rn(qs_s[m * G + gi], __ldg(ws + n * (long)G + gi));
#pragma unroll
                                for (int l = 0; l < 8; ++l) {
                                    int vs = __shfl_sync(0xffffffffu, st.part[m][l], sgi * seg);
                                    if (gi < G) st.cf8[m][l] = fma_rn(__int2float_rn(vs), sc, st.cf8[m][l]);
                                }
                            }
                        }
                    } else {
                        // TILED: whole-group integer sum.
                        int t = 0;
#pragma unroll
                        for (int l = 0; l < 8; ++l) t += st.part[m][l];
#pragma unroll
                        for (int d = seg / 2; d >= 1; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
                        if constexpr (SEGLOG >= 5) {
                            const int gi = it / IPG;
                            float p = mul_rn(__int2float_rn(t), qs_s[m * G + gi]);
                            st.cf[m] = fma_rn(p, __ldg(ws + n * (long)G + gi), st.cf[m]);
                        } else {
#pragma unroll
                            for (int sgi = 0; sgi < GPI; ++sgi) {
                                int ts = __shfl_sync(0xffffffffu, t, sgi * seg);
                                const int gi = it * GPI + sgi;
                                if (gi < G) {
                                    float p = mul_rn(__int2float_rn(ts), qs_s[m * G + gi]);
                                    st.cf[m] = fma_rn(p, __ldg(ws + n * (long)G + gi), st.cf[m]);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int l = 0; l < 8; ++l) st.part[m][l] = 0;
                }
            }
            // ---- row end ----
            if (it == IT - 1) {
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    if (m >= M) continue;
                    float out;
                    if constexpr (LANE) {
                        if constexpr (SEGLOG >= 3) out = seg_reduce8_ref<SEGLOG>(st.cf[m]);
                        else out = reduce8_ref(st.cf8[m]);
                    } else {
                        out = st.cf[m];
                    }
                    if (lane == 0) {
                float *yp = y + (long)m * ldy + n;
                *yp = acc ? add_rn(*yp, out) : out;   // residual add: add_vector order
            }
                }
                reset_row();
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) wbuf[u] = nbuf[u];
    }
}

namespace {

template <int MR, bool LANE, int SEGLOG>
cudaError_t launch_t(const GemvArgs &a, cudaStream_t stream) {
    const int G = a.K / a.g;
    size_t smem = (size_t)MR * a.K * sizeof(int16_t) + (size_t)MR * G * sizeof(float);
    auto kern = gemv_i8_kernel<MR, LANE, SEGLOG>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    int dev = 0, sms = 148, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (per_sm < 1) per_sm = 1;
    long want = (a.N + kWarpsPerBlock - 1) / kWarpsPerBlock;
    long cap = (long)sms * per_sm;
    int grid = (int)(want < cap ? want : cap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a.q, a.qs, a.W, a.ws, a.y, a.M, a.N, a.K, a.g, a.ldy, a.acc);
}

template <int MR, bool LANE>
cudaError_t launch_seg(const GemvArgs &a, cudaStream_t s) {
    const int cpg = a.g / 16;
    switch (cpg >= 32 ? 32 : cpg) {
        case 32: return launch_t<MR, LANE, 5>(a, s);
        case 16: return launch_t<MR, LANE, 4>(a, s);
        case 8: return launch_t<MR, LANE, 3>(a, s);
        case 4: return launch_t<MR, LANE, 2>(a, s);
        case 2: return launch_t<MR, LANE, 1>(a, s);
        case 1: return launch_t<MR, LANE, 0>(a, s);
    }
    return cudaErrorInvalidValue;
}

template <bool LANE>
cudaError_t launch_mr(const GemvArgs &a, cudaStream_t s) {
    if (a.M <= 1) return launch_seg<1, LANE>(a, s);
    if (a.M <= 2) return launch_seg<2, LANE>(a, s);
    if (a.M <= 4) return launch_seg<4, LANE>(a, s);
    return launch_seg<8, LANE>(a, s);
}

}  // namespace

bool gemv_shape_supported(int K, int g) {
    if (g <= 0 || K <= 0 || K % g || g % 16) return false;
    if (g >= 512) return g % 512 == 0;
    return 512 % g == 0;
}

size_t gemv_smem_bytes(int M, int K, int g) {
    int MR = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
    return (size_t)MR * K * 2 + (size_t)MR * (K / g) * 4;
}

cudaError_t launch_gemv_generic(const GemvArgs &a, bool lane8, cudaStream_t stream) {
    return lane8 ? launch_mr<true>(a, stream) : launch_mr<false>(a, stream);
}

}  // namespace qvl
