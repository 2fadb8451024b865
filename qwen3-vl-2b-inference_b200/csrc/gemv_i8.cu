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
#include "tail.cuh"

namespace qvl {

// ---------------------------------------------------------------------------
// Fast path: M <= 4 rows, g >= 128 (segments of >= 8 lanes), K <= 12*512,
// K/g <= 64.  Every lane issues all IT 16-byte loads of its warp's row at
// once (one 512-byte step per load), plus the row's weight scales, before
// touching any of them, so a single wave of warps keeps the decode-shape
// matrices in flight.  Rows are walked with pointer increments only; when
// IT <= 4 the next row's loads are issued before the current row is reduced.
template <int MR, int IT>
constexpr int fast_min_blocks() { return (MR == 1 && IT <= 4) ? 6 : 1; }

template <int MR, bool LANE, int IT>
__global__ void __launch_bounds__(kThreads, fast_min_blocks<MR, IT>())
gemv_i8_fast_kernel(const int16_t *__restrict q, const float *__restrict qs, GemvSegs sg,
                    int M, int N, int K, int g, int acc, int seglog, int pair, RowTail tail) {
    extern __shared__ __align__(16) unsigned char smem[];
    int16_t *q_s = reinterpret_cast<int16_t *>(smem);
    const int G = K / g;
    float *qs_s = reinterpret_cast<float *>(smem + (size_t)MR * K * sizeof(int16_t));

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = gridDim.x * kWarpsPerBlock;
    const int NCH = K / 16;
    const int seg = 1 << seglog;
    const int IPG = (seg == 32) ? (g >> 9) : 1;   // steps per group (g >= 512)
    const int GPI = 32 >> seglog;                  // groups per step (g < 512)
    // One wave covers the decode shapes at M=1, so the register budget goes to
    // occupancy there; otherwise the next row's loads are double-buffered.
    constexpr bool kDouble = IT <= 4 && MR > 1;

    // pair = 1 (gate/up with SwiGLU epilogue): virtual rows 2p (segment 0,
    // gate row p) and 2p+1 (segment 1, up row p) go to the same warp, one
    // after the other, and the warp writes swiglu(gate, up) into segment 0.
    const int wid = blockIdx.x * kWarpsPerBlock + warp;
    int n = pair ? 2 * wid : wid;
    auto next_row = [&](int r) { return pair ? ((r & 1) ? r - 1 + 2 * nwarps : r + 1) : r + nwarps; };
    uint4 wr[IT];
    float wsr[2];
    auto issue = [&](int row, uint4 *dst, float *sdst) {
        const int sid = pair ? (row & 1) : sg.seg_of(row);
        const int lr = pair ? (row >> 1) : row - sg.start(sid);
        const int8_t *W = sg.w_of(sid);
        const float *ws = sg.ws_of(sid) + (long)lr * G;
        const uint4 *base = reinterpret_cast<const uint4 *>(W + (long)lr * K) + lane;
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            const int c = it * 32 + lane;
            dst[it] = (c < NCH) ? ld_stream_v4(base + it * 32) : make_uint4(0, 0, 0, 0);
        }
        sdst[0] = (lane < G) ? __ldg(ws + lane) : 0.0f;
        sdst[1] = (lane + 32 < G) ? __ldg(ws + lane + 32) : 0.0f;
    };
    if (n < N) issue(n, wr, wsr);
    // the fused tail's constant operands (norm weight row and its scales) are
    // pulled into L2 now, off the serial path of the last CTA
    if (tail.counter && tail.wq && blockIdx.x == 0) {
        for (int i = threadIdx.x * 128; i < tail.H; i += kThreads * 128) prefetch_l2(tail.wq + i);
        if (threadIdx.x == 0) prefetch_l2(tail.ws);
    }

    pdl_launch_dependents();
    pdl_wait();
    {
        const int nq16 = M * K / 8;
        const int4 *src = reinterpret_cast<const int4 *>(q);
        int4 *dst = reinterpret_cast<int4 *>(q_s);
        for (int i = threadIdx.x; i < nq16; i += kThreads) dst[i] = src[i];
        for (int i = threadIdx.x; i < M * G; i += kThreads) qs_s[i] = qs[i];
        __syncthreads();
    }

    const unsigned full = 0xffffffffu;
    const int pos = lane & (seg - 1);
    const int d1 = seg >> 1, d2 = seg >> 2, d3 = seg >> 3;   // transposing-butterfly distances

    float gate_v[MR];
    for (; n < N; n = next_row(n)) {
        uint4 nx[kDouble ? IT : 1];
        float nws[2] = {0.0f, 0.0f};
        const int nn = next_row(n);
        if constexpr (kDouble) {
            if (nn < N) issue(nn, nx, nws);
        }
        float cf[MR];
        int part[MR][8];
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            cf[m] = 0.0f;
#pragma unroll
            for (int l = 0; l < 8; ++l) part[m][l] = 0;
        }
#pragma unroll
        for (int it = 0; it < IT; ++it) {
            if (it * 32 >= NCH) break;
            const int c = it * 32 + lane;
            const int cc = (c < NCH) ? c : 0;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                if (m < M) {
                    const int4 *ap = reinterpret_cast<const int4 *>(q_s + (size_t)m * K + cc * 16);
                    madd_chunk(wr[it], ap[0], ap[1], part[m]);
                }
            }
            const bool group_end = (seg == 32) ? ((it + 1) % IPG == 0) : true;
            if (!group_end) continue;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                if (m >= M) continue;
                if constexpr (LANE) {
                    int v[8];
#pragma unroll
                    for (int l = 0; l < 8; ++l) v[l] = part[m][l];
                    bool up = lane & d1;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        int send = up ? v[i] : v[i + 4];
                        int keep = up ? v[i + 4] : v[i];
                        v[i] = keep + __shfl_xor_sync(full, send, d1);
                    }
                    up = lane & d2;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        int send = up ? v[i] : v[i + 2];
                        int keep = up ? v[i + 2] : v[i];
                        v[i] = keep + __shfl_xor_sync(full, send, d2);
                    }
                    up = lane & d3;
                    int r = (up ? v[1] : v[0]) + __shfl_xor_sync(full, up ? v[0] : v[1], d3);
                    for (int d = seg >> 4; d >= 1; d >>= 1) r += __shfl_xor_sync(full, r, d);
                    if (seg == 32) {
                        const int gi = it / IPG;
                        const float wsv = __shfl_sync(full, (gi >> 5) ? wsr[1] : wsr[0], gi & 31);
                        cf[m] = fma_rn(__int2float_rn(r), mul_rn(qs_s[m * G + gi], wsv), cf[m]);
                    } else {
                        for (int sgi = 0; sgi < GPI; ++sgi) {
                            const int vs = __shfl_sync(full, r, sgi * seg + pos);
                            const int gi = it * GPI + sgi;
                            const float wsv = __shfl_sync(full, ((gi >> 5) & 1) ? wsr[1] : wsr[0], gi & 31);
                            if (gi < G) cf[m] = fma_rn(__int2float_rn(vs), mul_rn(qs_s[m * G + gi], wsv), cf[m]);
                        }
                    }
                } else {
                    int t = 0;
#pragma unroll
                    for (int l = 0; l < 8; ++l) t += part[m][l];
                    for (int d = seg >> 1; d >= 1; d >>= 1) t += __shfl_xor_sync(full, t, d);
                    if (seg == 32) {
                        const int gi = it / IPG;
                        const float wsv = __shfl_sync(full, (gi >> 5) ? wsr[1] : wsr[0], gi & 31);
                        cf[m] = fma_rn(mul_rn(__int2float_rn(t), qs_s[m * G + gi]), wsv, cf[m]);
                    } else {
                        for (int sgi = 0; sgi < GPI; ++sgi) {
                            const int ts = __shfl_sync(full, t, sgi * seg);
                            const int gi = it * GPI + sgi;
                            const float wsv = __shfl_sync(full, ((gi >> 5) & 1) ? wsr[1] : wsr[0], gi & 31);
                            if (gi < G) cf[m] = fma_rn(mul_rn(__int2float_rn(ts), qs_s[m * G + gi]), wsv, cf[m]);
                        }
                    }
                }
#pragma unroll
                for (int l = 0; l < 8; ++l) part[m][l] = 0;
            }
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m >= M) continue;
            float out = cf[m];
            if constexpr (LANE) {
                // (l, l+4) pairs, then (u0+u1) + (u2+u3): partners at d1, d3, d2
                float u = add_rn(out, __shfl_xor_sync(full, out, d1));
                float p = add_rn(u, __shfl_xor_sync(full, u, d3));
                out = add_rn(p, __shfl_xor_sync(full, p, d2));
            }
            if (pair) {
                if ((n & 1) == 0) {
                    gate_v[m] = out;
                } else if (lane == 0) {
                    sg.y[0][(long)m * sg.ldy[0] + (n >> 1)] = swiglu_one(gate_v[m], out);
                }
            } else if (lane == 0) {
                const int sid = sg.seg_of(n);
                float *yp = sg.y_of(sid) + (long)m * sg.ldy_of(sid) + (n - sg.start(sid));
                *yp = acc ? add_rn(*yp, out) : out;   // residual add: add_vector order
            }
        }
        if constexpr (kDouble) {
#pragma unroll
            for (int it = 0; it < IT; ++it) wr[it] = nx[it];
            wsr[0] = nws[0];
            wsr[1] = nws[1];
        } else {
            if (nn < N) issue(nn, wr, wsr);
        }
    }
    if (tail.counter) run_row_tail(tail, smem);   // last CTA: RMSNorm / quantisation of the finished rows
}

namespace {
template <int MR, bool LANE, int IT>
cudaError_t launch_fast_t(const GemvArgs &a, cudaStream_t stream) {
    const int G = a.K / a.g;
    size_t smem = (size_t)MR * a.K * sizeof(int16_t) + (size_t)MR * G * sizeof(float);
    if (a.tail.counter && row_tail_smem(a.tail.H, a.tail.wq) > smem) smem = row_tail_smem(a.tail.H, a.tail.wq);
    auto kern = gemv_i8_fast_kernel<MR, LANE, IT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    int dev = 0, sms = 148, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (per_sm < 1) per_sm = 1;
    const long total_rows = a.segs.nseg ? a.segs.total() : a.N;
    long want = (total_rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
    long cap = (long)sms * per_sm;
    int grid = (int)(want < cap ? want : cap);
    const int cpg = a.g / 16;
    int seglog = 0;
    while ((1 << seglog) < (cpg < 32 ? cpg : 32)) ++seglog;
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
    GemvSegs sg = a.segs;
    if (sg.nseg == 0) sg = GemvSegs::single(a.W, a.ws, a.y, a.N, a.ldy);
    return cudaLaunchKernelEx(&cfg, kern, a.q, a.qs, sg, a.M, sg.total(), a.K, a.g, a.acc, seglog, a.pair,
                              a.tail);
}

template <int MR, bool LANE>
cudaError_t launch_fast_it(const GemvArgs &a, cudaStream_t s) {
    const int it = (a.K + 511) / 512;
    if (it <= 1) return launch_fast_t<MR, LANE, 1>(a, s);
    if (it <= 2) return launch_fast_t<MR, LANE, 2>(a, s);
    if (it <= 4) return launch_fast_t<MR, LANE, 4>(a, s);
    if (it <= 8) return launch_fast_t<MR, LANE, 8>(a, s);
    return launch_fast_t<MR, LANE, 12>(a, s);
}

template <bool LANE>
cudaError_t launch_fast_mr(const GemvArgs &a, cudaStream_t s) {
    if (a.M <= 1) return launch_fast_it<1, LANE>(a, s);
    if (a.M <= 2) return launch_fast_it<2, LANE>(a, s);
    return launch_fast_it<4, LANE>(a, s);
}
}  // namespace

bool gemv_fast_eligible(int M, int K, int g) {
    return M <= 4 && g >= 128 && K <= 12 * 512 && (K / g) <= 64 && gemv_shape_supported(K, g);
}

cudaError_t launch_gemv_i8(const GemvArgs &a, bool lane8, cudaStream_t stream) {
    if (gemv_fast_eligible(a.M, a.K, a.g))
        return lane8 ? launch_fast_mr<true>(a, stream) : launch_fast_mr<false>(a, stream);
    return launch_gemv_generic(a, lane8, stream);
}


}  // namespace qvl
