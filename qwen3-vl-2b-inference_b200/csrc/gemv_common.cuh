// Shared pieces of the decode GEMV kernels (gemv_i8.cu, gemv_i8_generic.cu).
#pragma once
#include "common.cuh"
#include "gemv_i8.cuh"

namespace qvl {
namespace {

constexpr int kThreads = 256;
constexpr int kWarpsPerBlock = kThreads / kWarp;
constexpr int kUnroll = 4;  // steps in flight per warp (4 x 16 B per lane)

// 8 int32 madd lanes of one 16-byte weight chunk against 16 int16 activations.
__device__ __forceinline__ void madd_chunk(const uint4 &w, const int4 &a0, const int4 &a1,
                                           int p[8]) {
    p[0] = dp2a_lo(a0.x, (int)w.x, p[0]);
    p[1] = dp2a_hi(a0.y, (int)w.x, p[1]);
    p[2] = dp2a_lo(a0.z, (int)w.y, p[2]);
    p[3] = dp2a_hi(a0.w, (int)w.y, p[3]);
    p[4] = dp2a_lo(a1.x, (int)w.z, p[4]);
    p[5] = dp2a_hi(a1.y, (int)w.z, p[5]);
    p[6] = dp2a_lo(a1.z, (int)w.w, p[6]);
    p[7] = dp2a_hi(a1.w, (int)w.w, p[7]);
}

// Transposing butterfly over a segment of 2^SEGLOG lanes (SEGLOG >= 3):
// returns the segment total of lane index lane_id(), with
// lane_id = 4*bit(seg/2) + 2*bit(seg/4) + bit(seg/8) of the position.
template <int SEGLOG>
__device__ __forceinline__ int seg_transpose_reduce(int v[8], int lane) {
    constexpr int seg = 1 << SEGLOG;
    const unsigned full = 0xffffffffu;
    {
        constexpr int d = seg / 2;
        const bool up = lane & d;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int send = up ? v[i] : v[i + 4];
            int keep = up ? v[i + 4] : v[i];
            v[i] = keep + __shfl_xor_sync(full, send, d);
        }
    }
    {
        constexpr int d = seg / 4;
        const bool up = lane & d;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            int send = up ? v[i] : v[i + 2];
            int keep = up ? v[i + 2] : v[i];
            v[i] = keep + __shfl_xor_sync(full, send, d);
        }
    }
    int r;
    {
        constexpr int d = seg / 8;
        const bool up = lane & d;
        int send = up ? v[0] : v[1];
        int keep = up ? v[1] : v[0];
        r = keep + __shfl_xor_sync(full, send, d);
    }
#pragma unroll
    for (int d = seg / 16; d >= 1; d >>= 1) r += __shfl_xor_sync(full, r, d);
    return r;
}

template <int SEGLOG>
__device__ __forceinline__ int seg_lane_id(int lane) {
    constexpr int seg = 1 << SEGLOG;
    return ((lane & (seg / 2)) ? 4 : 0) + ((lane & (seg / 4)) ? 2 : 0) + ((lane & (seg / 8)) ? 1 : 0);
}

// Final reduce8 of per-lane accumulators held one per thread (seg >= 8):
// u_l = cf_l + cf_{l+4}; (u0+u1) + (u2+u3).  fp32 addition is commutative,
// so the partner order does not matter; the association does and is kept.
template <int SEGLOG>
__device__ __forceinline__ float seg_reduce8_ref(float cf) {
    constexpr int seg = 1 << SEGLOG;
    const unsigned full = 0xffffffffu;
    float u = add_rn(cf, __shfl_xor_sync(full, cf, seg / 2));
    float p = add_rn(u, __shfl_xor_sync(full, u, seg / 8));
    return add_rn(p, __shfl_xor_sync(full, p, seg / 4));
}

template <int MR, bool LANE, int SEGLOG>
struct RowState {
    int part[MR][8];
    float cf[MR];                    // LANE, seg >= 8: this thread's lane accumulator
    float cf8[(SEGLOG < 3) ? MR : 1][8];  // LANE, seg < 8: all 8 lanes in-thread
};

}  // namespace

cudaError_t launch_gemv_generic(const GemvArgs &a, bool lane8, cudaStream_t stream);

}  // namespace qvl
