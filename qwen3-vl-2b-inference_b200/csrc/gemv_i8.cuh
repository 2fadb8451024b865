#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>
#include "tail.cuh"

namespace qvl {

// Up to three weight matrices sharing one activation row set (q/k/v, or
// gate/up), walked as one concatenated row range by a single launch.
struct GemvSegs {
    const int8_t *W[3];
    const float *ws[3];
    float *y[3];
    long ldy[3];
    int end[3];   // cumulative row counts
    int nseg;
    __host__ __device__ int total() const { return end[nseg - 1]; }
    __device__ int seg_of(int row) const { return (row >= end[0]) + (nseg > 2 && row >= end[1]); }
    __device__ int start(int s) const { return s == 0 ? 0 : (s == 1 ? end[0] : end[1]); }
    __device__ const int8_t *w_of(int s) const { return s == 0 ? W[0] : (s == 1 ? W[1] : W[2]); }
    __device__ const float *ws_of(int s) const { return s == 0 ? ws[0] : (s == 1 ? ws[1] : ws[2]); }
    __device__ float *y_of(int s) const { return s == 0 ? y[0] : (s == 1 ? y[1] : y[2]); }
    __device__ long ldy_of(int s) const { return s == 0 ? ldy[0] : (s == 1 ? ldy[1] : ldy[2]); }
    static GemvSegs single(const int8_t *W0, const float *ws0, float *y0, int N, long ldy0) {
        GemvSegs g = {};
        g.W[0] = W0; g.ws[0] = ws0; g.y[0] = y0; g.ldy[0] = ldy0; g.end[0] = N; g.end[1] = g.end[2] = N;
        g.nseg = 1;
        return g;
    }
};

struct GemvArgs {
    const int16_t *q;   // [M, K] quantised activations
    const float *qs;    // [M, K/g] activation scales
    const int8_t *W;    // [N, K]
    const float *ws;    // [N * K/g]
    float *y;           // [M, ldy]
    int M, N, K, g;
    long ldy;
    int acc;            // 1: y += result (fused residual add), 0: y = result
    GemvSegs segs;      // nseg > 0: several matrices (fast path only); W/ws/y/N unused
    int pair;           // segs = {gate, up} of equal rows: y0 = swiglu(gate, up) (fast path only)
    RowTail tail;       // tail.counter != nullptr: fused RMSNorm / quantisation (fast path only)
};

bool gemv_shape_supported(int K, int g);
bool gemv_fast_eligible(int M, int K, int g);
size_t gemv_smem_bytes(int M, int K, int g);
// M <= 8 rows; lane8 selects the M=1 decode summation order.
cudaError_t launch_gemv_i8(const GemvArgs &a, bool lane8, cudaStream_t stream);

}  // namespace qvl
