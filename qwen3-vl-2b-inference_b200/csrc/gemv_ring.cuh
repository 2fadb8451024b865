#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace qvl {

// y[0, 0..N) (=, or += with acc) from one row of pre-quantised int16
// activations (one scale: group size K) and per-output-row INT8 weights,
// in the reference's M=1 8-lane order.  Weights stream through a shared-
// memory ring of bulk asynchronous copies fed by a producer warp.
struct RingGemvArgs {
    const int16_t *q;     // [K]
    const float *qs;      // [1]
    const int8_t *W;      // [N, K]
    const float *Ws;      // [N]
    float *y;             // [N]
    int N, K, acc;
    // fp32 activations [K] to quantise inside the kernel (the reference's
    // per-row activation quantisation, group K) instead of q / qs; K <= 4096
    const float *x = nullptr;
};

// Shapes the ring GEMV takes: N a multiple of 16, K a multiple of 2048 up to
// 6144, 16-byte aligned weights and scales.
bool gemv_ring_supported(const RingGemvArgs &a);
constexpr int kRingFusedMaxK = 4096;
cudaError_t launch_gemv_ring(const RingGemvArgs &a, cudaStream_t st);

}  // namespace qvl
