// Shared pieces of the weight-ring kernels (decode_persistent.cu,
// gemv_ring.cu): 16 compute warps, each owning row w of every 32 KB stage
// (16 row segments of 2048 int8), a producer warp issuing bulk asynchronous
// copies (cp.async.bulk, no multicast) into a ring of stages, and the M=1
// GEMV arithmetic of one row segment in the reference's 8-lane order.
#pragma once
#include <cstdint>
#include "common.cuh"
#include "gemv_common.cuh"
#include "tc_common.cuh"

namespace qvl {
namespace ring {

constexpr int kThreads = 512;                  // compute threads (16 warps)
constexpr int kWarps = kThreads / 32;
constexpr int kBlock = kThreads + 32;          // + one producer warp
constexpr int kRows = kWarps;                  // rows per stage: one per compute warp
constexpr int kSegBytes = 2048;                // bytes of a row (segment) per stage
constexpr int kStageBytes = kRows * kSegBytes;

// Barrier of the 16 compute warps only (named barrier 1); the producer warp
// never joins it.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// This lane's activation chunks [cbase, cbase + 128) of q_s (int16 pairs),
// held in registers for every row of a phase.
struct Act {
    int4 a[8];
};
__device__ __forceinline__ void load_act(const int4 *q_s, int cbase, int lane, Act &act) {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int c = cbase + it * 32 + lane;
        act.a[2 * it] = q_s[2 * c];
        act.a[2 * it + 1] = q_s[2 * c + 1];
    }
}

// int32 lane sums of one 2048-byte row segment (this warp's row of a stage)
// against the register-held activation chunks.
__device__ __forceinline__ void madd_seg(const unsigned char *stage, int warp, int lane, const Act &act, int p[8]) {
    const uint4 *row = reinterpret_cast<const uint4 *>(stage + warp * kSegBytes);
    uint4 w[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) w[it] = row[it * 32 + lane];
#pragma unroll
    for (int it = 0; it < 4; ++it) madd_chunk(w[it], act.a[2 * it], act.a[2 * it + 1], p);
}

// Row result from the int32 lane sums, in the reference's 8-lane order
// (cpu_f32a_i8f32sb_f32c_avx2.cpp:181-223): lane sums reduced over the warp,
// each lane's sum scaled (one group: the whole row), lanes added pairwise.
// Valid in all lanes.
__device__ __forceinline__ float finish_row(int (&p)[8], float a_s, float w_s, int lane) {
    const unsigned full = 0xffffffffu;
    bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int send = up ? p[i] : p[i + 4];
        int keep = up ? p[i + 4] : p[i];
        p[i] = keep + __shfl_xor_sync(full, send, 16);
    }
    up = lane & 8;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        int send = up ? p[i] : p[i + 2];
        int keep = up ? p[i + 2] : p[i];
        p[i] = keep + __shfl_xor_sync(full, send, 8);
    }
    up = lane & 4;
    int r = (up ? p[1] : p[0]) + __shfl_xor_sync(full, up ? p[0] : p[1], 4);
    r += __shfl_xor_sync(full, r, 2);
    r += __shfl_xor_sync(full, r, 1);
    const float cf = fma_rn(__int2float_rn(r), mul_rn(a_s, w_s), 0.0f);
    const float u = add_rn(cf, __shfl_xor_sync(full, cf, 16));
    const float pp = add_rn(u, __shfl_xor_sync(full, u, 4));
    return add_rn(pp, __shfl_xor_sync(full, pp, 8));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

}  // namespace ring
}  // namespace qvl
