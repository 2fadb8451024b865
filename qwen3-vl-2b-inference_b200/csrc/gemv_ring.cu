// M=1 INT8 GEMV with per-output-row scales over a weight-streaming ring:
// the decode GEMV of matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:122-224
// (LANE8 order) for the shapes of the text decoder (K = 2048 or 6144).
//
// One CTA per SM.  CTA b owns the 16-row blocks u = b, b + G, ... of W; a
// producer warp copies them (with their 16 scales) through a ring of 6
// 32 KB shared-memory stages with cp.async.bulk (no multicast), starting
// before the programmatic-dependent-launch wait: the weights do not depend on
// the previous kernel, so the HBM stream begins while it finishes.  Compute
// warp w takes row w of every stage; a K = 6144 row spans three stages, its
// int32 lane sums carried across them (exact).  Every wait is bounded.
#include "ring_common.cuh"
#include "qact.cuh"
#include "gemv_ring.cuh"

namespace qvl {

namespace {
using namespace ring;
constexpr int kStagesR = 6;
constexpr int kMaxK = 6144;
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, const volatile int *stop) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!tc::mbar_try_wait(bar, parity)) {
        if ((stop && *stop) || global_ns() - t0 > kWaitNs) return false;
    }
    return true;
}

__global__ void __launch_bounds__(kBlock, 1) gemv_ring_kernel(RingGemvArgs a) {
    extern __shared__ __align__(1024) unsigned char sm[];
    int16_t *q16 = reinterpret_cast<int16_t *>(sm + (size_t)kStagesR * kStageBytes);
    __shared__ __align__(8) uint64_t full_mb[kStagesR], empty_mb[kStagesR];
    __shared__ __align__(16) float scl[kStagesR][kRows];
    __shared__ int stop_flag, prod_done, issued_sh;
    __shared__ float a_s_sh, inv_sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ring = tc::smem_u32(sm), full = tc::smem_u32(full_mb), empty = tc::smem_u32(empty_mb);
    const uint32_t ring_s = tc::smem_u32(&scl[0][0]);
    const int segs = a.K / kSegBytes;
    const int U = a.N / kRows, G = (int)gridDim.x;
    const int my = U > (int)blockIdx.x ? (U - 1 - (int)blockIdx.x) / G + 1 : 0;
    const int total = my * segs;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStagesR; ++i) {
            tc::mbar_init(full + 8 * i, 1);
            tc::mbar_init(empty + 8 * i, kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        stop_flag = 0;
        prod_done = 0;
        issued_sh = 0;
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kWarps) {                    // producer
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            const volatile int *vstop = &stop_flag;
            for (int k = 0; k < total && !*vstop; ++k) {
                const int st = k % kStagesR;
                if (k >= kStagesR && !wait_bounded(empty + 8 * st, ((k / kStagesR) - 1) & 1, vstop)) break;
                const int j = k / segs, s = k - j * segs;
                const size_t row0 = ((size_t)blockIdx.x + (size_t)j * G) * kRows;
                const uint32_t bar = full + 8 * st, dst = ring + (uint32_t)st * kStageBytes;
                tc::mbar_expect_tx(bar, kStageBytes + kRows * 4);
                bulk_g2s(ring_s + (uint32_t)st * kRows * 4, a.Ws + row0, kRows * 4, bar, pol);
                const int8_t *src = a.W + row0 * a.K + (size_t)s * kSegBytes;
                if (segs == 1) {
                    bulk_g2s(dst, src, kStageBytes, bar, pol);
                } else {
#pragma unroll 1
                    for (int r = 0; r < kRows; ++r)
                        bulk_g2s(dst + r * kSegBytes, src + (size_t)r * a.K, kSegBytes, bar, pol);
                }
                *reinterpret_cast<volatile int *>(&issued_sh) = k + 1;
            }
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&prod_done) = 1;
        }
        return;
    }

    // compute warps: the activations are the previous kernel's output
    pdl_wait();
    float a_s;
    if (a.x) {
        // the activation quantisation of the reference's linear() (one group
        // of K), done by every CTA while its weight stages stream in:
        // fp32 row into shared memory, warp 0 forms the scale (the 16-lane
        // fused chain of group_sumsq_ref, both half-warps), all threads quantise
        float *xs = reinterpret_cast<float *>(q16 + a.K);
        for (int i = threadIdx.x; i < a.K / 4; i += kThreads)
            reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(a.x)[i];
        csync();
        if (threadIdx.x < 32) {
            const float ss = group_sumsq_ref(xs, a.K, threadIdx.x & 15);
            const float s = mul_rn(__fsqrt_rn(fma_rn(ss, __fdiv_rn(1.0f, (float)a.K), 1e-6f)), inv127());
            if (threadIdx.x == 0) {
                a_s_sh = s;
                inv_sh = __fdiv_rn(1.0f, s);
            }
        }
        csync();
        const float inv = inv_sh;
        for (int j = threadIdx.x; j < a.K; j += kThreads) q16[j] = quant_one(xs[j], inv);
        a_s = a_s_sh;
    } else {
        for (int i = threadIdx.x; i < a.K / 8; i += kThreads)
            reinterpret_cast<int4 *>(q16)[i] = reinterpret_cast<const int4 *>(a.q)[i];
        a_s = a.qs[0];
    }
    csync();
    const int4 *q_s = reinterpret_cast<const int4 *>(q16);
    Act act;
    if (segs == 1) load_act(q_s, 0, lane, act);
    bool failed = false;
    int k = 0;
    for (int j = 0; j < my; ++j) {
        const int n = ((int)blockIdx.x + j * G) * kRows + warp;
        int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float ws = 0.0f;
        for (int s = 0; s < segs; ++s, ++k) {
            const int st = k % kStagesR;
            if (!failed) failed = !__any_sync(0xffffffffu, wait_bounded(full + 8 * st, (k / kStagesR) & 1, nullptr));
            if (!failed) {
                if (segs > 1) load_act(q_s, s * (kSegBytes / 16), lane, act);
                madd_seg(sm + (size_t)st * kStageBytes, warp, lane, act, p);
                ws = scl[st][warp];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * st);
        }
        const float out = finish_row(p, a_s, ws, lane);
        if (lane == 0 && !failed) a.y[n] = a.acc ? add_rn(a.y[n], out) : out;
    }
    if (failed) {
        // leave only after the copies already issued have landed (bounded)
        csync();
        if (threadIdx.x == 0) {
            *reinterpret_cast<volatile int *>(&stop_flag) = 1;
            const unsigned long long t0 = global_ns();
            while (*reinterpret_cast<volatile int *>(&prod_done) == 0 && global_ns() - t0 < kWaitNs) {
            }
            const int issued = *reinterpret_cast<volatile int *>(&issued_sh);
            for (int i = max(0, issued - kStagesR); i < issued; ++i)
                wait_bounded(full + 8 * (i % kStagesR), (i / kStagesR) & 1, nullptr);
        }
    }
}

size_t ring_smem_bytes(int K, bool fused) {
    return (size_t)kStagesR * kStageBytes + (size_t)K * sizeof(int16_t) + (fused ? (size_t)K * sizeof(float) : 0);
}

int ring_grid(int N) {
    static int sms[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev < 64 && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int n_sm = dev < 64 ? sms[dev] : 148;
    const int units = N / kRows;
    return units < n_sm ? units : n_sm;
}

}  // namespace

bool gemv_ring_supported(const RingGemvArgs &a) {
    if (a.x ? (a.K > kRingFusedMaxK || ((uintptr_t)a.x & 15)) : ((uintptr_t)a.q & 15) != 0) return false;
    return a.N >= kRows && a.N % kRows == 0 && a.K >= kSegBytes && a.K % kSegBytes == 0 && a.K <= kMaxK &&
           ((uintptr_t)a.W & 15) == 0 && ((uintptr_t)a.Ws & 15) == 0;
}

cudaError_t launch_gemv_ring(const RingGemvArgs &a, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        const size_t mx = ring_smem_bytes(kMaxK, false) > ring_smem_bytes(kRingFusedMaxK, true)
                              ? ring_smem_bytes(kMaxK, false) : ring_smem_bytes(kRingFusedMaxK, true);
        cudaError_t e = cudaFuncSetAttribute(gemv_ring_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mx);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ring_grid(a.N));
    cfg.blockDim = dim3(kBlock);
    cfg.dynamicSmemBytes = ring_smem_bytes(a.K, a.x != nullptr);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_ring_kernel, a);
}

}  // namespace qvl
