// One decode token of the whole Qwen3-VL-2B text decoder (28 layers, LM head,
// greedy decode) in ONE persistent, cooperatively launched kernel, for a
// single request with per-output-row INT8 weights.
//
// Why: at batch 1 the step is a chain of small dependent operations (see
// forward_text, model/src/forward.cpp:458-720); as separate launches each
// costs >= 2.3 us of hand-off plus its own latency, and the weight stream
// stops at every hand-off.  Here every CTA stays resident, the phases are
// separated by a grid-wide barrier, and the weights never wait for them:
//
//   * Weight stream.  Every weight row the token needs is known in advance.
//     Each CTA owns a fixed list of 16-row blocks of every matrix (block
//     u = blockIdx.x + j * gridDim.x) and streams them, in the order it will
//     use them, through a ring of kStages 32 KB shared-memory stages with
//     bulk asynchronous copies (cp.async.bulk, completion on an mbarrier, no
//     multicast).  One thread keeps the ring full, so while the grid waits
//     at a barrier or computes attention, the next matrices are already
//     flowing from HBM.  Warp w computes row w of every stage.
//   * Small row operations (RMSNorm + quantisation, attention combine +
//     quantisation) are computed redundantly by every CTA from L2 instead
//     of by one CTA plus another barrier.
//
// Arithmetic is the multi-kernel path's, operation by operation (M=1 GEMV
// lane order with exact int32 lane sums, reference RMSNorm / quantisation /
// SwiGLU / RoPE / softmax rules); only the attention's split of the context
// (16 slices per KV head) changes fp32 summation order there.
//
// Safety: every wait (grid barrier, mbarrier) is bounded by the global timer;
// a timeout sets the abort flag, after which every CTA drains its own copies
// in flight (bounded) and leaves at its next barrier.  The launch is
// cooperative, so all CTAs are co-resident (the launch fails instead of
// deadlocking if they cannot be).
#include <cfloat>
#include <climits>
#include <cuda_fp16.h>
#include "gemv_common.cuh"
#include "tail.cuh"
#include "tc_common.cuh"
#include "ring_common.cuh"
#include "decode_persistent.cuh"

namespace qvl {

namespace {
using namespace ring;
constexpr int kPThreads = ring::kThreads;      // compute threads (16 warps)
constexpr int kPWarps = ring::kWarps;
constexpr int H = 2048, I = 6144, NH = 16, NKV = 8, D = 128;
constexpr int kSlices = kPersistSlices;        // attention context slices per KV head
constexpr int kSliceMax = 512;                 // tokens per slice (context <= 8192)
constexpr int kOrdChunk = 1024;               // positions staged per pass in reference-order attention
constexpr int kMaxPages = kSlices * kSliceMax / 16;   // page table entries (page_size >= 16)
constexpr unsigned long long kBarrierLimitNs = 2000000000ull;
constexpr unsigned kTraceSlots = kPersistTraceSlots;

// weight ring: kStages stages of 16 row segments of 2048 bytes, one per warp
constexpr int kStages = 5;

// dynamic shared memory: ring | q16 [I] int16 | xs [I] f32 | ts [H] f32 | sp [2][kSliceMax] f32 |
// nrm_w [H] f32 | nrm_s [H / norm_group] f32 (norm_group >= 16)
constexpr size_t kRingBytes = (size_t)kStages * kStageBytes;
constexpr size_t kSmemBytes = kRingBytes + (size_t)I * 2 + (size_t)I * 4 + (size_t)H * 4 + 2 * (size_t)kSliceMax * 4 +
                              (size_t)H * 4 + (size_t)H * 4 / 16;

// matrices in stream order; units are 16-row blocks, subs the stages per unit
enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_LM = 4, PH_DONE = 5 };
__device__ __forceinline__ int ph_units(int ph, int vocab) {
    return ph == PH_QKV ? (NH * D + 2 * NKV * D) / kRows
         : ph == PH_O ? H / kRows
         : ph == PH_GU ? I / kRows
         : ph == PH_DOWN ? H / kRows
         : vocab / kRows;
}
__device__ __forceinline__ int ph_subs(int ph) { return ph == PH_GU ? 2 : ph == PH_DOWN ? I / kSegBytes : 1; }
// units u = blockIdx.x + j * gridDim.x below U
__device__ __forceinline__ int cta_units(int U) {
    return U > (int)blockIdx.x ? (U - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
}

__device__ __forceinline__ unsigned ld_volatile(const unsigned *p) {
    return *reinterpret_cast<const volatile unsigned *>(p);
}
// Grid barrier with a bounded wait.  The counter only grows (it is zero
// when the workspace is cleared), so barrier k of a launch completes when
// the arrivals reach base + (k + 1) * gridDim.x, base being the counter at
// kernel entry rounded down to a multiple of gridDim.x: no reset, no second
// word, and the arrival is a fire-and-forget reduction (no reply to wait
// for).  Release on arrival / acquire on the wait, each after / before a CTA
// barrier (the CTA's writes are ordered by bar.sync, then published by the
// release).  Returns false if the wait gave up or another CTA aborted.
// CTA 0 records the time each barrier opens in S.trace[1 + k].
// Barrier of the kSlices CTAs of one KV head (the softmax needs the maximum
// over the head's slices only); same counter scheme as the grid barrier.
__device__ __forceinline__ bool head_sync(const PersistState &S, int kvh, unsigned long long &target) {
    csync();
    __shared__ int ok;
    if (threadIdx.x == 0) {
        // arrive without waiting for the atomic's reply: the target is known
        // (this CTA's count of head barriers so far, from the base read at entry)
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(S.head_bar + kvh) : "memory");
        target += kSlices;
        unsigned long long v;
        int good = 1;
        const unsigned long long t0 = global_ns();
        for (unsigned it = 1;; ++it) {
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(S.head_bar + kvh) : "memory");
            if (v >= target) break;
            if ((it & 15) == 0) {
                if (ld_volatile(reinterpret_cast<const unsigned *>(S.abort_flag))) { good = 0; break; }
                if (global_ns() - t0 > kBarrierLimitNs) {
                    atomicExch(S.abort_flag, 1);
                    good = 0;
                    break;
                }
            }
        }
        ok = good;
    }
    csync();
    return ok;
}

// Split into arrive and wait so that a CTA can load constants of the next
// phase (norm weights, RoPE row) while the barrier completes.
__device__ __forceinline__ void grid_arrive(const PersistState &S, unsigned long long &target) {
    csync();
    if (threadIdx.x == 0) {
        // no reply needed: the completing count is this CTA's previous target
        // plus the grid size (the base was read at kernel entry)
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(S.bar_count) : "memory");
        target += gridDim.x;
    }
}
__device__ __forceinline__ bool grid_wait(const PersistState &S, unsigned long long target, int &nsync) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        unsigned long long v;
        int good = 1;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(S.bar_count) : "memory");
        if (v < target) {
            const unsigned long long t0 = global_ns();
            for (unsigned it = 1;; ++it) {
                asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(S.bar_count) : "memory");
                if (v >= target) break;
                if ((it & 15) == 0) {
                    if (ld_volatile(reinterpret_cast<const unsigned *>(S.abort_flag))) { good = 0; break; }
                    if (global_ns() - t0 > kBarrierLimitNs) {
                        atomicExch(S.abort_flag, 1);
                        good = 0;
                        break;
                    }
                }
            }
        }
        ok = good;
        if (blockIdx.x == 0 && (unsigned)nsync + 1 < kTraceSlots) S.trace[nsync + 1] = global_ns();
    }
    ++nsync;
    csync();
    return ok;
}

__device__ __forceinline__ void h8f(const uint4 &v, float f[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 x = __half22float2(h[i]);
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
    }
}

// pt: the page table, staged in shared memory
__device__ __forceinline__ size_t kv_off(const PersistState &S, const int *pt, int layer, int t, int kvh) {
    const int page = pt[t / S.page_size];
    const int slot = t - (t / S.page_size) * S.page_size;
    return (size_t)layer * S.kv_layer_stride + (((size_t)page * NKV + kvh) * S.page_size + slot) * D;
}

// Position in this CTA's stream: layer, matrix phase, unit index j, stage s.
struct Cursor {
    int l, ph, j, s;
};

// Skip phases in which this CTA owns no unit.
// cnt[ph]: this CTA's unit count of each matrix phase.
__device__ __forceinline__ void cursor_settle(Cursor &c, int layers, const int *cnt) {
    while (c.ph != PH_DONE && cnt[c.ph] == 0) {
        if (c.ph < PH_DOWN) ++c.ph;
        else if (c.ph == PH_DOWN) { if (c.l + 1 < layers) { ++c.l; c.ph = PH_QKV; } else c.ph = PH_LM; }
        else c.ph = PH_DONE;
    }
}
__device__ __forceinline__ void cursor_next(Cursor &c, int layers, const int *cnt) {
    if (++c.s < ph_subs(c.ph)) return;
    c.s = 0;
    if (++c.j < cnt[c.ph]) return;
    c.j = 0;
    if (c.ph < PH_DOWN) ++c.ph;
    else if (c.ph == PH_DOWN) { if (c.l + 1 < layers) { ++c.l; c.ph = PH_QKV; } else c.ph = PH_LM; }
    else c.ph = PH_DONE;
    cursor_settle(c, layers, cnt);
}

// Global address of the first row segment of stage (c) and the row stride.
__device__ __forceinline__ const int8_t *cursor_src(const Cursor &c, const PersistWeights &W, size_t &stride) {
    const int u = (int)blockIdx.x + c.j * (int)gridDim.x;
    const size_t l = (size_t)c.l;
    stride = H;
    switch (c.ph) {
    case PH_QKV: {
        const int r = u * kRows;
        if (r < NH * D) return W.wq + (l * NH * D + r) * H;
        if (r < NH * D + NKV * D) return W.wk + (l * NKV * D + (r - NH * D)) * H;
        return W.wv + (l * NKV * D + (r - NH * D - NKV * D)) * H;
    }
    case PH_O: return W.wo + (l * H + (size_t)u * kRows) * H;
    case PH_GU: return (c.s == 0 ? W.wg : W.wu) + (l * I + (size_t)u * kRows) * H;
    case PH_DOWN: stride = I; return W.wd + (l * H + (size_t)u * kRows) * I + (size_t)c.s * kSegBytes;
    default: return W.embed + (size_t)u * kRows * H;
    }
}

// Global address of the 16 per-row scales of stage (c) (64 contiguous bytes).
__device__ __forceinline__ const float *cursor_scales(const Cursor &c, const PersistWeights &W) {
    const int u = (int)blockIdx.x + c.j * (int)gridDim.x;
    const size_t l = (size_t)c.l, r = (size_t)u * kRows;
    switch (c.ph) {
    case PH_QKV:
        if (r < (size_t)NH * D) return W.sq + l * NH * D + r;
        if (r < (size_t)NH * D + NKV * D) return W.sk + l * NKV * D + (r - NH * D);
        return W.sv + l * NKV * D + (r - NH * D - NKV * D);
    case PH_O: return W.so + l * H + r;
    case PH_GU: return (c.s == 0 ? W.sg : W.su) + l * I + r;
    case PH_DOWN: return W.sd + l * H + r;
    default: return W.embed_s + r;
    }
}

// Ring state, in shared memory: the next stage to issue and its place in
// the stream.
struct Producer {
    Cursor c;
    int cnt[PH_DONE];   // this CTA's unit count per matrix phase
    int issued;
    uint64_t policy;
};

// Issue the next stage of the stream into its ring slot (whose previous
// contents every warp has released), if the stream has one left.
__device__ __forceinline__ void issue_next(Producer &p, const PersistWeights &W, uint32_t ring, uint32_t ring_s,
                                           uint32_t full_bar) {
    if (p.c.ph == PH_DONE) return;
    const int st = p.issued % kStages;
    size_t stride;
    const int8_t *src = cursor_src(p.c, W, stride);
    const float *ssrc = cursor_scales(p.c, W);
    const uint32_t bar = full_bar + 8 * st;
    const uint32_t dst = ring + (uint32_t)st * kStageBytes;
    tc::mbar_expect_tx(bar, kStageBytes + kRows * 4);
    bulk_g2s(ring_s + (uint32_t)st * kRows * 4, ssrc, kRows * 4, bar, p.policy);
    if (stride == kSegBytes) {
        bulk_g2s(dst, src, kStageBytes, bar, p.policy);
    } else {
#pragma unroll 1
        for (int r = 0; r < kRows; ++r) bulk_g2s(dst + r * kSegBytes, src + (size_t)r * stride, kSegBytes, bar, p.policy);
    }
    ++p.issued;
    cursor_next(p.c, W.layers, p.cnt);
}

// The producer lane: streams every stage of this CTA in order, each into
// its slot once all compute warps have released the slot's previous stage.
// Leaves at the end of the stream, when the compute warps set *stop, or
// after a bounded wait (abort flag set); then sets *done.
__device__ __noinline__ void produce(Producer &p, const PersistWeights &W, uint32_t ring, uint32_t ring_s,
                                     uint32_t full_bar, uint32_t empty_bar, int *abort_flag, int *stop,
                                     int *issued_out, int *done) {
    volatile int *vstop = stop;
    p.c = Cursor{0, PH_QKV, 0, 0};
    p.issued = 0;
    p.policy = evict_first_policy();
    for (int ph = 0; ph < PH_DONE; ++ph) p.cnt[ph] = cta_units(ph_units(ph, W.vocab));
    cursor_settle(p.c, W.layers, p.cnt);
    while (p.c.ph != PH_DONE && *vstop == 0) {
        const int k = p.issued, st = k % kStages;
        if (k >= kStages) {
            const uint32_t bar = empty_bar + 8 * st, parity = ((k / kStages) - 1) & 1;
            const unsigned long long t0 = global_ns();
            bool ok = true;
            while (!tc::mbar_try_wait(bar, parity)) {
                if (*vstop) { ok = false; break; }
                if (global_ns() - t0 > kBarrierLimitNs) {
                    atomicExch(abort_flag, 1);
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
        }
        issue_next(p, W, ring, ring_s, full_bar);
        *reinterpret_cast<volatile int *>(issued_out) = p.issued;
    }
    __threadfence_block();
    *reinterpret_cast<volatile int *>(done) = 1;
}

// Quantisation of one whole row of N values (a single group, the per-row
// scale of the reference's activation quantisation) by the compute warps:
// warp 0 forms the scale (group_scale_ref; both half-warps compute
// it, so the full-mask shuffles of the reduction see all 32 lanes), then
// every thread quantises its elements.
template <int N>
__device__ __forceinline__ void quantize_row_n(const float *ts, int16_t *q, float *qs, float *scratch) {
    if (threadIdx.x < 32) {
        const float ss = group_sumsq_ref(ts, N, threadIdx.x & 15);
        const float sc = mul_rn(__fsqrt_rn(fma_rn(ss, __fdiv_rn(1.0f, (float)N), 1e-6f)), inv127());
        if (threadIdx.x == 0) {
            *qs = sc;
            scratch[0] = __fdiv_rn(1.0f, sc);
        }
    }
    csync();
    const float inv = scratch[0];
#pragma unroll
    for (int j = threadIdx.x; j < N; j += kPThreads) q[j] = quant_one(ts[j], inv);
    csync();
}

}  // namespace

__global__ void __launch_bounds__(kBlock, 1)
decode_persistent_kernel(PersistWeights W, PersistState S) {
    extern __shared__ __align__(1024) unsigned char smraw[];
    unsigned char *ring_ptr = smraw;
    int16_t *q16 = reinterpret_cast<int16_t *>(smraw + kRingBytes);
    float *xs = reinterpret_cast<float *>(smraw + kRingBytes + (size_t)I * sizeof(int16_t));
    float *ts = xs + I;
    float *sp = ts + H;
    const int4 *q_s = reinterpret_cast<const int4 *>(q16);
    float *nrm_w = sp + 2 * kSliceMax;     // [H] next RMSNorm weight (dequantised int8 value)
    float *nrm_s = nrm_w + H;               // [H / norm_group] its group scales
    // reference-order attention, phase 2 (q16 | xs | ts are free then):
    // exponentials [2][kOrdChunk] f32, V rows [kOrdChunk] x 8 halves, and the
    // same V transposed [8][kOrdChunk] halves -- 40 KB of the 44 KB region
    float *ord_e = reinterpret_cast<float *>(q16);
    uint4 *ord_v = reinterpret_cast<uint4 *>(ord_e + 2 * kOrdChunk);
    __half *ord_vt = reinterpret_cast<__half *>(ord_e + 6 * kOrdChunk);
    __shared__ __align__(8) uint64_t full_mb[kStages];
    __shared__ __align__(16) float ring_scales[kStages][kRows];   // per-row weight scales of each stage
    __shared__ __align__(8) uint64_t empty_mb[kStages];
    __shared__ int stop_flag;                  // compute warps leaving early: producer stops
    __shared__ int issued_sh;                  // stages issued so far (producer -> drain)
    __shared__ int prod_done;                  // the producer has left
    __shared__ float scratch[65];
    __shared__ float a_s_sh;
    __shared__ int aborted_at_entry;
    __shared__ int last_cta;
    __shared__ int pt_sm[kMaxPages];
    __shared__ float redf[2][kPWarps];
    __shared__ double redd[2][kPWarps];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ng = W.norm_group;
    const float eps = W.eps;
    const uint32_t ring = tc::smem_u32(ring_ptr);
    const uint32_t full_bar = tc::smem_u32(full_mb), empty_bar = tc::smem_u32(empty_mb);
    const uint32_t ring_s = tc::smem_u32(&ring_scales[0][0]);
    unsigned long long bar_target = 0;  // thread 0: count that completes the current grid barrier
    unsigned long long head_target = 0; // thread 0: count that completes the current head barrier
    Producer prod;                      // used by the producer lane only
    int cons = 0;                       // stages consumed (same count in every compute thread)
    int nsync = 0;                      // grid barriers passed
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) S.trace[0] = global_ns();
        // a workspace left aborted by an earlier call: decode nothing
        aborted_at_entry = ld_volatile(reinterpret_cast<const unsigned *>(S.abort_flag)) != 0;
        // a position past the KV cache / RoPE table, or a token outside the
        // vocabulary, decodes nothing either: every CTA sees the same values,
        // so all leave before any load that depends on them, and the word
        // tells the host why (token and pos are left unchanged).
        // barrier counters are monotonic across launches and complete at
        // multiples of their participant counts; no barrier of this launch can
        // complete before this CTA arrives, so rounding down gives the base
        {
            unsigned long long v;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(S.bar_count) : "memory");
            bar_target = (v / gridDim.x) * gridDim.x;
            if (blockIdx.x < NKV * kSlices) {
                asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(S.head_bar + blockIdx.x / kSlices) : "memory");
                head_target = (v / kSlices) * kSlices;
            }
        }
        const int p0 = S.pos[0], t0 = S.token[0];
        if (!aborted_at_entry && (p0 < 0 || p0 >= S.max_ctx || t0 < 0 || t0 >= W.vocab)) {
            aborted_at_entry = 1;
            if (blockIdx.x == 0) atomicCAS(S.abort_flag, 0, (p0 < 0 || p0 >= S.max_ctx) ? 2 : 3);
        }
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(full_bar + 8 * i, 1);
            tc::mbar_init(empty_bar + 8 * i, kPWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        stop_flag = 0;
        issued_sh = 0;
        prod_done = 0;
    }
    for (int i = threadIdx.x; i < (S.max_ctx + S.page_size - 1) / S.page_size; i += kBlock)
        pt_sm[i] = S.page_table[i];
    __syncthreads();
    if (aborted_at_entry) return;
    if (warp == kPWarps) {                   // the producer warp
        if (lane == 0) produce(prod, W, ring, ring_s, full_bar, empty_bar, S.abort_flag, &stop_flag, &issued_sh, &prod_done);
        return;
    }
    const int token = S.token[0];
    const int pos = S.pos[0];
    const int ctx = min(pos + 1, S.max_ctx);

    // Wait (bounded) for every stage still in flight, so that no copy
    // targets shared memory after the CTA has left.
    auto drain = [&]() {
        if (threadIdx.x == 0) {
            *reinterpret_cast<volatile int *>(&stop_flag) = 1;
            // the producer leaves within one issue; then its count is final
            const unsigned long long t0 = global_ns();
            while (*reinterpret_cast<volatile int *>(&prod_done) == 0 && global_ns() - t0 < kBarrierLimitNs) {
            }
            const int issued = *reinterpret_cast<volatile int *>(&issued_sh);
            for (int k = max(0, issued - kStages); k < issued; ++k)
                tc::mbar_wait(full_bar + 8 * (k % kStages), (k / kStages) & 1, nullptr);
        }
    };
#ifdef QVL_PERSIST_DETAIL
#define DETAIL(slot) do { if (blockIdx.x == 0 && threadIdx.x == 0) S.trace[slot] = global_ns(); } while (0)
#define DETAIL_ALL(slot) do { if (threadIdx.x == 0) S.trace[(slot) + blockIdx.x] = global_ns(); } while (0)
#else
#define DETAIL(slot) do { } while (0)
#define DETAIL_ALL(slot) do { } while (0)
#endif
#define GRID_ARRIVE() grid_arrive(S, bar_target)
#define GRID_WAIT_OR_EXIT()                                                               \
    do {                                                                                  \
        if (!grid_wait(S, bar_target, nsync)) { drain(); return; }                        \
    } while (0)
#define SYNC_OR_EXIT()                                                                    \
    do {                                                                                  \
        GRID_ARRIVE();                                                                    \
        GRID_WAIT_OR_EXIT();                                                              \
    } while (0)

    // Run fn(stage, row scale) on the next stage of the ring once it has
    // landed (all lanes), then release the slot to the producer warp.
    auto consume = [&](auto &&fn) {
        const int st = cons % kStages;
        bool ok = tc::mbar_wait(full_bar + 8 * st, (cons / kStages) & 1, S.abort_flag);
        ok = __any_sync(0xffffffffu, ok);          // the phase completes once for all lanes
        if (ok) fn(ring_ptr + (size_t)st * kStageBytes, ring_scales[st][warp]);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar + 8 * st);
        ++cons;
        __syncwarp();
    };

    // Stage RMSNorm weights (int8 -> float, group scales) in shared memory;
    // done before the barrier that precedes the norm.  Reads them after
    // the CTA barrier at the top of the next grid barrier.
    auto stage_norm = [&](const int8_t *wq, const float *wsc) {
        for (int j = threadIdx.x; j < H; j += kPThreads) nrm_w[j] = (float)__ldg(wq + j);
        for (int j = threadIdx.x; j < H / ng; j += kPThreads) nrm_s[j] = __ldg(wsc + j);
    };
    // x (residual, written by other CTAs) -> RMSNorm with the staged weight
    // -> quantisation (one scale) into q16 / a_s_sh; arithmetic of
    // cta_norm_quant_row.
    auto norm_quant_x = [&](bool inplace_form, int dbg = -1, bool x_in_smem = false) {
        if (!x_in_smem)
            for (int i = threadIdx.x; i < H / 4; i += kPThreads)
                reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(S.x) + i);
        csync();
        if (dbg >= 0) DETAIL(dbg);
        if (threadIdx.x < 32) {
            const float ss = rms_sumsq_ref(xs, H);
            if (threadIdx.x == 0) scratch[64] = rms_inv(ss, H, eps, inplace_form);
        }
        csync();
        if (dbg >= 0) DETAIL(dbg + 1);
        const float inv = scratch[64];
        for (int j = threadIdx.x; j < H; j += kPThreads) ts[j] = mul_rn(nrm_w[j], mul_rn(mul_rn(nrm_s[j / ng], inv), xs[j]));
        csync();
        if (dbg >= 0) DETAIL(dbg + 2);
        quantize_row_n<H>(ts, q16, &a_s_sh, scratch);
        if (dbg >= 0) DETAIL(dbg + 3);
    };

    // embedding_lookup (per-row scale) of the input token: every CTA forms
    // the row in shared memory for the first RMSNorm (no barrier needed);
    // CTA 0 also writes it to the residual stream, read after the next barrier
    {
        const int id = (token >= 0 && token < W.vocab) ? token : 0;
        const float sc = W.embed_s[id];
        for (int j = threadIdx.x; j < H; j += kPThreads) {
            const float v = mul_rn((float)W.embed[(size_t)id * H + j], sc);
            xs[j] = v;
            if (blockIdx.x == 0) S.x[j] = v;
        }
    }
    stage_norm(W.in_norm, W.in_norm_s);

    const int per = (ctx + kSlices - 1) / kSlices;
    const bool attn_cta = blockIdx.x < NKV * kSlices;
    const int kvh = blockIdx.x / kSlices, sl = blockIdx.x % kSlices;
    const int t0 = min(ctx, sl * per), t1 = min(ctx, t0 + per), len = t1 - t0;
    const int t16 = threadIdx.x & 15, hw = threadIdx.x >> 4;

    for (int l = 0; l < W.layers; ++l) {
        // this layer's cached K/V rows of the slice (all but the new token) into L2
        if (attn_cta) {
            const int n_old = min(len, max(0, pos - t0));
            for (int e = threadIdx.x; e < 4 * n_old; e += kPThreads) {
                const int t = e >> 2, half = e & 1;
                const uint16_t *base = (e & 2) ? S.v_pages : S.k_pages;
                prefetch_l2(base + kv_off(S, pt_sm, l, t0 + t, kvh) + half * (D / 2));
            }
        }
        // ---- input rms_norm + quantisation (every CTA), q/k/v blocks of the ring
        norm_quant_x(false, l == 5 ? 240 : -1, l == 0);
        if (l == 5) DETAIL(230);
        {
            const int nu = cta_units(ph_units(PH_QKV, W.vocab));
            Act act;
            load_act(q_s, 0, lane, act);
            for (int j = 0; j < nu; ++j) {
                const int n = ((int)blockIdx.x + j * (int)gridDim.x) * kRows + warp;
                consume([&](const unsigned char *st, float sc) {
                    int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    madd_seg(st, warp, lane, act, p);
                    const float out = finish_row(p, a_s_sh, sc, lane);
                    if (lane == 0) S.qkv[n] = out;
                });
            }
        }
        if (l == 5) DETAIL(231);
        GRID_ARRIVE();
        // QK-norm weights and this position's RoPE row, read while the barrier completes
        float qn_w = 0.0f, qn_s = 0.0f, kn_w = 0.0f, kn_s = 0.0f, rc = 0.0f, rs = 0.0f;
        if (attn_cta && threadIdx.x < D) {
            qn_w = (float)__ldg(W.q_norm + (size_t)l * D + threadIdx.x);
            qn_s = __ldg(W.q_norm_s + (size_t)l * (D / ng) + threadIdx.x / ng);
            kn_w = (float)__ldg(W.k_norm + (size_t)l * D + threadIdx.x);
            kn_s = __ldg(W.k_norm_s + (size_t)l * (D / ng) + threadIdx.x / ng);
            if (threadIdx.x < D / 2) {
                rc = __ldg(S.rope_cos + (size_t)pos * (D / 2) + threadIdx.x);
                rs = __ldg(S.rope_sin + (size_t)pos * (D / 2) + threadIdx.x);
            }
        }
        GRID_WAIT_OR_EXIT();
        if (l == 5) DETAIL_ALL(760);

        // ---- attention, phase 1.  q/k rms_norm_inplace + RoPE of this KV
        // head's two query heads (every slice CTA of the head, redundantly)
        // and of its key (the CTA whose slice holds the new position, which
        // appends k and v to the pages as fp16); then the scores of the slice
        // and their maximum.  (A position past the cache is not appended;
        // the host keeps pos < max_ctx.)
        if (attn_cta) {
            const bool owner = pos < S.max_ctx && t0 <= pos && pos < t1;
            float *raw = xs;                 // [3][D]: q (2 heads), k
            float *nrm = xs + 3 * D;         // [3][D] normalised
            float *qrot = xs + 6 * D;        // [2][D] rotated queries
            const int rows = owner ? 3 : 2;
            if (threadIdx.x < rows * D) {
                const int r = threadIdx.x / D, j = threadIdx.x - r * D;
                const float *src = r < 2 ? S.qkv + (kvh * 2 + r) * D : S.qkv + NH * D + kvh * D;
                raw[threadIdx.x] = __ldcg(src + j);
            }
            csync();
            if (warp < rows) {
                const float ss = rms_sumsq_ref(raw + warp * D, D);
                if (lane == 0) scratch[warp] = rms_inv(ss, D, eps, true);
            }
            csync();
            if (threadIdx.x < D)
                for (int r = 0; r < rows; ++r)
                    nrm[r * D + threadIdx.x] = mul_rn(r < 2 ? qn_w : kn_w,
                                                      mul_rn(mul_rn(r < 2 ? qn_s : kn_s, scratch[r]), raw[r * D + threadIdx.x]));
            csync();
            if (threadIdx.x < D / 2) {
                const int j = threadIdx.x;
                for (int r = 0; r < rows; ++r) {
                    const float x1 = nrm[r * D + j], x2 = nrm[r * D + j + D / 2];
                    const float y1 = fma_rn(x1, rc, -mul_rn(x2, rs));
                    const float y2 = fma_rn(x1, rs, mul_rn(x2, rc));
                    if (r < 2) {
                        qrot[r * D + j] = y1;
                        qrot[r * D + j + D / 2] = y2;
                    } else {
                        const size_t off = kv_off(S, pt_sm, l, pos, kvh);
                        S.k_pages[off + j] = __half_as_ushort(__float2half_rn(y1));
                        S.k_pages[off + j + D / 2] = __half_as_ushort(__float2half_rn(y2));
                    }
                }
            }
            if (owner && threadIdx.x >= D && threadIdx.x < 2 * D) {
                const int j = threadIdx.x - D;
                const size_t off = kv_off(S, pt_sm, l, pos, kvh);
                S.v_pages[off + j] = __half_as_ushort(__float2half_rn(__ldcg(S.qkv + NH * D + NKV * D + kvh * D + j)));
            }
            csync();                 // the appended key row is read back below
            if (l == 5) DETAIL(250);
            float qv[2][8];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) qv[h][e] = qrot[h * D + t16 * 8 + e];
            const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
            const unsigned hmask = 0xffffu << (threadIdx.x & 16);
            float mx[2] = {-INFINITY, -INFINITY};
            if (S.ordered) {
                // reference order: one thread per (token, query head) runs the
                // score's whole chain -- 8 fused lanes + add_reduce_mm_256_layer
                // below 8*(pos/8), 8 unfused lanes added in order in the tail
                // (layers/src/text_layer.cpp:590-645).  Key rows are staged
                // through shared memory 64 at a time (rows padded to 272 B).
                const int tail0 = (pos / 8) * 8;
                uint4 *kst = reinterpret_cast<uint4 *>(xs + 8 * D);
                for (int c0 = 0; c0 < len; c0 += 64) {
                    const int n = min(64, len - c0);
                    for (int e = threadIdx.x; e < n * 16; e += kPThreads)
                        kst[(e >> 4) * 17 + (e & 15)] = __ldcg(
                            reinterpret_cast<const uint4 *>(S.k_pages + kv_off(S, pt_sm, l, t0 + c0 + (e >> 4), kvh)) + (e & 15));
                    csync();
                    if (threadIdx.x < 2 * n) {
                        const int t = c0 + (threadIdx.x >> 1), h = threadIdx.x & 1;
                        const uint4 *kr = kst + (threadIdx.x >> 1) * 17;
                        const float *qh = qrot + h * D;
                        float l8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                        const bool tail = t0 + t >= tail0;
#pragma unroll 4
                        for (int c = 0; c < D / 8; ++c) {
                            float kf[8];
                            h8f(kr[c], kf);
                            if (!tail) {
#pragma unroll
                                for (int j = 0; j < 8; ++j) l8[j] = fma_rn(qh[8 * c + j], kf[j], l8[j]);
                            } else {
#pragma unroll
                                for (int j = 0; j < 8; ++j) l8[j] = add_rn(l8[j], mul_rn(qh[8 * c + j], kf[j]));
                            }
                        }
                        float r;
                        if (!tail) {
                            r = reduce8_ref(l8);
                        } else {
                            r = l8[0];
#pragma unroll
                            for (int j = 1; j < 8; ++j) r = add_rn(r, l8[j]);
                            r = add_rn(0.0f, r);
                        }
                        const float sc = mul_rn(r, inv_sqrt_d);
                        sp[h * kSliceMax + t] = sc;
                        __stcg(S.att_e + (size_t)(kvh * 2 + h) * (kSlices * kSliceMax) + t0 + t, sc);
                        if (h == 0) mx[0] = fmaxf(mx[0], sc); else mx[1] = fmaxf(mx[1], sc);
                    }
                    csync();
                }
            }
            for (int tb = S.ordered ? len : hw; tb < len; tb += 32 * 4) {
                uint4 kr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    kr[u] = (t < len) ? __ldcg(reinterpret_cast<const uint4 *>(S.k_pages + kv_off(S, pt_sm, l, t0 + t, kvh)) + t16)
                                      : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    float kf[8];
                    h8f(kr[u], kf);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float acc = 0.0f;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc = fma_rn(qv[h][e], kf[e], acc);
#pragma unroll
                        for (int o = 8; o >= 1; o >>= 1) acc += __shfl_xor_sync(hmask, acc, o, 16);
                        const float sc = mul_rn(acc, inv_sqrt_d);
                        if (t < len) {
                            mx[h] = fmaxf(mx[h], sc);
                            if (t16 == 0) sp[h * kSliceMax + t] = sc;
                        }
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float m = mx[h];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (lane == 0) redf[h][warp] = m;
            }
            csync();
            if (threadIdx.x < 2) {
                float m = redf[threadIdx.x][0];
                for (int w = 1; w < kPWarps; ++w) m = fmaxf(m, redf[threadIdx.x][w]);
                S.att_lmax[(kvh * 2 + threadIdx.x) * kSlices + sl] = m;
            }
            if (S.ordered && ctx <= kOrdChunk) {
                // this slice CTA's output columns [8*sl, 8*sl+8) of V at every
                // cached position, fetched while the head barrier completes;
                // the new position's row (appended by its owner slice in this
                // phase) is read after the barrier
                csync();            // the key staging area (xs) is free
                const uint32_t vb = tc::smem_u32(ord_v);
                for (int t = threadIdx.x; t < ctx - 1; t += kPThreads)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vb + 16u * (uint32_t)t),
                                 "l"(S.v_pages + kv_off(S, pt_sm, l, t, kvh) + 8 * sl)
                                 : "memory");
                asm volatile("cp.async.commit_group;" ::: "memory");
            }
            if (l == 5) DETAIL(251);
            if (!head_sync(S, kvh, head_target)) { drain(); return; }
            if (l == 5) DETAIL(252);
        }

        // ---- attention, phase 2: probabilities (global max), slice sum, partial P.V
        if (attn_cta) {
            __shared__ float gm[2];
            // reference order, one chunk: this thread's scores (2 per thread
            // at ctx <= 512, 4 at 1024) load while the maxima are combined
            float pre[4];
            const bool pre_ok = S.ordered && ctx <= kOrdChunk && 2 * ctx <= 4 * kPThreads;
            if (pre_ok) {
                const float *s0 = S.att_e + (size_t)(kvh * 2) * (kSlices * kSliceMax);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int e = threadIdx.x + u * kPThreads;
                    const int h = e >= ctx, k = h ? e - ctx : e;
                    pre[u] = e < 2 * ctx ? __ldcg(s0 + (size_t)h * (kSlices * kSliceMax) + k) : 0.0f;
                }
            }
            if (threadIdx.x < 2) {
                float m = -INFINITY;
                for (int s2 = 0; s2 < kSlices; ++s2) m = fmaxf(m, __ldcg(S.att_lmax + (kvh * 2 + threadIdx.x) * kSlices + s2));
                gm[threadIdx.x] = m;
            }
            csync();
            if (l == 5) DETAIL(256);
            if (S.ordered) {
                // reference order (layers/src/text_layer.cpp:473-535, 677-689).
                // Every slice CTA reads all of the head's scores (written to the
                // workspace in phase 1) and forms the exponentials with the
                // global maximum itself, so no second barrier is needed; it then
                // sums them into 8 float lanes t-ascending, the lanes then the
                // tail in double, and runs the fma chains (one per output
                // element, t ascending) of its 8 output dimensions of both
                // query heads, p = e * (float)(1/sum).  The exponentials and the
                // V column are staged in shared memory, kOrdChunk positions at
                // a time (V already fetched during the head barrier when the
                // context fits one chunk).
                constexpr int kCh = kOrdChunk;
                float *ebuf = ord_e;                                // [2][kCh]
                uint4 *vbuf = ord_v;                                // [kCh] 8 halves each
                const int d0 = 8 * sl, n8 = (ctx / 8) * 8;
                const float *s0 = S.att_e + (size_t)(kvh * 2) * (kSlices * kSliceMax);
                const float *s1 = s0 + kSlices * kSliceMax;
                const bool one = ctx <= kCh;
                auto stage = [&](int c0, int n, bool with_v) {
                    if (pre_ok) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int e = threadIdx.x + u * kPThreads;
                            if (e < 2 * n) {
                                const int h = e >= n, k = h ? e - n : e;
                                ebuf[h * kCh + k] = (pre[u] > -INFINITY) ? exp_ref(pre[u] - gm[h]) : 0.0f;
                            }
                        }
                    } else {
                        for (int e = threadIdx.x; e < 2 * n; e += kPThreads) {
                            const int h = e >= n, k = h ? e - n : e;
                            const float sv = __ldcg((h ? s1 : s0) + c0 + k);
                            ebuf[h * kCh + k] = (sv > -INFINITY) ? exp_ref(sv - gm[h]) : 0.0f;
                        }
                    }
                    if (with_v)
                        for (int e = threadIdx.x; e < n; e += kPThreads)
                            vbuf[e] = __ldcg(reinterpret_cast<const uint4 *>(S.v_pages + kv_off(S, pt_sm, l, c0 + e, kvh) + d0));
                    csync();
                };
                float lane_acc = 0.0f;             // thread h*8+ln: lane ln of head h
                if (one && threadIdx.x == kPThreads - 1)    // the new position's row (see phase 1)
                    vbuf[ctx - 1] = __ldcg(reinterpret_cast<const uint4 *>(S.v_pages + kv_off(S, pt_sm, l, ctx - 1, kvh) + d0));
                for (int c0 = 0; c0 < ctx; c0 += kCh) {
                    const int n = min(kCh, ctx - c0);
                    stage(c0, n, false);
                    if (threadIdx.x < 16) {
                        const float *eb = ebuf + (threadIdx.x >> 3) * kCh;
                        const int ln = threadIdx.x & 7;
                        // t = c0 + k with t = ln mod 8 (c0 is a multiple of 8), t < n8
                        const int kend = min(n, n8 - c0);
                        int k = ln;
                        for (; k + 56 < kend; k += 64) {        // 8 loads ahead of the serial adds
                            float e8[8];
#pragma unroll
                            for (int u = 0; u < 8; ++u) e8[u] = eb[k + 8 * u];
#pragma unroll
                            for (int u = 0; u < 8; ++u) lane_acc = add_rn(lane_acc, e8[u]);
                        }
                        for (; k < kend; k += 8) lane_acc = add_rn(lane_acc, eb[k]);
                    }
                    if (!one) csync();
                }
                if (l == 5) DETAIL(257);
                if (threadIdx.x < 16) scratch[threadIdx.x] = lane_acc;
                csync();
                if (l == 5) DETAIL(258);
                if (threadIdx.x < 2) {
                    // the tail (at most 7 positions), still staged when one chunk
                    const int h = threadIdx.x;
                    double sum = 0.0;
                    for (int ln = 0; ln < 8; ++ln) sum = __dadd_rn(sum, (double)scratch[h * 8 + ln]);
                    for (int t = n8; t < ctx; ++t) {
                        const float sv = one ? 0.0f : __ldcg((h ? s1 : s0) + t);
                        const float e = one ? ebuf[h * kCh + t] : ((sv > -INFINITY) ? exp_ref(sv - gm[h]) : 0.0f);
                        sum = __dadd_rn(sum, (double)e);
                    }
                    const bool zero = !isfinite(gm[h]) || !(sum > 0.0) || !isfinite(sum);
                    scratch[32 + h] = zero ? 0.0f : 1.0f;
                    scratch[34 + h] = __double2float_rn(__ddiv_rn(1.0, sum));
                }
                if (one) asm volatile("cp.async.wait_group 0;" ::: "memory");
                csync();
                if (l == 5) DETAIL(259);
                const int h = threadIdx.x >> 3, j = threadIdx.x & 7;
                float a = 0.0f;
                for (int c0 = 0; c0 < ctx; c0 += kCh) {
                    const int n = min(kCh, ctx - c0);
                    if (!one) stage(c0, n, true);
                    // p = e * (float)(1/sum) in place, and V transposed to
                    // [d][t] so that a chain reads 8 positions per 16-byte load
                    for (int e = threadIdx.x; e < 2 * n; e += kPThreads) {
                        const int hh = e >= n, k = hh ? e - n : e;
                        ebuf[hh * kCh + k] = mul_rn(ebuf[hh * kCh + k], scratch[34 + hh]);
                    }
                    for (int e = threadIdx.x; e < n; e += kPThreads) {
                        const uint4 r = vbuf[e];
                        const __half *hv = reinterpret_cast<const __half *>(&r);
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) ord_vt[jj * kCh + e] = hv[jj];
                    }
                    csync();
                    if (threadIdx.x < 16) {
                        const float4 *pb = reinterpret_cast<const float4 *>(ebuf + h * kCh);
                        const uint4 *vt = reinterpret_cast<const uint4 *>(ord_vt + j * kCh);
                        const int n8c = n & ~7;
                        for (int k = 0; k < n8c; k += 8) {
                            const float4 p0 = pb[k / 4], p1 = pb[k / 4 + 1];
                            const uint4 vr = vt[k / 8];
                            float vf[8];
                            h8f(vr, vf);
                            a = fma_rn(p0.x, vf[0], a);
                            a = fma_rn(p0.y, vf[1], a);
                            a = fma_rn(p0.z, vf[2], a);
                            a = fma_rn(p0.w, vf[3], a);
                            a = fma_rn(p1.x, vf[4], a);
                            a = fma_rn(p1.y, vf[5], a);
                            a = fma_rn(p1.z, vf[6], a);
                            a = fma_rn(p1.w, vf[7], a);
                        }
                        for (int k = n8c; k < n; ++k) a = fma_rn(ebuf[h * kCh + k], __half2float(ord_vt[j * kCh + k]), a);
                    }
                    if (!one) csync();
                }
                if (threadIdx.x < 16) S.att_out[(kvh * 2 + h) * D + d0 + j] = scratch[32 + h] != 0.0f ? a : 0.0f;
                if (l == 5) DETAIL(255);
            } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                double part = 0.0;
                for (int t = threadIdx.x; t < len; t += kPThreads) {
                    const float sv = sp[h * kSliceMax + t];
                    const float p = (sv > -INFINITY) ? exp_ref(sv - gm[h]) : 0.0f;
                    sp[h * kSliceMax + t] = p;
                    part += (double)p;
                }
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
                if (lane == 0) redd[h][warp] = part;
            }
            csync();
            if (threadIdx.x < 2) {
                double sum = 0.0;
                for (int w = 0; w < kPWarps; ++w) sum += redd[threadIdx.x][w];
                S.att_lsum[(kvh * 2 + threadIdx.x) * kSlices + sl] = sum;
            }
            float acc[2][8];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[h][e] = 0.0f;
            for (int tb = hw; tb < len; tb += 32 * 4) {
                uint4 vr[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    vr[u] = (t < len) ? __ldcg(reinterpret_cast<const uint4 *>(S.v_pages + kv_off(S, pt_sm, l, t0 + t, kvh)) + t16)
                                      : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = tb + 32 * u;
                    if (t < len) {
                        float vf[8];
                        h8f(vr[u], vf);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float p = sp[h * kSliceMax + t];
#pragma unroll
                            for (int e = 0; e < 8; ++e) acc[h][e] = fma_rn(p, vf[e], acc[h][e]);
                        }
                    }
                }
            }
            float *red = xs;   // [32 token lanes][2][D]
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 8; ++e) red[(hw * 2 + h) * D + t16 * 8 + e] = acc[h][e];
            csync();
            for (int e = threadIdx.x; e < 2 * D; e += kPThreads) {
                const int h = e / D, dd = e - h * D;
                float s2 = 0.0f;
                for (int w = 0; w < 32; ++w) s2 += red[(w * 2 + h) * D + dd];
                S.att_pacc[((kvh * 2 + h) * kSlices + sl) * D + dd] = s2;
            }
            // The last of the head's 16 slice CTAs to finish combines its two
            // query heads (softmax normalisation included) into att_out, so
            // that the o_proj phase reads 8 KB instead of every partial.
            __threadfence();
            csync();
            if (threadIdx.x == 0) last_cta = atomicAdd(S.att_cnt + kvh, 1) == kSlices - 1;
            csync();
            if (last_cta) {
                __threadfence();
                if (threadIdx.x < 2 * D / 4) {
                    const int e0 = threadIdx.x * 4, head = kvh * 2 + e0 / D, dd = e0 % D;
                    float4 pv[kSlices];
                    float lm[kSlices];
                    double ls[kSlices];
#pragma unroll
                    for (int s2 = 0; s2 < kSlices; ++s2) {
                        pv[s2] = __ldcg(reinterpret_cast<const float4 *>(S.att_pacc + (head * kSlices + s2) * D + dd));
                        lm[s2] = __ldcg(S.att_lmax + head * kSlices + s2);
                        ls[s2] = __ldcg(S.att_lsum + head * kSlices + s2);
                    }
                    float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    float m = -INFINITY;
                    double sum = 0.0;
#pragma unroll
                    for (int s2 = 0; s2 < kSlices; ++s2) {
                        a.x += pv[s2].x; a.y += pv[s2].y; a.z += pv[s2].z; a.w += pv[s2].w;
                        m = fmaxf(m, lm[s2]);
                        sum += ls[s2];
                    }
                    // the reference zeroes the row when the max is not finite or the
                    // sum is not a positive finite number (text_layer.cpp:466-469, :514-517)
                    const bool zero = ctx <= 0 || !isfinite(m) || !(sum > 0.0) || !isfinite(sum);
                    const float inv = zero ? 0.0f : (float)(1.0 / sum);
                    reinterpret_cast<float4 *>(S.att_out)[(head * D + dd) / 4] =
                        zero ? make_float4(0.0f, 0.0f, 0.0f, 0.0f)
                             : make_float4(mul_rn(a.x, inv), mul_rn(a.y, inv), mul_rn(a.z, inv), mul_rn(a.w, inv));
                }
                if (threadIdx.x == 0) S.att_cnt[kvh] = 0;     // next used a grid barrier later
            }
            }   // fast order
        }
        SYNC_OR_EXIT();
        if (l == 5) DETAIL_ALL(600);

        // ---- attention output (combined above) -> quantisation -> o_proj + residual
        for (int i = threadIdx.x; i < H / 4; i += kPThreads)
            reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(S.att_out) + i);
        csync();
        if (l == 5) DETAIL(245);
        quantize_row_n<H>(xs, q16, &a_s_sh, scratch);
        if (l == 5) DETAIL(246);
        {
            const int nu = cta_units(ph_units(PH_O, W.vocab));
            Act act;
            load_act(q_s, 0, lane, act);
            for (int j = 0; j < nu; ++j) {
                const int n = ((int)blockIdx.x + j * (int)gridDim.x) * kRows + warp;
                const float xn = lane == 0 ? __ldcg(S.x + n) : 0.0f;
                consume([&](const unsigned char *st, float sc) {
                    int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    madd_seg(st, warp, lane, act, p);
                    const float out = finish_row(p, a_s_sh, sc, lane);
                    if (lane == 0) S.x[n] = add_rn(xn, out);
                });
            }
        }
        if (l == 5) DETAIL(247);
        GRID_ARRIVE();
        if (l == 5) DETAIL_ALL(300);
        stage_norm(W.post_norm + (size_t)l * H, W.post_norm_s + (size_t)l * (H / ng));
        if (l == 5) DETAIL(248);
        GRID_WAIT_OR_EXIT();

        // ---- post-attention rms_norm + quantisation (every CTA), gate/up + SwiGLU
        norm_quant_x(false);
        if (l == 5) DETAIL(232);

        {
            const int nu = cta_units(ph_units(PH_GU, W.vocab));
            Act act;
            load_act(q_s, 0, lane, act);
            // lane j keeps unit j's gate/up pair; the SwiGLUs (double-precision
            // exp) run once, in parallel, after the last unit
            float g_keep = 0.0f, u_keep = 0.0f;
            for (int j = 0; j < nu; ++j) {
                float gate_v = 0.0f;
                consume([&](const unsigned char *st, float sc) {
                    int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    madd_seg(st, warp, lane, act, p);
                    gate_v = finish_row(p, a_s_sh, sc, lane);
                });
                consume([&](const unsigned char *st, float sc) {
                    int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    madd_seg(st, warp, lane, act, p);
                    const float up = finish_row(p, a_s_sh, sc, lane);
                    if (lane == j) { g_keep = gate_v; u_keep = up; }
                });
            }
            if (lane < nu) S.h[((int)blockIdx.x + lane * (int)gridDim.x) * kRows + warp] = swiglu_one(g_keep, u_keep);
        }
        if (l == 5) DETAIL(233);

        SYNC_OR_EXIT();

        // ---- quantisation of the SwiGLU row (every CTA), down + residual
        for (int i = threadIdx.x; i < I / 4; i += kPThreads)
            reinterpret_cast<float4 *>(xs)[i] = __ldcg(reinterpret_cast<const float4 *>(S.h) + i);
        csync();
        quantize_row_n<I>(xs, q16, &a_s_sh, scratch);
        if (l == 5) DETAIL(234);
        {
            const int nu = cta_units(ph_units(PH_DOWN, W.vocab));
            for (int j = 0; j < nu; ++j) {
                const int n = ((int)blockIdx.x + j * (int)gridDim.x) * kRows + warp;
                float ws = 0.0f;
                const float xn = lane == 0 ? __ldcg(S.x + n) : 0.0f;
                int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int s = 0; s < I / kSegBytes; ++s)
                    consume([&](const unsigned char *st, float sc) {
                        Act act;
                        load_act(q_s, s * (kSegBytes / 16), lane, act);
                        madd_seg(st, warp, lane, act, p);
                        ws = sc;
                    });
                const float out = finish_row(p, a_s_sh, ws, lane);
                if (lane == 0) S.x[n] = add_rn(xn, out);
            }
        }
        if (l == 5) DETAIL(235);
        GRID_ARRIVE();
        if (l == 5) DETAIL_ALL(500);
        if (l + 1 < W.layers) stage_norm(W.in_norm + (size_t)(l + 1) * H, W.in_norm_s + (size_t)(l + 1) * (H / ng));
        else stage_norm(W.final_norm, W.final_norm_s);
        GRID_WAIT_OR_EXIT();
    }

    // ---- final rms_norm_inplace + quantisation (every CTA), LM head + greedy
    norm_quant_x(true);
    {
        float best_v = -FLT_MAX;
        int best_i = INT_MAX;
        const int nu = cta_units(ph_units(PH_LM, W.vocab));
        Act act;
        load_act(q_s, 0, lane, act);
        DETAIL(200);
        for (int j = 0; j < nu; ++j) {
            if ((j & 7) == 7) DETAIL(201 + (j >> 3));
            const int n = ((int)blockIdx.x + j * (int)gridDim.x) * kRows + warp;
            consume([&](const unsigned char *st, float sc) {
                int p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                madd_seg(st, warp, lane, act, p);
                const float out = finish_row(p, a_s_sh, sc, lane);
                if (lane == 0) S.logits[n] = out;
                if (out > best_v) { best_v = out; best_i = n; }   // ascending n: strict > keeps the first
            });
        }
        if (lane == 0) {
            const int gw = blockIdx.x * kPWarps + warp;
            S.warp_best_v[gw] = best_v;
            S.warp_best_i[gw] = best_i;
        }
    }
    SYNC_OR_EXIT();
#undef SYNC_OR_EXIT
    if (blockIdx.x == 0) {
        const int nw = gridDim.x * kPWarps;
        float v = -FLT_MAX;
        int bi = INT_MAX;
        for (int w = threadIdx.x; w < nw; w += kPThreads) {
            const float v2 = __ldcg(S.warp_best_v + w);
            const int i2 = __ldcg(S.warp_best_i + w);
            if (v2 > v || (v2 == v && i2 < bi)) { v = v2; bi = i2; }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (v2 > v || (v2 == v && i2 < bi)) { v = v2; bi = i2; }
        }
        if (lane == 0) { redf[0][warp] = v; reinterpret_cast<int *>(scratch)[warp] = bi; }
        csync();
        if (threadIdx.x == 0) {
            float fv = -FLT_MAX;
            int fi = INT_MAX;
            for (int w = 0; w < kPWarps; ++w) {
                const float v2 = redf[0][w];
                const int i2 = reinterpret_cast<int *>(scratch)[w];
                if (v2 > fv || (v2 == fv && i2 < fi)) { fv = v2; fi = i2; }
            }
            S.token[0] = (fi == INT_MAX) ? 0 : fi;
            S.pos[0] = pos + 1;
        }
    }
}

size_t persist_smem_bytes() { return kSmemBytes; }

int persist_grid_ctas() {
    static int cached[64] = {};                 // per device, computed on first use
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev < 64 && cached[dev] > 0) return cached[dev];
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)persist_smem_bytes()) != cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, kBlock,
                                                      persist_smem_bytes()) != cudaSuccess)
        return 0;
    // every attention (KV head, slice) pair and QK row needs a CTA of its own
    const int ctas = sms * (per_sm > 1 ? 1 : per_sm);
    if (ctas < NKV * kSlices) return 0;
    if (dev < 64) cached[dev] = ctas;
    return ctas;
}

bool persist_supported(int hidden, int intermediate, int heads, int kv_heads, int head_dim, int max_ctx) {
    return hidden == H && intermediate == I && heads == NH && kv_heads == NKV && head_dim == D && max_ctx >= 1 &&
           max_ctx <= kSlices * kSliceMax;
}

cudaError_t launch_decode_persistent(const PersistWeights &w, const PersistState &s, int ctas, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kBlock);
    cfg.dynamicSmemBytes = persist_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, w, s);
}

}  // namespace qvl
