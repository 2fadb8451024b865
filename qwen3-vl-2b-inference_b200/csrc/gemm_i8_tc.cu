// INT8 GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) for
// prefill-shaped products: C[M, N] = A[M, K] . dequant(W[N, K])^T with the
// reference's TILED summation (matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:
// 538-653) and per-output-row weight scales (group = K).
//
// Exactness.  The reference multiplies int16 activations by int8 weights.
// int16 does not fit an int8 MMA operand, so each quantised activation is
// split exactly as q = 256*hi + lo with hi = q >> 8 (signed 8-bit) and
// lo = q & 255 (unsigned 8-bit).  Two MMAs per K step accumulate
// D_hi = W.hi and D_lo = W.lo in int32 in tensor memory, and the epilogue
// forms S = 256*D_hi + D_lo, the exact integer dot product (|S| < 2^31 for
// any quantised row).  The fp32 epilogue is the reference's:
// C = fma(float(S) * a_s, w_s, 0).
//
// Tiling.  "Swap AB": the MMA's M dimension is 128 weight rows (TMEM lanes),
// its N dimension a tile of NT activation rows (TMEM columns), K steps of 32
// bytes.  A CTA computes a 128 x NT tile; one thread issues the TMA loads of
// a stage ring (128 B of K per stage, 128-byte swizzle), another thread
// issues the MMAs and commits each stage back to the ring, and four warps
// read the accumulators (tcgen05.ld) for the epilogue, with the tile's
// activation scales staged in shared memory beforehand.  Products of two or
// more waves of tiles run on a persistent kernel with double-buffered
// accumulators; smaller ones split K over a thread-block cluster.  Every wait
// is bounded.
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <cooperative_groups.h>
#include "tc_common.cuh"
#include "gemm_i8_tc.cuh"

namespace qvl {

namespace {
constexpr int kBM = 128;          // weight rows per CTA (MMA M)
constexpr int kBK = 128;          // bytes of K per stage
constexpr int kStages = 4;
constexpr int kThreads = 128;
constexpr int kUmmaK = 32;        // K per kind::i8 MMA
}  // namespace

// Set (to 1) when a bounded wait in this kernel gave up; while it is set the
// kernel computes nothing.  The host reads and clears it through
// qvl_tc_timeout_word().
__device__ int g_gemm_tc_timeout = 0;

__device__ __forceinline__ void mbar_arrive_cta(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <int NT>
struct TcSmem {
    static constexpr int kA = kBM * kBK;          // 16 KB
    static constexpr int kB = NT * kBK;           // one activation plane
    static constexpr int kStage = kA + 2 * kB;
    // 128-row activation tiles: 2 stages (96 KB), so two CTAs share an SM and
    // one's epilogue overlaps the other's main loop; smaller tiles keep 4
    static constexpr int kSt = NT >= 128 ? 2 : (NT >= 64 ? 3 : kStages);
    static constexpr int kBytes = kSt * kStage + 1024 /* align */ + 256 /* barriers */;
};

// Epilogue of one 128 x NT accumulator tile for the 32 weight rows of this
// warp (TMEM lanes lane_off >> 16 ..+31; this thread: row n, weight scale ws).
// as_s: the tile's NT activation scales, staged in shared memory before the
// accumulators are waited for.  32 columns per tcgen05.wait::ld; in the
// accumulate form the C values of a chunk are loaded before that wait.
template <int NT>
__device__ __forceinline__ void epilogue_rows(uint32_t d_hi, uint32_t d_lo, uint32_t lane_off,
                                              const float *as_s, float ws, int n, int m0, int M, int N,
                                              float *__restrict C, int acc) {
    constexpr int kC = NT < 32 ? NT : 32;
#pragma unroll 1
    for (int c0 = 0; c0 < NT; c0 += kC) {
        uint32_t hi[kC], lo[kC];
#pragma unroll
        for (int h = 0; h < kC; h += 16) {
            tc::tmem_ld16(d_hi + lane_off + c0 + h, *reinterpret_cast<uint32_t(*)[16]>(hi + h));
            tc::tmem_ld16(d_lo + lane_off + c0 + h, *reinterpret_cast<uint32_t(*)[16]>(lo + h));
        }
        float cv[kC];
        if (acc) {
#pragma unroll
            for (int j = 0; j < kC; ++j) {
                const int m = m0 + c0 + j;
                cv[j] = (m < M && n < N) ? C[(size_t)m * N + n] : 0.0f;
            }
        }
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < kC; ++j) {
            const int m = m0 + c0 + j;
            if (m < M && n < N) {
                const int S = (int)(hi[j] * 256u + lo[j]);   // exact mod 2^32, |S| < 2^31
                const float p = mul_rn(__int2float_rn(S), as_s[c0 + j]);
                const float v = fma_rn(p, ws, 0.0f);
                C[(size_t)m * N + n] = acc ? add_rn(cv[j], v) : v;   // residual add (add_vector order)
            }
        }
    }
}

// Up to three weight matrices of the same activations in one launch (q/k/v,
// gate/up): their 128-row weight tiles are numbered one after the other.
constexpr int kMaxMats = 3;
struct TcMats {
    CUtensorMap w[kMaxMats];
    const float *ws[kMaxMats];
    float *C[kMaxMats];
    int N[kMaxMats];
    int tile0[kMaxMats + 1];   // first weight tile of each matrix; tile0[n] = all tiles
    int n;
};

// grid: (ceil(M/NT), weight tiles of all matrices, SPLIT); block 128; with
// SPLIT > 1 the SPLIT CTAs of a cluster (1, 1, SPLIT) each take K/SPLIT and
// their exact int32 partial sums are added through distributed shared memory
// (split-K keeps small-N products -- decode batches -- spread over the GPU).
template <int NT, int SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8_tc_kernel(const __grid_constant__ TcMats mats, const __grid_constant__ CUtensorMap tm_hi,
                  const __grid_constant__ CUtensorMap tm_lo, const float *__restrict a_scale, int M, int K,
                  int acc) {
    const int mi = (mats.n > 1 && (int)blockIdx.y >= mats.tile0[1]) + (mats.n > 2 && (int)blockIdx.y >= mats.tile0[2]);
    const CUtensorMap *tm_w = &mats.w[mi];
    const float *__restrict w_scale = mats.ws[mi];
    float *__restrict C = mats.C[mi];
    const int N = mats.N[mi];
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    using L = TcSmem<NT>;
    constexpr int kStages = L::kSt;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * L::kStage);
    const uint32_t full0 = tc::smem_u32(bars);                 // [kStages]
    const uint32_t empty0 = tc::smem_u32(bars + kStages);      // [kStages]
    const uint32_t accbar = tc::smem_u32(bars + 2 * kStages);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kStages + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // x = activation tile (fastest): the CTAs that share a weight tile run
    // together, so the tile is read from HBM once and from L2 after
    const int n0 = ((int)blockIdx.y - mats.tile0[mi]) * kBM;
    const int m0 = blockIdx.x * NT;
    const int nk = K / kBK / SPLIT;             // stages of this CTA's K slice
    const int kb0 = blockIdx.z * nk;
    constexpr uint32_t kCols = (2 * NT < 32) ? 32 : 2 * NT;   // power of two >= 32

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, 1);
        }
        tc::mbar_init(accbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tc::prefetch_tmap(tm_w);
        tc::prefetch_tmap(&tm_hi);
        tc::prefetch_tmap(&tm_lo);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), kCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t d_hi = tmem, d_lo = tmem + NT;

    pdl_launch_dependents();
    // an earlier launch timed out: leave before issuing anything
    __shared__ int timed_out_at_entry;
    if (threadIdx.x == 0) timed_out_at_entry = *reinterpret_cast<volatile int *>(&g_gemm_tc_timeout) != 0;
    __syncthreads();
    if (timed_out_at_entry) {
        tc::tc_fence_before();
        __syncthreads();
        if (warp == 1) tc::tmem_dealloc(tmem, kCols);
        return;
    }
    bool ok = true;
    int issued = 0;                 // stages the producer issued (producer thread only)
    if (warp == 0 && lane == 0) {
        // ---- TMA producer (weights first: they do not depend on the previous kernel)
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % kStages;
            if (kb >= kStages) ok = tc::mbar_wait(empty0 + 8 * s, ((kb / kStages) - 1) & 1, &g_gemm_tc_timeout);
            if (!ok) break;
            unsigned char *st = smem + s * L::kStage;
            tc::mbar_expect_tx(full0 + 8 * s, L::kStage);
            tc::tma_load_2d(tc::smem_u32(st), tm_w, (kb0 + kb) * kBK, n0, full0 + 8 * s);
            if (kb == 0) pdl_wait();   // activations come from the previous kernel
            tc::tma_load_2d(tc::smem_u32(st + L::kA), &tm_hi, (kb0 + kb) * kBK, m0, full0 + 8 * s);
            tc::tma_load_2d(tc::smem_u32(st + L::kA + L::kB), &tm_lo, (kb0 + kb) * kBK, m0, full0 + 8 * s);
            issued = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t id_hi = tc::idesc_i8(kBM, NT, true);
        constexpr uint32_t id_lo = tc::idesc_i8(kBM, NT, false);
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % kStages;
            ok = tc::mbar_wait(full0 + 8 * s, (kb / kStages) & 1, &g_gemm_tc_timeout);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t a_base = tc::smem_u32(smem + s * L::kStage);
            const uint32_t h_base = a_base + L::kA;
            const uint32_t l_base = h_base + L::kB;
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
                const uint64_t ad = tc::sdesc_k_sw128(a_base + k * kUmmaK);
                const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                tc::mma_i8(d_hi, ad, tc::sdesc_k_sw128(h_base + k * kUmmaK), id_hi, acc);
                tc::mma_i8(d_lo, ad, tc::sdesc_k_sw128(l_base + k * kUmmaK), id_lo, acc);
            }
            tc::tc_commit(empty0 + 8 * s);   // frees the stage once these MMAs have read it
        }
        tc::tc_commit(accbar);               // accumulators complete
    }
    __syncwarp();

    // ---- epilogue: 4 warps, warp w owns TMEM lanes (weight rows) 32w..32w+31
    pdl_wait();   // activation scales and C belong to the stream order
    __shared__ float as_s[NT];
    for (int i = threadIdx.x; i < NT; i += kThreads) as_s[i] = (m0 + i < M) ? __ldg(a_scale + m0 + i) : 0.0f;
    const int n_row = n0 + warp * 32 + lane;
    const float ws_row = (n_row < N) ? __ldg(w_scale + n_row) : 0.0f;
    __syncthreads();
    const bool acc_ok = tc::mbar_wait(accbar, 0, &g_gemm_tc_timeout);
    tc::tc_fence_after();
    if constexpr (SPLIT == 1) {
        if (acc_ok)
            epilogue_rows<NT>(d_hi, d_lo, (uint32_t)(warp * 32) << 16, as_s, ws_row, n_row, m0, M, N, C, acc);
    } else {
        // partial integer sums of this K slice -> shared memory [NT][128 weight
        // rows] (a warp writes 32 consecutive words: no bank conflicts; the
        // stage ring is idle now), then rank r of the cluster adds the SPLIT
        // partials of weight rows [r*128/SPLIT, (r+1)*128/SPLIT) and finishes
        // them, consecutive threads on consecutive weight rows (contiguous
        // distributed-shared-memory reads, coalesced C stores).
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        static_assert(kBM * NT * 4 <= TcSmem<NT>::kSt * TcSmem<NT>::kStage, "partials exceed the stage ring");
        int32_t *part = reinterpret_cast<int32_t *>(smem);
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const int row = warp * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < NT; c0 += 16) {
            uint32_t hi[16], lo[16];
            tc::tmem_ld16(d_hi + lane_off + c0, hi);
            tc::tmem_ld16(d_lo + lane_off + c0, lo);
            tc::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) part[(c0 + j) * kBM + row] = acc_ok ? (int)(hi[j] * 256u + lo[j]) : 0;
        }
        cluster.sync();
        const int rank = (int)cluster.block_rank();
        constexpr int kRows = kBM / SPLIT;
        for (int e = threadIdx.x; e < kRows * NT; e += kThreads) {
            const int r = rank * kRows + e % kRows, j = e / kRows;
            uint32_t S = 0;
#pragma unroll
            for (int k = 0; k < SPLIT; ++k) S += (uint32_t)cluster.map_shared_rank(part, k)[j * kBM + r];
            const int n = n0 + r, m = m0 + j;
            if (acc_ok && m < M && n < N) {
                const float p = mul_rn(__int2float_rn((int)S), as_s[j]);
                const float v = fma_rn(p, __ldg(w_scale + n), 0.0f);
                float *cp = C + (size_t)m * N + n;
                *cp = acc ? add_rn(*cp, v) : v;
            }
        }
        cluster.sync();   // partials stay alive until every rank has read them
    }
    if (warp == 0 && lane == 0 && !ok) {
        // the producer gave up: wait (bounded) for the copies it already
        // issued, so none lands in shared memory after the CTA has left
        for (int kb = issued - 1; kb >= 0 && kb >= issued - kStages; --kb)
            tc::mbar_wait(full0 + 8 * (kb % kStages), (kb / kStages) & 1, nullptr);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kCols);
}

// Persistent form for large products (M >= 512, many tiles): one CTA per SM
// walks the tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... (activation
// tile fastest, so the CTAs working at the same time share weight tiles in
// L2).  Warp 0 issues the TMA loads of a 4-stage ring across tile boundaries,
// warp 1 the MMAs, and warps 2-5 drain the accumulators; the accumulators are
// double-buffered in tensor memory (2 x hi/lo x NT columns = all 512 columns
// at NT = 128), so the epilogue of tile i overlaps the main loop of tile i+1.
// Same arithmetic as gemm_i8_tc_kernel (exact int32 sums, the reference's fp32
// epilogue); every wait is bounded.
constexpr int kPersistThreads = 192;
template <int NT>
struct TcPersistSmem {
    static constexpr int kA = kBM * kBK;
    static constexpr int kB = NT * kBK;
    static constexpr int kStage = kA + 2 * kB;
    static constexpr int kSt = 4;
    static constexpr int kBytes = kSt * kStage + 1024 + 256;
};

template <int NT>
__global__ void __launch_bounds__(kPersistThreads, 1)
gemm_i8_tc_persistent(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_hi,
                      const __grid_constant__ CUtensorMap tm_lo, const float *__restrict a_scale,
                      const float *__restrict w_scale, float *__restrict C, int M, int N, int K, int acc) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    using L = TcPersistSmem<NT>;
    constexpr int kS = L::kSt;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kS * L::kStage);
    const uint32_t full0 = tc::smem_u32(bars);                 // [kS]
    const uint32_t empty0 = tc::smem_u32(bars + kS);           // [kS]
    const uint32_t tfull0 = tc::smem_u32(bars + 2 * kS);       // [2] accumulator b complete
    const uint32_t tempty0 = tc::smem_u32(bars + 2 * kS + 2);  // [2] accumulator b drained
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kS + 4);
    __shared__ int timed_out_at_entry;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + NT - 1) / NT, ntl = (N + kBM - 1) / kBM;
    const int tiles = mt * ntl;
    const int nk = K / kBK;
    constexpr uint32_t kCols = 4 * NT;           // 2 buffers x (hi, lo)

    if (threadIdx.x == 0) {
        timed_out_at_entry = *reinterpret_cast<volatile int *>(&g_gemm_tc_timeout) != 0;
        for (int i = 0; i < kS; ++i) {
            tc::mbar_init(full0 + 8 * i, 1);
            tc::mbar_init(empty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(tfull0 + 8 * b, 1);
            tc::mbar_init(tempty0 + 8 * b, 4);    // one elected lane per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tc::prefetch_tmap(&tm_w);
        tc::prefetch_tmap(&tm_hi);
        tc::prefetch_tmap(&tm_lo);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), kCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    bool ok = !timed_out_at_entry;
    int issued = 0;

    if (warp == 0) {
        if (lane == 0 && ok) {
            int kk = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (t % mt) * NT, n0 = (t / mt) * kBM;
                for (int kb = 0; kb < nk && ok; ++kb, ++kk) {
                    const int s = kk % kS;
                    if (kk >= kS) ok = tc::mbar_wait(empty0 + 8 * s, ((kk / kS) - 1) & 1, &g_gemm_tc_timeout);
                    if (!ok) break;
                    unsigned char *st = smem + s * L::kStage;
                    tc::mbar_expect_tx(full0 + 8 * s, L::kStage);
                    tc::tma_load_2d(tc::smem_u32(st), &tm_w, kb * kBK, n0, full0 + 8 * s);
                    if (kk == 0) pdl_wait();   // activations come from the previous kernel
                    tc::tma_load_2d(tc::smem_u32(st + L::kA), &tm_hi, kb * kBK, m0, full0 + 8 * s);
                    tc::tma_load_2d(tc::smem_u32(st + L::kA + L::kB), &tm_lo, kb * kBK, m0, full0 + 8 * s);
                    issued = kk + 1;
                }
            }
            if (!ok) {
                // wait (bounded) for the copies already issued, so that none
                // lands in shared memory after the CTA has left
                for (int k2 = issued - 1; k2 >= 0 && k2 >= issued - kS; --k2)
                    tc::mbar_wait(full0 + 8 * (k2 % kS), (k2 / kS) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && ok) {
            constexpr uint32_t id_hi = tc::idesc_i8(kBM, NT, true);
            constexpr uint32_t id_lo = tc::idesc_i8(kBM, NT, false);
            int kk = 0, i = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
                const int b = i & 1, u = i >> 1;
                if (u >= 1) ok = tc::mbar_wait(tempty0 + 8 * b, (u - 1) & 1, &g_gemm_tc_timeout);
                if (!ok) break;
                tc::tc_fence_after();
                const uint32_t d_hi = tmem + (uint32_t)(b * 2 * NT), d_lo = d_hi + NT;
                for (int kb = 0; kb < nk && ok; ++kb, ++kk) {
                    const int s = kk % kS;
                    ok = tc::mbar_wait(full0 + 8 * s, (kk / kS) & 1, &g_gemm_tc_timeout);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint32_t a_base = tc::smem_u32(smem + s * L::kStage);
                    const uint32_t h_base = a_base + L::kA;
                    const uint32_t l_base = h_base + L::kB;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        const uint64_t ad = tc::sdesc_k_sw128(a_base + k * kUmmaK);
                        const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
                        tc::mma_i8(d_hi, ad, tc::sdesc_k_sw128(h_base + k * kUmmaK), id_hi, accum);
                        tc::mma_i8(d_lo, ad, tc::sdesc_k_sw128(l_base + k * kUmmaK), id_lo, accum);
                    }
                    tc::tc_commit(empty0 + 8 * s);
                }
                if (ok) tc::tc_commit(tfull0 + 8 * b);
            }
        }
    } else {
        // epilogue warps 2..5: TMEM lanes 32 * (warp % 4) .. + 31 = weight rows;
        // each warp stages the tile's activation scales in its own as_s[.][b]
        // (no block barrier, whose wait could not be bounded) before the
        // accumulators are waited for
        __shared__ float as_s[4][2][NT];
        pdl_wait();
        const int q4 = warp & 3;
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        int i = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
            const int m0 = (t % mt) * NT, n0 = (t / mt) * kBM;
            const int b = i & 1, u = i >> 1;
            for (int r = lane; r < NT; r += 32) as_s[q4][b][r] = (m0 + r < M) ? __ldg(a_scale + m0 + r) : 0.0f;
            const int n = n0 + q4 * 32 + lane;
            const float ws = (n < N) ? __ldg(w_scale + n) : 0.0f;
            __syncwarp();
            ok = tc::mbar_wait(tfull0 + 8 * b, u & 1, &g_gemm_tc_timeout);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t d_hi = tmem + (uint32_t)(b * 2 * NT), d_lo = d_hi + NT;
            epilogue_rows<NT>(d_hi, d_lo, lane_off, as_s[q4][b], ws, n, m0, M, N, C, acc);
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(tempty0 + 8 * b);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kCols);
}

// Group-wise weight scales (g in {32, 64} or a multiple of 128, g < K): the
// reference's M > 1 order per output is acc = fma(float(S_g) * a_s[m, g],
// w_s[n, g], acc) over the groups in ascending order, S_g the exact integer
// sum of group g.  A "unit" is what one accumulator set holds: one group when
// g >= 128 (g / 128 stages of K), else the GPK = 128 / g groups of one stage.
// Each unit's hi/lo sums go to their own TMEM columns (GPK x 2 x NT per
// buffer, two buffers); eight epilogue warps (two per TMEM lane quarter, each
// taking half of the tile's columns) drain every unit as soon as it is
// complete and keep the fp32 chains in registers, so the integer sums of unit
// u+1 run on the tensor cores while unit u is scaled.  Persistent over tiles
// like gemm_i8_tc_persistent; every wait is bounded, no block barrier inside
// the loops.
constexpr int kGroupedThreads = 320;   // producer, MMA, 8 epilogue warps
template <int NT>
struct TcGroupedSmem {
    static constexpr int kA = kBM * kBK;
    static constexpr int kB = NT * kBK;
    static constexpr int kStage = kA + 2 * kB;
    static constexpr int kSt = (192 * 1024) / kStage;
    static constexpr int kBytes = kSt * kStage + 1024 + 256;
};

template <int NT, int GPK>
__global__ void __launch_bounds__(kGroupedThreads, 1)
gemm_i8_tc_grouped(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_hi,
                   const __grid_constant__ CUtensorMap tm_lo, const float *__restrict a_scale,
                   const float *__restrict w_scale, float *__restrict C, int M, int N, int K, int g, int acc) {
    static_assert(GPK * NT <= 128 && (GPK == 1 || GPK == 2 || GPK == 4), "unit exceeds 256 TMEM columns");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    using L = TcGroupedSmem<NT>;
    constexpr int kS = L::kSt;
    constexpr int kHalf = NT / 2;                       // columns per epilogue warp
    constexpr uint32_t kBuf = GPK * 2 * NT;             // TMEM columns per unit buffer
    constexpr uint32_t kCols = 2 * kBuf < 32 ? 32 : 2 * kBuf;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kS * L::kStage);
    const uint32_t full0 = tc::smem_u32(bars);
    const uint32_t empty0 = tc::smem_u32(bars + kS);
    const uint32_t tfull0 = tc::smem_u32(bars + 2 * kS);
    const uint32_t tempty0 = tc::smem_u32(bars + 2 * kS + 2);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kS + 4);
    __shared__ int timed_out_at_entry;
    __shared__ float as_w[8][GPK * kHalf];              // per epilogue warp: this unit's activation scales

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (M + NT - 1) / NT, ntl = (N + kBM - 1) / kBM;
    const int tiles = mt * ntl;
    const int G = K / g;
    const int units = G / GPK;                         // per tile
    const int kpu = GPK == 1 ? g / kBK : 1;            // stages per unit

    if (threadIdx.x == 0) {
        timed_out_at_entry = *reinterpret_cast<volatile int *>(&g_gemm_tc_timeout) != 0;
        for (int i = 0; i < kS; ++i) {
            tc::mbar_init(full0 + 8 * i, 1);
            tc::mbar_init(empty0 + 8 * i, 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(tfull0 + 8 * b, 1);
            tc::mbar_init(tempty0 + 8 * b, 8);    // one elected lane per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tc::prefetch_tmap(&tm_w);
        tc::prefetch_tmap(&tm_hi);
        tc::prefetch_tmap(&tm_lo);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), kCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    bool ok = !timed_out_at_entry;
    const int nk = K / kBK;

    if (warp == 0) {
        if (lane == 0 && ok) {
            int kk = 0, issued = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (t % mt) * NT, n0 = (t / mt) * kBM;
                for (int kb = 0; kb < nk && ok; ++kb, ++kk) {
                    const int s = kk % kS;
                    if (kk >= kS) ok = tc::mbar_wait(empty0 + 8 * s, ((kk / kS) - 1) & 1, &g_gemm_tc_timeout);
                    if (!ok) break;
                    unsigned char *st = smem + s * L::kStage;
                    tc::mbar_expect_tx(full0 + 8 * s, L::kStage);
                    tc::tma_load_2d(tc::smem_u32(st), &tm_w, kb * kBK, n0, full0 + 8 * s);
                    if (kk == 0) pdl_wait();
                    tc::tma_load_2d(tc::smem_u32(st + L::kA), &tm_hi, kb * kBK, m0, full0 + 8 * s);
                    tc::tma_load_2d(tc::smem_u32(st + L::kA + L::kB), &tm_lo, kb * kBK, m0, full0 + 8 * s);
                    issued = kk + 1;
                }
            }
            if (!ok)
                for (int k2 = issued - 1; k2 >= 0 && k2 >= issued - kS; --k2)
                    tc::mbar_wait(full0 + 8 * (k2 % kS), (k2 / kS) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0 && ok) {
            constexpr uint32_t id_hi = tc::idesc_i8(kBM, NT, true);
            constexpr uint32_t id_lo = tc::idesc_i8(kBM, NT, false);
            constexpr int kPerGroup = (kBK / kUmmaK) / GPK;   // MMA K steps per group inside a stage
            int kk = 0, u = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                for (int uu = 0; uu < units && ok; ++uu, ++u) {
                    const int b = u & 1;
                    if (u >= 2) ok = tc::mbar_wait(tempty0 + 8 * b, ((u >> 1) - 1) & 1, &g_gemm_tc_timeout);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint32_t dbase = tmem + (uint32_t)b * kBuf;
                    for (int kq = 0; kq < kpu && ok; ++kq, ++kk) {
                        const int s = kk % kS;
                        ok = tc::mbar_wait(full0 + 8 * s, (kk / kS) & 1, &g_gemm_tc_timeout);
                        if (!ok) break;
                        tc::tc_fence_after();
                        const uint32_t a_base = tc::smem_u32(smem + s * L::kStage);
                        const uint32_t h_base = a_base + L::kA;
                        const uint32_t l_base = h_base + L::kB;
#pragma unroll
                        for (int k = 0; k < kBK / kUmmaK; ++k) {
                            const int gk = k / kPerGroup;
                            const uint32_t d_hi = dbase + (uint32_t)(gk * 2 * NT), d_lo = d_hi + NT;
                            const uint32_t accum = GPK == 1 ? ((kq > 0 || k > 0) ? 1u : 0u)
                                                            : ((k % kPerGroup) != 0 ? 1u : 0u);
                            const uint64_t ad = tc::sdesc_k_sw128(a_base + k * kUmmaK);
                            tc::mma_i8(d_hi, ad, tc::sdesc_k_sw128(h_base + k * kUmmaK), id_hi, accum);
                            tc::mma_i8(d_lo, ad, tc::sdesc_k_sw128(l_base + k * kUmmaK), id_lo, accum);
                        }
                        tc::tc_commit(empty0 + 8 * s);
                    }
                    if (ok) tc::tc_commit(tfull0 + 8 * b);
                }
            }
        }
    } else {
        // epilogue warps 2..9: TMEM lane quarter warp % 4, column half (warp - 2) / 4
        pdl_wait();
        const int we = warp - 2, q4 = warp & 3, h = we >> 2;
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        float *asw = as_w[we];
        int u = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const int m0 = (t % mt) * NT, n0 = (t / mt) * kBM;
            const int n = n0 + q4 * 32 + lane;
            const int mc = m0 + h * kHalf;                 // this warp's first column
            float accv[kHalf];
#pragma unroll
            for (int j = 0; j < kHalf; ++j) accv[j] = 0.0f;
            for (int uu = 0; uu < units && ok; ++uu, ++u) {
                const int b = u & 1;
                // this unit's scales: a_s[m, gi] for the warp's columns, w_s[n, gi]
                __syncwarp();
                for (int e = lane; e < GPK * kHalf; e += 32) {
                    const int gk = e / kHalf, m = mc + e % kHalf;
                    asw[e] = m < M ? __ldg(a_scale + (size_t)m * G + uu * GPK + gk) : 0.0f;
                }
                float wsg[GPK];
#pragma unroll
                for (int gk = 0; gk < GPK; ++gk) wsg[gk] = n < N ? __ldg(w_scale + (size_t)n * G + uu * GPK + gk) : 0.0f;
                __syncwarp();
                ok = tc::mbar_wait(tfull0 + 8 * b, (u >> 1) & 1, &g_gemm_tc_timeout);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (int gk = 0; gk < GPK; ++gk) {
                    const uint32_t dh = tmem + (uint32_t)b * kBuf + (uint32_t)(gk * 2 * NT + h * kHalf) + lane_off;
#pragma unroll
                    for (int c0 = 0; c0 < kHalf; c0 += 16) {
                        uint32_t hi[16], lo[16];
                        tc::tmem_ld16(dh + c0, hi);
                        tc::tmem_ld16(dh + NT + c0, lo);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int S = (int)(hi[j] * 256u + lo[j]);
                            const float p = mul_rn(__int2float_rn(S), asw[gk * kHalf + c0 + j]);
                            accv[c0 + j] = fma_rn(p, wsg[gk], accv[c0 + j]);
                        }
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cta(tempty0 + 8 * b);
            }
            if (!ok) break;
            if (n < N) {
#pragma unroll
                for (int j = 0; j < kHalf; ++j) {
                    const int m = mc + j;
                    if (m < M) {
                        float *cp = C + (size_t)m * N + n;
                        *cp = acc ? add_rn(*cp, accv[j]) : accv[j];
                    }
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kCols);
}

// q int16 [M, K] -> hi int8 [M, K] (q >> 8), lo uint8 [M, K] (q & 255).
__global__ void split_hi_lo_kernel(const int16_t *__restrict q, int8_t *__restrict hi, uint8_t *__restrict lo,
                                   long n) {
    pdl_launch_dependents();
    pdl_wait();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n / 8; i += (long)gridDim.x * blockDim.x) {
        const int4 v = reinterpret_cast<const int4 *>(q)[i];
        const int16_t *e = reinterpret_cast<const int16_t *>(&v);
        uint2 h, l;
        unsigned char *hb = reinterpret_cast<unsigned char *>(&h);
        unsigned char *lb = reinterpret_cast<unsigned char *>(&l);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            hb[j] = (unsigned char)(e[j] >> 8);
            lb[j] = (unsigned char)(e[j] & 255);
        }
        reinterpret_cast<uint2 *>(hi)[i] = h;
        reinterpret_cast<uint2 *>(lo)[i] = l;
    }
}

// ---------------------------------------------------------------- host side
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled get_encode() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// 2-D uint8 tensor [rows, cols] (cols contiguous), box {128 bytes, box_rows}, 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiled enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int SPLIT>
cudaError_t launch_nt(const TcMats &mats, const CUtensorMap &mh, const CUtensorMap &ml, const float *as, int M,
                      int K, int acc, cudaStream_t st) {
    auto kern = gemm_i8_tc_kernel<NT, SPLIT>;
    const int smem = TcSmem<NT>::kBytes;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + NT - 1) / NT, mats.tile0[mats.n], SPLIT);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = SPLIT;
    cfg.attrs = attr;
    cfg.numAttrs = SPLIT > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, mats, mh, ml, as, M, K, acc);
}

template <int NT>
cudaError_t launch_split(int split, const TcMats &mats, const CUtensorMap &mh, const CUtensorMap &ml,
                         const float *as, int M, int K, int acc, cudaStream_t st) {
    switch (split) {
        case 8: return launch_nt<NT, 8>(mats, mh, ml, as, M, K, acc, st);
        case 4: return launch_nt<NT, 4>(mats, mh, ml, as, M, K, acc, st);
        case 2: return launch_nt<NT, 2>(mats, mh, ml, as, M, K, acc, st);
        default: return launch_nt<NT, 1>(mats, mh, ml, as, M, K, acc, st);
    }
}

template <int NT>
cudaError_t launch_persistent(const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &ml, const float *as,
                              const float *ws, float *C, int M, int N, int K, int acc, cudaStream_t st) {
    auto kern = gemm_i8_tc_persistent<NT>;
    const int smem = TcPersistSmem<NT>::kBytes;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long tiles = (long)((M + NT - 1) / NT) * ((N + kBM - 1) / kBM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles < sms ? tiles : sms));
    cfg.blockDim = dim3(kPersistThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, mw, mh, ml, as, ws, C, M, N, K, acc);
}

template <int NT, int GPK>
cudaError_t launch_grouped(const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &ml, const float *as,
                           const float *ws, float *C, int M, int N, int K, int g, int acc, cudaStream_t st) {
    auto kern = gemm_i8_tc_grouped<NT, GPK>;
    const int smem = TcGroupedSmem<NT>::kBytes;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long tiles = (long)((M + NT - 1) / NT) * ((N + kBM - 1) / kBM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles < sms ? tiles : sms));
    cfg.blockDim = dim3(kGroupedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, mw, mh, ml, as, ws, C, M, N, K, g, acc);
}

}  // namespace

int *gemm_tc_timeout_word() {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_tc_timeout) != cudaSuccess) return nullptr;
    return static_cast<int *>(p);
}

// QVL_GEMM_PERSIST=0 in the environment keeps the one-tile-per-CTA kernel.
static bool persist_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("QVL_GEMM_PERSIST");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

bool gemm_tc_grouped_size(size_t g, size_t K) {
    return g < K && (g == 32 || g == 64 || (g % kBK == 0 && K % g == 0));
}

bool gemm_tc_supported(size_t M, size_t N, size_t K, size_t g) {
    return M >= 16 && (g == K || gemm_tc_grouped_size(g, K)) && K % kBK == 0 && N >= kBM && (N + kBM - 1) / kBM <= 65535 && get_encode() != nullptr;
}

size_t gemm_tc_planes_bytes(size_t M, size_t K) { return 2 * ((M * K + 255) & ~(size_t)255); }

cudaError_t launch_split_hi_lo(const int16_t *q, int8_t *hi, uint8_t *lo, int M, int K, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    const long n = (long)M * K;
    long blocks = (n / 8 + 255) / 256;
    cfg.gridDim = dim3((unsigned)(blocks < 148 * 8 ? blocks : 148 * 8));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, split_hi_lo_kernel, q, hi, lo, n);
}

cudaError_t launch_gemm_i8_tc_planes(const int8_t *hi, const uint8_t *lo, const float *qs, const int8_t *W,
                                     const float *ws, float *C, int M, int N, int K, int acc,
                                     cudaStream_t stream, int g) {
    if (g != 0 && g != K) {
        // group-wise scales: groups per stage GPK = 128 / g (1 from g = 128);
        // the widest activation tile that fits the unit's TMEM columns,
        // narrowed while the tiles would not cover the GPU
        const int gpk = g >= kBK ? 1 : kBK / g;
        int NT = 128 / gpk;
        while (NT > 32 && (long)((M + NT - 1) / NT) * ((N + kBM - 1) / kBM) < 148) NT /= 2;
        CUtensorMap mw, mh, ml;
        if (!make_map(&mw, W, N, K, kBM) || !make_map(&mh, hi, M, K, NT) || !make_map(&ml, lo, M, K, NT))
            return cudaErrorInvalidValue;
        if (gpk == 1) {
            if (NT == 128) return launch_grouped<128, 1>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
            if (NT == 64) return launch_grouped<64, 1>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
            return launch_grouped<32, 1>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
        }
        if (gpk == 2) {
            if (NT == 64) return launch_grouped<64, 2>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
            return launch_grouped<32, 2>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
        }
        return launch_grouped<32, 4>(mw, mh, ml, qs, ws, C, M, N, K, g, acc, stream);
    }
    const int8_t *Ws[1] = {W};
    const float *wss[1] = {ws};
    float *Cs[1] = {C};
    const int Ns[1] = {N};
    return launch_gemm_i8_tc_planes_multi(hi, lo, qs, 1, Ws, wss, Cs, Ns, M, K, acc, stream);
}

cudaError_t launch_gemm_i8_tc_planes_multi(const int8_t *hi, const uint8_t *lo, const float *qs, int n_mats,
                                           const int8_t *const *W, const float *const *ws, float *const *C,
                                           const int *N, int M, int K, int acc, cudaStream_t stream) {
    if (n_mats < 1 || n_mats > kMaxMats) return cudaErrorInvalidValue;
    // Activation tile: 128 rows from M >= 256 (64 from 64, else 32).  A
    // single product of two or more waves of 128 x 128 tiles runs on the
    // persistent kernel; the others (and every multi-matrix launch) split K
    // over a cluster until there are ~2 CTAs per SM (exact int32 partial
    // sums, added through distributed shared memory).
    const int NT = M >= 256 ? 128 : (M >= 64 ? 64 : 32);
    CUtensorMap mh, ml;
    if (!make_map(&mh, hi, M, K, NT) || !make_map(&ml, lo, M, K, NT)) return cudaErrorInvalidValue;
    TcMats mats = {};
    mats.n = n_mats;
    mats.tile0[0] = 0;
    for (int i = 0; i < n_mats; ++i) {
        if (!make_map(&mats.w[i], W[i], N[i], K, kBM)) return cudaErrorInvalidValue;
        mats.ws[i] = ws[i];
        mats.C[i] = C[i];
        mats.N[i] = N[i];
        mats.tile0[i + 1] = mats.tile0[i] + (N[i] + kBM - 1) / kBM;
    }
    const long tiles = (long)mats.tile0[n_mats] * ((M + NT - 1) / NT);
    if (n_mats == 1 && NT == 128 && tiles >= 2 * 148 && persist_enabled())
        return launch_persistent<128>(mats.w[0], mh, ml, qs, ws[0], C[0], M, N[0], K, acc, stream);
    const int nkb = K / kBK;
    int split = 1;
    while (split < 8 && tiles * split * 2 <= 2 * 148 && nkb % (split * 2) == 0) split *= 2;
    if (NT == 128) return launch_split<128>(split, mats, mh, ml, qs, M, K, acc, stream);
    if (NT == 64) return launch_split<64>(split, mats, mh, ml, qs, M, K, acc, stream);
    return launch_split<32>(split, mats, mh, ml, qs, M, K, acc, stream);
}

cudaError_t launch_gemm_i8_tc(const int16_t *q, const float *qs, int8_t *hi, uint8_t *lo, const int8_t *W,
                              const float *ws, float *C, int M, int N, int K, cudaStream_t stream) {
    cudaError_t e = launch_split_hi_lo(q, hi, lo, M, K, stream);
    if (e != cudaSuccess) return e;
    return launch_gemm_i8_tc_planes(hi, lo, qs, W, ws, C, M, N, K, 0, stream);
}

}  // namespace qvl
