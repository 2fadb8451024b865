// GQA decode attention in the reference's own summation order, bit for bit
// (given the same fp16-valued cache): attn_scores_all_heads, softmax and
// attn_weighted_sum_all_heads, layers/src/text_layer.cpp:436-710.
//
//   scores   t < 8*(pos/8): 8 fused lanes over d = l, l+8, ... (:590-633),
//            then add_reduce_mm_256_layer ((v_i + v_{i+4}), two hadds);
//            the 0-7 tail (:636-645): 8 unfused lanes added 0..7 in order
//            (what g++ makes of `#pragma omp simd reduction(+:score)`);
//            times 1/sqrtf(D).
//   softmax  max; for t < 8*(n/8): exp256_ps(s - max), masked where s is
//            -inf, summed into 8 float lanes t-ascending, the lanes added in
//            double 0..7; then the tail, each term added in double; p = e *
//            (float)(1/sum) (:436-535).
//   P.V      out[h][d] = one fma chain over t ascending (:677-689).
//
// Two launches: scores (one thread per token and KV head, every score of the
// KV head's query heads) into a caller workspace, then one CTA per (query,
// head) for the softmax and the 128 P.V chains (one thread per d).  The
// chains are sequential by construction -- this path trades the split
// context of qvl_attention_decode for exact agreement with the reference.
#include <cuda_fp16.h>
#include "common.cuh"
#include "attention_ordered.cuh"

namespace qvl {

namespace {
constexpr int kD = 128;
constexpr int kThreads = 128;

__device__ __forceinline__ size_t kv_index(const int32_t *pt_row, int t, int kvh, int NKV, int P) {
    const int pg = t / P;
    return (((size_t)pt_row[pg] * NKV + kvh) * P + (t - pg * P)) * kD;
}
}  // namespace

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kKRow = kD * 2 + 16;     // staged key row: 256 B + 16 B of padding (no bank conflicts)

// grid (ceil(max_ctx / 128), NKV, nq); block 128; dynamic smem: the KV
// head's query rows (kv_mul * 128 floats), then the block's 128 key rows.
// The key rows are staged with contiguous 16-byte cp.async copies (16
// threads per row) and each thread then reads its own row from shared memory.
// ROPE: the query rows are the raw q/k/v projections of a decode step (one
// query per sequence).  Every CTA applies the QK-norm and RoPE of its KV
// head's query heads itself (rope_append_kernel's arithmetic, attention.cu);
// the CTA whose block holds the query's position also normalises and rotates
// the new key, appends key and value to the pages as fp16 and puts the key
// row straight into its staging area.  One launch less per layer; the cache
// row at the position is not read before it is written.
template <int KVM, bool ROPE>
__global__ void __launch_bounds__(kThreads, 6)
attn_ordered_scores_kernel(const float *__restrict q, const uint16_t *__restrict k_pages,
                           const int32_t *__restrict page_table, const int32_t *__restrict seq_ids,
                           const int32_t *__restrict positions, float *__restrict scores, int max_ctx, int NH,
                           int NKV, int P, int maxp, OrdRope rp) {
    extern __shared__ __align__(16) float qs[];
    pdl_launch_dependents();
    // ROPE (a decode step): the cached key rows before the position are
    // complete when the call is made, so they are staged before the
    // dependent-launch wait; the projections are read after it
    if (!ROPE) pdl_wait();
    const int i = blockIdx.z, kvh = blockIdx.y;
    constexpr int kvm = KVM;
    const int pos = positions[i];
    const int t0 = blockIdx.x * kThreads;
    if (pos < 0 || pos >= max_ctx || t0 > pos) return;
    const bool owner = ROPE && pos < t0 + kThreads;     // this block holds the new position
    float *kraw = qs + kvm * kD;                          // ROPE: the new key row
    unsigned char *ks = reinterpret_cast<unsigned char *>(qs + (ROPE ? kvm + 1 : kvm) * kD);
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * maxp;
    const int rows = min(kThreads, pos + 1 - t0);
    __shared__ size_t rowoff[kThreads];     // 16-byte index of each staged key row (one page lookup per row)
    if (threadIdx.x < rows) rowoff[threadIdx.x] = kv_index(pt_row, t0 + threadIdx.x, kvh, NKV, P) / 8;
    __syncthreads();
    const uint4 *kp = reinterpret_cast<const uint4 *>(k_pages);
    const int staged = owner ? rows - 1 : rows;           // the position's row comes from registers
    for (int e = threadIdx.x; e < staged * 16; e += kThreads) {
        const int r = e >> 4, c = e & 15;
        cp_async16(ks + r * kKRow + c * 16, kp + rowoff[r] + c);
    }
    cp_async_commit();
    if (ROPE) pdl_wait();
    for (int e = threadIdx.x; e < kvm * kD; e += blockDim.x) qs[e] = q[((size_t)i * NH + kvh * kvm) * kD + e];
    if constexpr (ROPE) {
        constexpr int half = kD / 2;
        const int nr = owner ? kvm + 1 : kvm;             // rows to normalise and rotate
        if (owner) {
            kraw[threadIdx.x] = rp.k_new[((size_t)i * NKV + kvh) * kD + threadIdx.x];
            const size_t off = rowoff[pos - t0] * 8 + threadIdx.x;
            rp.v_pages[off] = __half_as_ushort(__float2half_rn(rp.v_new[((size_t)i * NKV + kvh) * kD + threadIdx.x]));
        }
        __syncthreads();
        if (rp.norm.q_w) {
            __shared__ float red[(KVM + 1) * 8];
            __shared__ float invh[KVM + 1];
            if (threadIdx.x < nr * 8) {
                const int h = threadIdx.x >> 3, l = threadIdx.x & 7;
                const float *xh = qs + h * kD;
                float acc = 0.0f;
#pragma unroll
                for (int j = 0; j < kD; j += 8) acc = add_rn(acc, mul_rn(xh[j + l], xh[j + l]));
                red[threadIdx.x] = acc;
            }
            __syncthreads();
            if (threadIdx.x < nr) {
                float ss = 0.0f;
#pragma unroll
                for (int l = 0; l < 8; ++l) ss = add_rn(ss, red[threadIdx.x * 8 + l]);
                const float a = fma_rn(ss, __fdiv_rn(1.0f, (float)kD), rp.norm.eps);
                invh[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(a));
            }
            __syncthreads();
            for (int e = threadIdx.x; e < nr * kD; e += blockDim.x) {
                const int h = e / kD, j = e - h * kD;
                const bool isq = h < kvm;
                const int8_t *w = isq ? rp.norm.q_w : rp.norm.k_w;
                const float *ws = isq ? rp.norm.q_s : rp.norm.k_s;
                qs[e] = mul_rn((float)w[j], mul_rn(mul_rn(ws[j / rp.norm.gs], invh[h]), qs[e]));
            }
            __syncthreads();
        }
        const float *c = rp.rope_cos + (size_t)pos * half;
        const float *sn = rp.rope_sin + (size_t)pos * half;
        for (int e = threadIdx.x; e < nr * half; e += blockDim.x) {
            const int h = e / half, j = e - h * half;
            float *x = qs + h * kD;
            const float x1 = x[j], x2 = x[j + half];
            const float y1 = fma_rn(x1, c[j], -mul_rn(x2, sn[j]));
            const float y2 = fma_rn(x1, sn[j], mul_rn(x2, c[j]));
            if (h < kvm) {
                x[j] = y1;
                x[j + half] = y2;
            } else {
                const uint16_t k1 = __half_as_ushort(__float2half_rn(y1)), k2 = __half_as_ushort(__float2half_rn(y2));
                const size_t off = rowoff[pos - t0] * 8;
                rp.k_pages[off + j] = k1;
                rp.k_pages[off + j + half] = k2;
                uint16_t *kr = reinterpret_cast<uint16_t *>(ks + (pos - t0) * kKRow);
                kr[j] = k1;
                kr[j + half] = k2;
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t > pos) return;
    const uint4 *kr = reinterpret_cast<const uint4 *>(ks + threadIdx.x * kKRow);
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)kD));
    const bool tail = t >= (pos / 8) * 8;
    // the KVM heads' 8-lane chains advance together, 8 key values at a time
    // (each head's chain in its own order: lane l over d = l, l+8, ...)
    float l8[KVM][8];
#pragma unroll
    for (int hh = 0; hh < KVM; ++hh)
#pragma unroll
        for (int l = 0; l < 8; ++l) l8[hh][l] = 0.0f;
#pragma unroll
    for (int c = 0; c < kD / 8; ++c) {
        const uint4 v = kr[c];
        const __half2 *hv = reinterpret_cast<const __half2 *>(&v);
        float kc[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(hv[j]);
            kc[2 * j] = f.x;
            kc[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int hh = 0; hh < KVM; ++hh) {
            const float4 qa = reinterpret_cast<const float4 *>(qs + hh * kD + 8 * c)[0];
            const float4 qb = reinterpret_cast<const float4 *>(qs + hh * kD + 8 * c)[1];
            if (!tail) {
                l8[hh][0] = fma_rn(qa.x, kc[0], l8[hh][0]);
                l8[hh][1] = fma_rn(qa.y, kc[1], l8[hh][1]);
                l8[hh][2] = fma_rn(qa.z, kc[2], l8[hh][2]);
                l8[hh][3] = fma_rn(qa.w, kc[3], l8[hh][3]);
                l8[hh][4] = fma_rn(qb.x, kc[4], l8[hh][4]);
                l8[hh][5] = fma_rn(qb.y, kc[5], l8[hh][5]);
                l8[hh][6] = fma_rn(qb.z, kc[6], l8[hh][6]);
                l8[hh][7] = fma_rn(qb.w, kc[7], l8[hh][7]);
            } else {
                l8[hh][0] = add_rn(l8[hh][0], mul_rn(qa.x, kc[0]));
                l8[hh][1] = add_rn(l8[hh][1], mul_rn(qa.y, kc[1]));
                l8[hh][2] = add_rn(l8[hh][2], mul_rn(qa.z, kc[2]));
                l8[hh][3] = add_rn(l8[hh][3], mul_rn(qa.w, kc[3]));
                l8[hh][4] = add_rn(l8[hh][4], mul_rn(qb.x, kc[4]));
                l8[hh][5] = add_rn(l8[hh][5], mul_rn(qb.y, kc[5]));
                l8[hh][6] = add_rn(l8[hh][6], mul_rn(qb.z, kc[6]));
                l8[hh][7] = add_rn(l8[hh][7], mul_rn(qb.w, kc[7]));
            }
        }
    }
#pragma unroll
    for (int hh = 0; hh < KVM; ++hh) {
        float r;
        if (!tail) {
            // reduce8_ref's order: (v0+v4, v1+v5, v2+v6, v3+v7), then (u0+u1)+(u2+u3)
            const float u0 = add_rn(l8[hh][0], l8[hh][4]), u1 = add_rn(l8[hh][1], l8[hh][5]);
            const float u2 = add_rn(l8[hh][2], l8[hh][6]), u3 = add_rn(l8[hh][3], l8[hh][7]);
            r = add_rn(add_rn(u0, u1), add_rn(u2, u3));
        } else {
            r = l8[hh][0];
#pragma unroll
            for (int l = 1; l < 8; ++l) r = add_rn(r, l8[hh][l]);
            r = add_rn(0.0f, r);
        }
        scores[((size_t)i * NH + kvh * KVM + hh) * max_ctx + t] = mul_rn(r, inv_sqrt_d);
    }
}

constexpr int kSumChunk = 1024;    // exponentials staged per pass of the lane sums (per query head)
constexpr int kPvChunk = 64;       // V rows per P.V stage (16 KB)
// stages in flight (cp.async ring): 4, or 2 when there are many queries
// (more CTAs resident per SM outweigh the shallower ring: a 452-token
// causal prompt pass)
constexpr int kPvStagesMax = 4;
// Few queries and short contexts (a decode batch): 5 stages, 4 in flight; the
// shared memory (~90 KB) still lets two CTAs share an SM
constexpr int kPvStagesDeep = 5;
constexpr int kPvDeepCtx = 1024;
constexpr int kPvManyQueries = 64;

template <int KVM, int kPvStages>
struct PvSmem {
    static constexpr size_t kV = (size_t)kPvStages * kPvChunk * kD * 2;        // fp16 V rows
    static constexpr size_t kP = (size_t)kPvStages * KVM * kPvChunk * 4;       // probabilities (global path)
    static constexpr size_t kE = (size_t)KVM * kSumChunk * 4;                  // exponentials staged for the sums
    static constexpr size_t kBytes = kV + kP + kE;
};
// Contexts up to this many positions keep the whole score row of each query
// head in shared memory (KVM * 4 B per position).
constexpr int kSmemCtx = 4096;

// grid (NKV, nq); block KVM * 128: the KVM query heads that share a KV head,
// thread (hh, d) = output dimension d of query head kvh * KVM + hh.  Each
// head's 128 threads form its softmax in the reference's order (maximum,
// exponentials, 8 float lane sums t-ascending, the lanes and the tail in
// double, p = e * (float)(1 / sum)); then every V row is staged once for all
// KVM heads through a 4-stage cp.async ring and each thread runs its fma
// chain over t ascending.  SE: the row (n <= kSmemCtx) lives in shared
// memory from the first read on; otherwise the exponentials are formed in
// place in `scores` and staged in chunks.
template <int KVM, bool SE, int kPvStages>
__global__ void __launch_bounds__(KVM * kThreads)
attn_ordered_softmax_pv_kernel(const uint16_t *__restrict v_pages, const int32_t *__restrict page_table,
                               const int32_t *__restrict seq_ids, const int32_t *__restrict positions,
                               float *__restrict scores, float *__restrict out, int max_ctx, int NH, int NKV,
                               int P, int maxp, int early) {
    extern __shared__ __align__(16) unsigned char pv_smem[];
    using L = PvSmem<KVM, kPvStages>;
    uint4 *vbuf = reinterpret_cast<uint4 *>(pv_smem);                              // [stage][64 * 16]
    float *pbuf = reinterpret_cast<float *>(pv_smem + L::kV);                     // [stage][KVM][64]
    float *ebuf_all = reinterpret_cast<float *>(pv_smem + L::kV + L::kP);         // SE: [KVM][max_ctx]
    __shared__ float red[KVM][kThreads / 32];
    __shared__ float lane_sum[KVM][8];
    __shared__ float inv_sh[KVM];
    __shared__ int zero_sh[KVM];
    pdl_launch_dependents();
    if (!early) pdl_wait();
    const int kvh = blockIdx.x, i = blockIdx.y;
    const int hh = threadIdx.x / kThreads, d = threadIdx.x % kThreads;
    const int h = kvh * KVM + hh;
    const int pos = positions[i];
    float *o = out + ((size_t)i * NH + h) * kD;
    if (pos < 0 || pos >= max_ctx) return;
    const int n = pos + 1, n8 = (n / 8) * 8;
    float *s = scores + ((size_t)i * NH + h) * max_ctx;
    float *ebuf = ebuf_all + (size_t)hh * (SE ? ((max_ctx + 3) & ~3) : kSumChunk);   // rows 16-byte aligned
    float *e = SE ? ebuf : s;              // where the score row / exponentials live
    // V rows do not depend on the softmax: the first stages of the P.V ring
    // are in flight from here on
    const int32_t *pt_row = page_table + (size_t)seq_ids[i] * maxp;
    const int nch = (n + kPvChunk - 1) / kPvChunk;
    // thread x of the block copies 16-byte column x & 15 of rows
    // (x >> 4) + j * kRowStep of every chunk; their pages and slots advance
    // by 64 positions per chunk (no division after the first)
    constexpr int kRowStep = KVM * kThreads / 16, kRowsPer = kPvChunk / kRowStep;
    const int qcol = threadIdx.x & 15;
    int pg[kRowsPer], slot[kRowsPer];
#pragma unroll
    for (int j = 0; j < kRowsPer; ++j) {
        const int t = (threadIdx.x >> 4) + j * kRowStep;
        pg[j] = t / P;
        slot[j] = t - pg[j] * P;
    }
    const uint4 *vp = reinterpret_cast<const uint4 *>(v_pages);
    auto issue = [&](int c) {
        if (c < nch) {
            const int cn = min(kPvChunk, n - c * kPvChunk);
            uint4 *vb = vbuf + (c % kPvStages) * (kPvChunk * kD / 8);
#pragma unroll
            for (int j = 0; j < kRowsPer; ++j) {
                const int r = (threadIdx.x >> 4) + j * kRowStep;
                if (r < cn)
                    cp_async16(vb + r * 16 + qcol,
                               vp + (((size_t)pt_row[pg[j]] * NKV + kvh) * P + slot[j]) * (kD / 8) + qcol);
            }
        }
#pragma unroll
        for (int j = 0; j < kRowsPer; ++j) {
            slot[j] += kPvChunk;
            while (slot[j] >= P) {
                slot[j] -= P;
                ++pg[j];
            }
        }
        cp_async_commit();    // an empty group past the end keeps the wait counts uniform
    };
    // early: the V chunks wholly before the position are issued before the
    // programmatic-dependent-launch wait (only the previous kernel -- the score
    // pass, which appends the row at the position -- may still be running)
    const int pre = early ? min(kPvStages - 1, pos / kPvChunk) : 0;
    for (int c = 0; c < pre; ++c) issue(c);
    if (early) pdl_wait();
    for (int c = pre; c < kPvStages - 1; ++c) issue(c);
    if constexpr (SE) {
        for (int t = d; t < n; t += kThreads) ebuf[t] = s[t];
        __syncthreads();
    }
    // 1. maximum (order-free)
    float m = -__int_as_float(0x7f800000);
    for (int t = d; t < n; t += kThreads) m = fmaxf(m, e[t]);
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((d & 31) == 0) red[hh][d >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[hh][0], red[hh][1]), fmaxf(red[hh][2], red[hh][3]));
    const bool finite_max = isfinite(m);   // every score -inf or NaN: the row is zeros
    // 2. exponentials in place (-inf scores give 0)
    const float ninf = -__int_as_float(0x7f800000);
    if (finite_max)
        for (int t = d; t < n; t += kThreads) {
            const float x = e[t];
            e[t] = x > ninf ? exp_ref(add_rn(x, -m)) : 0.0f;
        }
    __syncthreads();
    // 3. the sum: 8 float lanes t-ascending, the lanes in double, the tail in double
    float acc8 = 0.0f;
    if constexpr (SE) {
        if (d < 8)
            for (int k = d; k < n8; k += 8) acc8 = add_rn(acc8, ebuf[k]);
    } else {
        for (int c0 = 0; c0 < n8; c0 += kSumChunk) {
            const int cn = min(kSumChunk, n8 - c0);
            for (int t = d; t < cn; t += kThreads) ebuf[t] = s[c0 + t];
            __syncthreads();
            if (d < 8)
                for (int k = d; k < cn; k += 8) acc8 = add_rn(acc8, ebuf[k]);
            __syncthreads();
        }
    }
    if (d < 8) lane_sum[hh][d] = acc8;
    __syncthreads();
    if (d == 0) {
        double sum = 0.0;
        for (int l = 0; l < 8; ++l) sum = __dadd_rn(sum, (double)lane_sum[hh][l]);
        for (int t = n8; t < n; ++t) sum = __dadd_rn(sum, (double)e[t]);
        zero_sh[hh] = !finite_max || !(sum > 0.0) || !isfinite(sum);
        inv_sh[hh] = __double2float_rn(__ddiv_rn(1.0, sum));
    }
    __syncthreads();
    const bool zero = zero_sh[hh] != 0;
    const float inv = inv_sh[hh];
    if constexpr (SE) {
        // probabilities in place
        for (int t = d; t < n; t += kThreads) ebuf[t] = zero ? 0.0f : mul_rn(ebuf[t], inv);
        __syncthreads();
    }
    // 4. P.V: one fma chain per (head, d) over t ascending; V staged once for
    //    the KVM heads
    float acc = 0.0f;
    for (int c = 0; c < nch; ++c) {
        issue(c + kPvStages - 1);
        const int st = c % kPvStages;
        const int cn = min(kPvChunk, n - c * kPvChunk);
        if (!SE && d < cn) pbuf[(st * KVM + hh) * kPvChunk + d] = zero ? 0.0f : mul_rn(s[c * kPvChunk + d], inv);
        cp_async_wait<kPvStages - 1>();
        __syncthreads();
        const __half *vb = reinterpret_cast<const __half *>(vbuf + st * (kPvChunk * kD / 8)) + d;
        const float *pb = SE ? ebuf + c * kPvChunk : pbuf + (st * KVM + hh) * kPvChunk;
        int k = 0;
        for (; k + 8 <= cn; k += 8) {
            const float4 pa = reinterpret_cast<const float4 *>(pb + k)[0];
            const float4 pc = reinterpret_cast<const float4 *>(pb + k)[1];
            float vv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vv[j] = __half2float(vb[(k + j) * kD]);
            acc = fma_rn(pa.x, vv[0], acc);
            acc = fma_rn(pa.y, vv[1], acc);
            acc = fma_rn(pa.z, vv[2], acc);
            acc = fma_rn(pa.w, vv[3], acc);
            acc = fma_rn(pc.x, vv[4], acc);
            acc = fma_rn(pc.y, vv[5], acc);
            acc = fma_rn(pc.z, vv[6], acc);
            acc = fma_rn(pc.w, vv[7], acc);
        }
        for (; k < cn; ++k) acc = fma_rn(pb[k], __half2float(vb[k * kD]), acc);
        __syncthreads();   // stage st is refilled by the next iteration's issue
    }
    cp_async_wait<0>();
    o[d] = zero ? 0.0f : acc;
}

size_t attn_ordered_workspace_bytes(size_t nq, int max_ctx, int NH) {
    return ((nq * (size_t)NH * (size_t)max_ctx * sizeof(float)) + 255) & ~(size_t)255;
}

cudaError_t launch_attention_ordered(const AttnArgs &a, void *workspace, cudaStream_t stream, const OrdRope *rope) {
    float *scores = static_cast<float *>(workspace);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = stream;
    cfg.gridDim = dim3((a.max_ctx + kThreads - 1) / kThreads, a.NKV, (unsigned)a.nq);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)(a.NH / a.NKV + (rope ? 1 : 0)) * kD * sizeof(float) + (size_t)kThreads * kKRow;
    const int kvm = a.NH / a.NKV;
    const OrdRope rp = rope ? *rope : OrdRope{};
    // one query per sequence with the rope inside the score pass (a decode
    // step): the cache rows before each position are not written by the
    // score pass, so the P.V pass may fetch them before its dependent-launch wait
    const int early = rope ? 1 : 0;
    auto sc = [&](auto kern) {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)cfg.dynamicSmemBytes);
        if (e2 != cudaSuccess) return e2;
        return cudaLaunchKernelEx(&cfg, kern, a.q, a.k_pages, a.page_table, a.seq_ids, a.positions, scores,
                                  a.max_ctx, a.NH, a.NKV, a.P, a.maxp, rp);
    };
    cudaError_t e = cudaErrorInvalidValue;
    if (rope) {
        e = kvm == 1 ? sc(attn_ordered_scores_kernel<1, true>)
          : kvm == 2 ? sc(attn_ordered_scores_kernel<2, true>)
          : kvm == 4 ? sc(attn_ordered_scores_kernel<4, true>) : cudaErrorInvalidValue;
    } else {
        e = kvm == 1 ? sc(attn_ordered_scores_kernel<1, false>)
          : kvm == 2 ? sc(attn_ordered_scores_kernel<2, false>)
          : kvm == 4 ? sc(attn_ordered_scores_kernel<4, false>) : cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(a.NKV, (unsigned)a.nq);
    auto pv = [&](auto kern, size_t smem) {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e2 != cudaSuccess) return e2;
        cfg.blockDim = dim3(kvm * kThreads);
        cfg.dynamicSmemBytes = smem;
        return cudaLaunchKernelEx(&cfg, kern, a.v_pages, a.page_table, a.seq_ids, a.positions, scores, a.out,
                                  a.max_ctx, a.NH, a.NKV, a.P, a.maxp, early);
    };
    // the score rows in shared memory when they fit
    const bool se = a.max_ctx <= kSmemCtx;
    const bool many = a.nq >= (size_t)kPvManyQueries;
    auto se_bytes = [&](int m, int st) {
        return (size_t)st * kPvChunk * kD * 2 + (size_t)st * m * kPvChunk * 4 + (size_t)m * ((a.max_ctx + 3) & ~3) * 4;
    };
    if (se) {
        if (many) {
            if (kvm == 1) return pv(attn_ordered_softmax_pv_kernel<1, true, 2>, se_bytes(1, 2));
            if (kvm == 2) return pv(attn_ordered_softmax_pv_kernel<2, true, 2>, se_bytes(2, 2));
            if (kvm == 4) return pv(attn_ordered_softmax_pv_kernel<4, true, 2>, se_bytes(4, 2));
        }
        if (a.max_ctx <= kPvDeepCtx) {
            if (kvm == 1) return pv(attn_ordered_softmax_pv_kernel<1, true, kPvStagesDeep>, se_bytes(1, kPvStagesDeep));
            if (kvm == 2) return pv(attn_ordered_softmax_pv_kernel<2, true, kPvStagesDeep>, se_bytes(2, kPvStagesDeep));
            if (kvm == 4) return pv(attn_ordered_softmax_pv_kernel<4, true, kPvStagesDeep>, se_bytes(4, kPvStagesDeep));
        }
        if (kvm == 1) return pv(attn_ordered_softmax_pv_kernel<1, true, kPvStagesMax>, se_bytes(1, kPvStagesMax));
        if (kvm == 2) return pv(attn_ordered_softmax_pv_kernel<2, true, kPvStagesMax>, se_bytes(2, kPvStagesMax));
        if (kvm == 4) return pv(attn_ordered_softmax_pv_kernel<4, true, kPvStagesMax>, se_bytes(4, kPvStagesMax));
    }
    if (kvm == 1) return pv(attn_ordered_softmax_pv_kernel<1, false, kPvStagesMax>, PvSmem<1, kPvStagesMax>::kBytes);
    if (kvm == 2) return pv(attn_ordered_softmax_pv_kernel<2, false, kPvStagesMax>, PvSmem<2, kPvStagesMax>::kBytes);
    if (kvm == 4) return pv(attn_ordered_softmax_pv_kernel<4, false, kPvStagesMax>, PvSmem<4, kPvStagesMax>::kBytes);
    return cudaErrorInvalidValue;
}

}  // namespace qvl
