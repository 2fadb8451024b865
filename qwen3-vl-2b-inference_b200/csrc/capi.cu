// extern "C" entry points declared in include/qvl_b200.h: argument checks,
// workspace carving and kernel sequencing.  No entry point allocates memory,
// synchronises the stream, exits or traps.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include "common.cuh"
#include "qact.cuh"
#include "gemv_i8.cuh"
#include "gemm_i8_tc.cuh"
#include "gemv_ring.cuh"
#include "swiglu.cuh"
#include "attention_ordered.cuh"
#include "gemm_f16_tc.cuh"
#include "attention.cuh"
#include "argmax.cuh"
#include "norm.cuh"

namespace {
int g_last_cuda_error = 0;

inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

inline bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

size_t qbuf_bytes(size_t M, size_t K, size_t g) {
    return align256(M * K * sizeof(int16_t)) + align256(M * (K / g) * sizeof(float));
}

// Largest row tile (<= 8) whose int16 activations fit in shared memory.
int gemv_rows_per_launch(size_t K, size_t g) {
    for (int mr = 8; mr >= 1; mr >>= 1)
        if (qvl::gemv_smem_bytes(mr, (int)K, (int)g) <= 200 * 1024) return mr;
    return 0;
}

// Single-row per-row-scale GEMVs of at least this many weight bytes stream
// through the ring kernel (gemv_ring.cu); smaller ones keep the direct-load
// kernel.  QVL_GEMV_RING=0 in the environment disables the ring kernel.
constexpr size_t kRingMinBytes = 4u << 20;
bool ring_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("QVL_GEMV_RING");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

bool lane8_for(int semantics, size_t M, size_t N, size_t K) {
    if (semantics == QVL_SEM_LANE8) return true;
    if (semantics == QVL_SEM_TILED) return false;
    return M == 1 && N >= 1024 && K >= 1024;   // cpu_f32a_i8f32sb_f32c_avx2.cpp:464
}

// y[M,N] from pre-quantised activations on the CUDA cores: the ring GEMV
// for large single-row products, else the tiled GEMV in row tiles.  (The
// tensor-core products are launched by the callers on hi/lo planes that their
// quantisation kernels write.)
int run_q16_linear(const int16_t *q, const float *qs, const int8_t *B, const float *Bs, float *C,
                   size_t M, size_t N, size_t K, size_t g, bool lane8, cudaStream_t st, int acc = 0) {
    if (M == 1 && lane8 && g == K && N * K >= kRingMinBytes && ring_enabled()) {
        qvl::RingGemvArgs r{q, qs, B, Bs, C, (int)N, (int)K, acc};
        if (qvl::gemv_ring_supported(r)) {
            QVL_CUDA_TRY(qvl::launch_gemv_ring(r, st));
            return QVL_OK;
        }
    }
    const int mr = gemv_rows_per_launch(K, g);
    if (mr == 0) return QVL_ERR_UNSUPPORTED;
    const size_t G = K / g;
    for (size_t m0 = 0; m0 < M; m0 += mr) {
        qvl::GemvArgs a = {};
        a.q = q + m0 * K;
        a.qs = qs + m0 * G;
        a.W = B;
        a.ws = Bs;
        a.y = C + m0 * N;
        a.M = (int)((M - m0) < (size_t)mr ? (M - m0) : (size_t)mr);
        a.N = (int)N;
        a.K = (int)K;
        a.g = (int)g;
        a.ldy = (long)N;
        a.acc = acc;
        QVL_CUDA_TRY(qvl::launch_gemv_i8(a, lane8, st));
    }
    return QVL_OK;
}

// The products of one set of hi/lo planes: a single tensor-core launch over
// all matrices; with up_scratch, matrix 1's product goes there and is folded
// into matrix 0's as swiglu(C0, up) (gate/up pair).
int run_planes_batched(const int8_t *hi, const uint8_t *lo, const float *q_scales, size_t n_mats,
                       const int8_t *const *B, const float *const *B_scales, float *const *C, const size_t *N,
                       size_t M, size_t K, int acc, float *up_scratch, cudaStream_t st) {
    float *outs[3];
    int Ns[3];
    for (size_t i = 0; i < n_mats; ++i) {
        outs[i] = (up_scratch && i == 1) ? up_scratch : C[i];
        Ns[i] = (int)N[i];
    }
    QVL_CUDA_TRY(qvl::launch_gemm_i8_tc_planes_multi(hi, lo, q_scales, (int)n_mats, B, B_scales, outs, Ns, (int)M,
                                                     (int)K, acc, st));
    if (up_scratch) QVL_CUDA_TRY(qvl::launch_swiglu(C[0], up_scratch, (long)(M * N[0]), st));
    return QVL_OK;
}

int check_linear_shape(size_t M, size_t N, size_t K, size_t g) {
    if (M == 0 || N == 0 || K == 0) return QVL_ERR_INVALID;
    if (K > (1u << 30) || N > (1u << 30) || M > (1u << 20)) return QVL_ERR_INVALID;
    if (!qvl::gemv_shape_supported((int)K, (int)g)) return QVL_ERR_UNSUPPORTED;
    return QVL_OK;
}
}  // namespace

extern "C" void qvl_internal_set_cuda_error(int err) { g_last_cuda_error = err; }

extern "C" {

const char *qvl_status_string(int s) {
    switch (s) {
        case QVL_OK: return "ok";
        case QVL_ERR_INVALID: return "invalid argument";
        case QVL_ERR_UNSUPPORTED: return "unsupported shape or dtype combination";
        case QVL_ERR_CUDA: return "CUDA runtime error";
        case QVL_ERR_WORKSPACE: return "workspace missing or too small";
    }
    return "unknown status";
}

int qvl_last_cuda_error(void) { return g_last_cuda_error; }

const char *qvl_version(void) { return "qvl_b200 0.1"; }

// Host code: the text section of qwen_rope_precompute
// (model/src/load_model.cpp:413-490) with the host's single-precision libm, as
// the reference computes it: inv_freq[i] = 1 / powf(theta, 2i / D), then
// cosf / sinf of pos * inv_freq[i].  For text positions the three M-RoPE
// sections carry the same position, so the interleave leaves section 0 equal
// to this table.
int qvl_rope_table(int theta, int head_dim, int rows, float *cos_out, float *sin_out) {
    if (!cos_out || !sin_out || head_dim <= 0 || head_dim % 2 || rows < 0) return QVL_ERR_INVALID;
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) {
        const volatile float e = (2.0f * (float)i) / (float)head_dim;
        const float inv_freq = 1.0f / powf((float)theta, e);
        for (int p = 0; p < rows; ++p) {
            const volatile float f = (float)p * inv_freq;
            cos_out[(size_t)p * half + i] = cosf(f);
            sin_out[(size_t)p * half + i] = sinf(f);
        }
    }
    return QVL_OK;
}

int qvl_tc_timeout_status(int *timed_out, int clear, void *stream) {
    if (!timed_out) return QVL_ERR_INVALID;
    int *words[2] = {qvl::gemm_tc_timeout_word(), qvl::gemm_f16_timeout_word()};
    if (!words[0] || !words[1]) return QVL_ERR_CUDA;
    cudaStream_t st = (cudaStream_t)stream;
    int v[2] = {0, 0};
    for (int i = 0; i < 2; ++i) QVL_CUDA_TRY(cudaMemcpyAsync(&v[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, st));
    QVL_CUDA_TRY(cudaStreamSynchronize(st));
    *timed_out = (v[0] | v[1]) != 0;
    if (clear && *timed_out) {
        for (int i = 0; i < 2; ++i) QVL_CUDA_TRY(cudaMemsetAsync(words[i], 0, sizeof(int), st));
        QVL_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return QVL_OK;
}

int qvl_internal_set_tc_timeout(void *stream) {
    int *word = qvl::gemm_tc_timeout_word();
    if (!word) return QVL_ERR_CUDA;
    const int one = 1;
    QVL_CUDA_TRY(cudaMemcpyAsync(word, &one, sizeof(int), cudaMemcpyHostToDevice, (cudaStream_t)stream));
    QVL_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    return QVL_OK;
}

int qvl_quantize_rows(const float *x, int16_t *q, float *q_scales, size_t M, size_t K,
                      size_t group_size, void *stream) {
    if (!x || !q || !q_scales) return QVL_ERR_INVALID;
    if (!aligned(x, 16) || !aligned(q, 8)) return QVL_ERR_INVALID;
    if (M == 0 || K == 0 || group_size == 0 || K % group_size || group_size % 16) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_quantize_rows(x, q, q_scales, (int)M, (int)K, (int)group_size,
                                           (cudaStream_t)stream));
    return QVL_OK;
}

size_t qvl_linear_i8_workspace_bytes(size_t M, size_t K, size_t group_size) {
    if (group_size == 0 || K % group_size) return 0;
    size_t b = qbuf_bytes(M, K, group_size);
    if (M >= 16 && K % 128 == 0 && (group_size == K || qvl::gemm_tc_grouped_size(group_size, K)))
        b += qvl::gemm_tc_planes_bytes(M, K);
    return b;
}

int qvl_linear_q16_i8(const int16_t *q, const float *q_scales, const int8_t *B,
                      const float *B_scales, float *C, size_t M, size_t N, size_t K,
                      size_t group_size, int semantics, void *stream) {
    if (!q || !q_scales || !B || !B_scales || !C) return QVL_ERR_INVALID;
    int rc = check_linear_shape(M, N, K, group_size);
    if (rc) return rc;
    if (!aligned(q, 16) || !aligned(B, 16) || (K * sizeof(int8_t)) % 16) return QVL_ERR_INVALID;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    semantics &= ~QVL_SEM_ACCUMULATE;
    if (semantics < QVL_SEM_REFERENCE || semantics > QVL_SEM_TILED) return QVL_ERR_INVALID;
    return run_q16_linear(q, q_scales, B, B_scales, C, M, N, K, group_size,
                          lane8_for(semantics, M, N, K), (cudaStream_t)stream, acc);
}

int qvl_linear_i8(const float *A, const int8_t *B, const float *B_scales, float *C, size_t M,
                  size_t N, size_t K, int group_quantized, size_t group_size, int semantics,
                  void *workspace, size_t workspace_bytes, void *stream) {
    if (!A || !B || !B_scales || !C) return QVL_ERR_INVALID;
    const size_t g = group_quantized ? group_size : K;
    int rc = check_linear_shape(M, N, K, g);
    if (rc) return rc;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    semantics &= ~QVL_SEM_ACCUMULATE;
    if (semantics < QVL_SEM_REFERENCE || semantics > QVL_SEM_TILED) return QVL_ERR_INVALID;
    const size_t need = qbuf_bytes(M, K, g);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    if (!aligned(B, 16) || !aligned(A, 16)) return QVL_ERR_INVALID;
    int16_t *q = static_cast<int16_t *>(workspace);
    float *qs = reinterpret_cast<float *>(static_cast<char *>(workspace) + align256(M * K * 2));
    cudaStream_t st = (cudaStream_t)stream;
    // M = 1 per-row products large enough for the ring GEMV: the activation
    // quantisation happens inside it (one launch instead of two)
    if (M == 1 && g == K && lane8_for(semantics, M, N, K) && N * K >= kRingMinBytes && ring_enabled()) {
        qvl::RingGemvArgs r{nullptr, nullptr, B, B_scales, C, (int)N, (int)K, acc, A};
        if (qvl::gemv_ring_supported(r)) {
            QVL_CUDA_TRY(qvl::launch_gemv_ring(r, st));
            return QVL_OK;
        }
    }
    const bool lane8 = lane8_for(semantics, M, N, K);
    // tensor-core product: the quantisation writes its hi/lo planes directly
    if (!lane8 && !acc && workspace_bytes >= need + qvl::gemm_tc_planes_bytes(M, K) &&
        qvl::gemm_tc_supported(M, N, K, g)) {
        int8_t *hi = reinterpret_cast<int8_t *>(static_cast<char *>(workspace) + need);
        uint8_t *lo = reinterpret_cast<uint8_t *>(hi) + qvl::gemm_tc_planes_bytes(M, K) / 2;
        QVL_CUDA_TRY(qvl::launch_quantize_rows(A, q, qs, (int)M, (int)K, (int)g, st, hi, lo));
        QVL_CUDA_TRY(qvl::launch_gemm_i8_tc_planes(hi, lo, qs, B, B_scales, C, (int)M, (int)N, (int)K, 0, st,
                                                   (int)g));
        return QVL_OK;
    }
    QVL_CUDA_TRY(qvl::launch_quantize_rows(A, q, qs, (int)M, (int)K, (int)g, st));
    return run_q16_linear(q, qs, B, B_scales, C, M, N, K, g, lane8, st, acc);
}

int qvl_linear_q16_i8_multi(const int16_t *q, const float *q_scales, size_t n_mats,
                            const int8_t *const *B, const float *const *B_scales, float *const *C,
                            const size_t *N, size_t M, size_t K, size_t group_size, int semantics,
                            void *stream) {
    if (!q || !q_scales || !B || !B_scales || !C || !N || n_mats == 0 || n_mats > 3) return QVL_ERR_INVALID;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    const int sem = semantics & ~QVL_SEM_ACCUMULATE;
    if (sem < QVL_SEM_REFERENCE || sem > QVL_SEM_TILED) return QVL_ERR_INVALID;
    size_t total = 0;
    for (size_t i = 0; i < n_mats; ++i) {
        if (!B[i] || !B_scales[i] || !C[i] || !aligned(B[i], 16)) return QVL_ERR_INVALID;
        int rc = check_linear_shape(M, N[i], K, group_size);
        if (rc) return rc;
        total += N[i];
    }
    if (!aligned(q, 16) || total > (size_t)INT32_MAX) return QVL_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    bool same_sem = true;
    for (size_t i = 1; i < n_mats; ++i) same_sem &= lane8_for(sem, M, N[i], K) == lane8_for(sem, M, N[0], K);
    if (qvl::gemv_fast_eligible((int)M, (int)K, (int)group_size) && same_sem) {
        qvl::GemvArgs a = {};
        a.q = q; a.qs = q_scales; a.M = (int)M; a.K = (int)K; a.g = (int)group_size; a.acc = acc;
        size_t end = 0;
        for (size_t i = 0; i < 3; ++i) {
            if (i < n_mats) {
                a.segs.W[i] = B[i]; a.segs.ws[i] = B_scales[i]; a.segs.y[i] = C[i]; a.segs.ldy[i] = (long)N[i];
                end += N[i];
            }
            a.segs.end[i] = (int)end;
        }
        a.segs.nseg = (int)n_mats;
        a.N = (int)total;
        QVL_CUDA_TRY(qvl::launch_gemv_i8(a, lane8_for(sem, M, N[0], K), st));
        return QVL_OK;
    }
    for (size_t i = 0; i < n_mats; ++i) {
        int rc = run_q16_linear(q, q_scales, B[i], B_scales[i], C[i], M, N[i], K, group_size,
                                lane8_for(sem, M, N[i], K), st, acc);
        if (rc) return rc;
    }
    return QVL_OK;
}

int qvl_gate_up_swiglu_q16_i8(const int16_t *q, const float *q_scales, const int8_t *Wg,
                              const float *sg, const int8_t *Wu, const float *su, float *h,
                              float *up_scratch, size_t M, size_t I, size_t K, size_t group_size,
                              int semantics, void *stream) {
    if (!q || !q_scales || !Wg || !sg || !Wu || !su || !h) return QVL_ERR_INVALID;
    if (semantics < QVL_SEM_REFERENCE || semantics > QVL_SEM_TILED) return QVL_ERR_INVALID;
    int rc = check_linear_shape(M, I, K, group_size);
    if (rc) return rc;
    if (!aligned(q, 16) || !aligned(Wg, 16) || !aligned(Wu, 16) || 2 * I > (size_t)INT32_MAX)
        return QVL_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    const bool lane8 = lane8_for(semantics, M, I, K);
    if (qvl::gemv_fast_eligible((int)M, (int)K, (int)group_size)) {
        qvl::GemvArgs a = {};
        a.q = q; a.qs = q_scales; a.M = (int)M; a.K = (int)K; a.g = (int)group_size;
        a.segs.W[0] = Wg; a.segs.ws[0] = sg; a.segs.y[0] = h; a.segs.ldy[0] = (long)I;
        a.segs.W[1] = Wu; a.segs.ws[1] = su; a.segs.y[1] = h; a.segs.ldy[1] = (long)I;
        a.segs.end[0] = (int)I; a.segs.end[1] = a.segs.end[2] = (int)(2 * I);
        a.segs.nseg = 2;
        a.N = (int)(2 * I);
        a.pair = 1;
        QVL_CUDA_TRY(qvl::launch_gemv_i8(a, lane8, st));
        return QVL_OK;
    }
    if (!up_scratch) return QVL_ERR_WORKSPACE;
    rc = run_q16_linear(q, q_scales, Wg, sg, h, M, I, K, group_size, lane8, st);
    if (!rc) rc = run_q16_linear(q, q_scales, Wu, su, up_scratch, M, I, K, group_size, lane8, st);
    if (rc) return rc;
    QVL_CUDA_TRY(qvl::launch_swiglu(h, up_scratch, (long)(M * I), st));
    return QVL_OK;
}

int qvl_linear_q16_i8_tail(const int16_t *q, const float *q_scales, size_t n_mats,
                           const int8_t *const *B, const float *const *B_scales, float *const *C,
                           const size_t *N, size_t M, size_t K, size_t group_size, int semantics,
                           int swiglu_pair, const qvl_row_tail *tail, void *stream) {
    if (!q || !q_scales || !B || !B_scales || !C || !N || !tail || !tail->counter || !tail->q ||
        !tail->q_scales || n_mats == 0 || n_mats > 3)
        return QVL_ERR_INVALID;
    if (swiglu_pair && (n_mats != 2 || N[0] != N[1])) return QVL_ERR_INVALID;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    const int sem = semantics & ~QVL_SEM_ACCUMULATE;
    if (sem < QVL_SEM_REFERENCE || sem > QVL_SEM_TILED) return QVL_ERR_INVALID;
    const size_t H = N[0];
    if (H % 16 || H > 16384 || tail->quant_group == 0 || tail->quant_group % 16 || H % tail->quant_group ||
        H / tail->quant_group > 64 || (tail->norm_w && (!tail->norm_s || tail->norm_group == 0 ||
                                                         H % tail->norm_group)))
        return QVL_ERR_UNSUPPORTED;
    size_t total = 0;
    for (size_t i = 0; i < n_mats; ++i) {
        if (!B[i] || !B_scales[i] || !C[i] || !aligned(B[i], 16)) return QVL_ERR_INVALID;
        int rc = check_linear_shape(M, N[i], K, group_size);
        if (rc) return rc;
        total += N[i];
    }
    if (!aligned(q, 16) || !aligned(C[0], 16) || total > (size_t)INT32_MAX) return QVL_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    const bool lane8 = lane8_for(sem, M, N[0], K);
    if (qvl::gemv_fast_eligible((int)M, (int)K, (int)group_size)) {
        qvl::GemvArgs a = {};
        a.q = q; a.qs = q_scales; a.M = (int)M; a.K = (int)K; a.g = (int)group_size; a.acc = acc;
        size_t end = 0;
        for (size_t i = 0; i < 3; ++i) {
            if (i < n_mats) {
                a.segs.W[i] = B[i]; a.segs.ws[i] = B_scales[i]; a.segs.y[i] = C[i];
                a.segs.ldy[i] = (long)N[i];
                end += N[i];
            }
            a.segs.end[i] = (int)end;
        }
        a.segs.nseg = (int)n_mats;
        a.N = (int)total;
        a.pair = swiglu_pair ? 1 : 0;
        a.tail.counter = tail->counter;
        a.tail.x = C[0];
        a.tail.wq = tail->norm_w; a.tail.ws = tail->norm_s; a.tail.ngs = (int)tail->norm_group;
        a.tail.eps = tail->eps; a.tail.inplace_form = tail->inplace_form;
        a.tail.out = tail->norm_out; a.tail.q = tail->q; a.tail.qs = tail->q_scales;
        a.tail.qg = (int)tail->quant_group; a.tail.H = (int)H; a.tail.rows = (int)M;
        QVL_CUDA_TRY(qvl::launch_gemv_i8(a, lane8, st));
        return QVL_OK;
    }
    // separate launches
    if (swiglu_pair) {
        return QVL_ERR_UNSUPPORTED;   // needs an up buffer: use qvl_gate_up_swiglu_q16_i8 + qvl_quantize_rows
    }
    for (size_t i = 0; i < n_mats; ++i) {
        int rc = run_q16_linear(q, q_scales, B[i], B_scales[i], C[i], M, N[i], K, group_size,
                                lane8_for(sem, M, N[i], K), st, acc);
        if (rc) return rc;
    }
    QVL_CUDA_TRY(qvl::launch_rmsnorm_quant(C[0], tail->norm_w, tail->norm_s, tail->norm_out, tail->q,
                                           tail->q_scales, (int)M, (int)H, (int)(tail->norm_w ? tail->norm_group : H),
                                           tail->eps, tail->inplace_form != 0, (int)tail->quant_group, st));
    return QVL_OK;
}

size_t qvl_linear_q16_i8_batched_workspace_bytes(size_t M, size_t K) {
    return qvl::gemm_tc_planes_bytes(M, K);
}

int qvl_linear_q16_i8_batched(const int16_t *q, const float *q_scales, size_t n_mats,
                              const int8_t *const *B, const float *const *B_scales, float *const *C,
                              const size_t *N, size_t M, size_t K, int semantics, int swiglu_pair,
                              float *up_scratch, void *workspace, size_t workspace_bytes, void *stream) {
    if (!q || !q_scales || !B || !B_scales || !C || !N || n_mats == 0 || n_mats > 3) return QVL_ERR_INVALID;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    const int sem = semantics & ~QVL_SEM_ACCUMULATE;
    if (sem != QVL_SEM_TILED && !(sem == QVL_SEM_REFERENCE && M > 1)) return QVL_ERR_UNSUPPORTED;
    if (swiglu_pair && (n_mats != 2 || N[0] != N[1] || !up_scratch || acc)) return QVL_ERR_INVALID;
    for (size_t i = 0; i < n_mats; ++i) {
        if (!B[i] || !B_scales[i] || !C[i] || !aligned(B[i], 16)) return QVL_ERR_INVALID;
        if (!qvl::gemm_tc_supported(M, N[i], K, K)) return QVL_ERR_UNSUPPORTED;
    }
    const size_t need = qvl::gemm_tc_planes_bytes(M, K);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    int8_t *hi = static_cast<int8_t *>(workspace);
    uint8_t *lo = reinterpret_cast<uint8_t *>(hi) + need / 2;
    QVL_CUDA_TRY(qvl::launch_split_hi_lo(q, hi, lo, (int)M, (int)K, st));
    return run_planes_batched(hi, lo, q_scales, n_mats, B, B_scales, C, N, M, K, acc, swiglu_pair ? up_scratch : nullptr,
                              st);
}

int qvl_linear_planes_i8_batched(const int8_t *hi, const uint8_t *lo, const float *q_scales, size_t n_mats,
                                 const int8_t *const *B, const float *const *B_scales, float *const *C,
                                 const size_t *N, size_t M, size_t K, int semantics, void *stream) {
    if (!hi || !lo || !q_scales || !B || !B_scales || !C || !N || n_mats == 0 || n_mats > 3) return QVL_ERR_INVALID;
    const int acc = (semantics & QVL_SEM_ACCUMULATE) ? 1 : 0;
    const int sem = semantics & ~QVL_SEM_ACCUMULATE;
    if (sem != QVL_SEM_TILED && !(sem == QVL_SEM_REFERENCE && M > 1)) return QVL_ERR_UNSUPPORTED;
    if (!aligned(hi, 16) || !aligned(lo, 16) || (M * K) % 16) return QVL_ERR_INVALID;
    for (size_t i = 0; i < n_mats; ++i) {
        if (!B[i] || !B_scales[i] || !C[i] || !aligned(B[i], 16)) return QVL_ERR_INVALID;
        if (!qvl::gemm_tc_supported(M, N[i], K, K)) return QVL_ERR_UNSUPPORTED;
    }
    return run_planes_batched(hi, lo, q_scales, n_mats, B, B_scales, C, N, M, K, acc, nullptr,
                              (cudaStream_t)stream);
}

// Test hook: the expf the SwiGLU kernels use, elementwise (not in the header).
int qvl_internal_expf(const float *x, float *y, size_t n, void *stream) {
    if (!x || !y) return QVL_ERR_INVALID;
    if (n == 0) return QVL_OK;
    QVL_CUDA_TRY(qvl::launch_expf_host(x, y, (long)n, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_swiglu(float *gate, const float *up, size_t n, void *stream) {
    if (!gate || !up) return QVL_ERR_INVALID;
    if (n == 0) return QVL_OK;
    QVL_CUDA_TRY(qvl::launch_swiglu(gate, up, (long)n, (cudaStream_t)stream));
    return QVL_OK;
}

size_t qvl_swiglu_mlp_workspace_bytes(size_t M, size_t H, size_t I, size_t g) {
    const size_t g_in = g ? g : H, g_h = g ? g : I;     // 0: per-row, group = each product's K
    if (H == 0 || I == 0 || H % g_in || I % g_h) return 0;
    return qbuf_bytes(M, H, g_in) + 2 * align256(M * I * sizeof(float)) + qbuf_bytes(M, I, g_h) +
           align256(qvl::gemm_tc_planes_bytes(M, H > I ? H : I));
}

int qvl_swiglu_mlp_i8(const float *x, const int8_t *Wg, const float *sg, const int8_t *Wu,
                      const float *su, const int8_t *Wd, const float *sd, float *out, size_t M,
                      size_t H, size_t I, size_t group_size, int semantics, void *workspace,
                      size_t workspace_bytes, void *stream) {
    if (!x || !Wg || !sg || !Wu || !su || !Wd || !sd || !out) return QVL_ERR_INVALID;
    if (!aligned(x, 16)) return QVL_ERR_INVALID;
    const size_t g_in = group_size ? group_size : H, g_h = group_size ? group_size : I;
    int rc = check_linear_shape(M, I, H, g_in);
    if (!rc) rc = check_linear_shape(M, H, I, g_h);
    if (rc) return rc;
    if (semantics < QVL_SEM_REFERENCE || semantics > QVL_SEM_TILED) return QVL_ERR_INVALID;
    const size_t need = qvl_swiglu_mlp_workspace_bytes(M, H, I, group_size);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    char *w = static_cast<char *>(workspace);
    int16_t *qx = reinterpret_cast<int16_t *>(w);
    float *qxs = reinterpret_cast<float *>(w + align256(M * H * 2));
    w += qbuf_bytes(M, H, g_in);
    float *gate = reinterpret_cast<float *>(w);
    w += align256(M * I * 4);
    float *up = reinterpret_cast<float *>(w);
    w += align256(M * I * 4);
    int16_t *qh = reinterpret_cast<int16_t *>(w);
    float *qhs = reinterpret_cast<float *>(w + align256(M * I * 2));
    w += qbuf_bytes(M, I, g_h);
    // hi/lo activation planes of the tensor-core path (M >= 16, TILED), written
    // by the quantisation kernels themselves
    int8_t *hi = reinterpret_cast<int8_t *>(w);
    cudaStream_t st = (cudaStream_t)stream;
    const bool l_gu = lane8_for(semantics, M, I, H), l_d = lane8_for(semantics, M, H, I);
    const bool tc_gu = !l_gu && qvl::gemm_tc_supported(M, I, H, g_in);
    const bool tc_d = !l_d && qvl::gemm_tc_supported(M, H, I, g_h);
    uint8_t *lo_gu = reinterpret_cast<uint8_t *>(hi) + qvl::gemm_tc_planes_bytes(M, H) / 2;
    uint8_t *lo_d = reinterpret_cast<uint8_t *>(hi) + qvl::gemm_tc_planes_bytes(M, I) / 2;
    QVL_CUDA_TRY(qvl::launch_quantize_rows(x, qx, qxs, (int)M, (int)H, (int)g_in, st, tc_gu ? hi : nullptr,
                                           tc_gu ? lo_gu : nullptr));
    if (tc_gu) {
        QVL_CUDA_TRY(qvl::launch_gemm_i8_tc_planes(hi, lo_gu, qxs, Wg, sg, gate, (int)M, (int)I, (int)H, 0, st,
                                                   (int)g_in));
        QVL_CUDA_TRY(qvl::launch_gemm_i8_tc_planes(hi, lo_gu, qxs, Wu, su, up, (int)M, (int)I, (int)H, 0, st,
                                                   (int)g_in));
    } else {
        rc = run_q16_linear(qx, qxs, Wg, sg, gate, M, I, H, g_in, l_gu, st);
        if (!rc) rc = run_q16_linear(qx, qxs, Wu, su, up, M, I, H, g_in, l_gu, st);
        if (rc) return rc;
    }
    if (g_h >= 4096 || tc_d) {
        // whole-row groups: the SwiGLUs (double-precision exp) spread over the
        // GPU in place in the gate scratch, then the row quantisation
        QVL_CUDA_TRY(qvl::launch_swiglu(gate, up, (long)(M * I), st));
        QVL_CUDA_TRY(qvl::launch_quantize_rows(gate, qh, qhs, (int)M, (int)I, (int)g_h, st, tc_d ? hi : nullptr,
                                               tc_d ? lo_d : nullptr));
    } else {
        QVL_CUDA_TRY(qvl::launch_swiglu_quant(gate, up, qh, qhs, (int)M, (int)I, (int)g_h, st));
    }
    if (tc_d) {
        QVL_CUDA_TRY(qvl::launch_gemm_i8_tc_planes(hi, lo_d, qhs, Wd, sd, out, (int)M, (int)H, (int)I, 0, st,
                                                   (int)g_h));
        return QVL_OK;
    }
    return run_q16_linear(qh, qhs, Wd, sd, out, M, H, I, g_h, l_d, st);
}

static int check_attn_dims(const qvl_attn_dims *d) {
    if (!d) return QVL_ERR_INVALID;
    if (d->head_dim != 128) return QVL_ERR_UNSUPPORTED;
    if (d->num_heads <= 0 || d->num_kv_heads <= 0 || d->num_heads % d->num_kv_heads) return QVL_ERR_INVALID;
    const int kvm = d->num_heads / d->num_kv_heads;
    if (kvm != 1 && kvm != 2 && kvm != 4) return QVL_ERR_UNSUPPORTED;
    if (d->page_size <= 0 || d->max_pages_per_seq <= 0 || d->max_pos <= 0) return QVL_ERR_INVALID;
    return QVL_OK;
}

int qvl_rope_kv_append(float *q, const float *k_new, const float *v_new, uint16_t *k_pages,
                       uint16_t *v_pages, const int32_t *page_table, const int32_t *seq_ids,
                       const int32_t *positions, size_t nq, const float *rope_cos,
                       const float *rope_sin, const qvl_attn_dims *dims, void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !positions || !rope_cos || !rope_sin) return QVL_ERR_INVALID;
    if (k_new && (!v_new || !k_pages || !v_pages || !page_table || !seq_ids)) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    qvl::RopeArgs a;
    a.q = q; a.k_new = k_new; a.v_new = v_new; a.k_pages = k_pages; a.v_pages = v_pages;
    a.page_table = page_table; a.seq_ids = seq_ids; a.positions = positions; a.nq = nq;
    a.rope_cos = rope_cos; a.rope_sin = rope_sin;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    a.norm = qvl::QkNorm{nullptr, nullptr, nullptr, nullptr, 1, 0.0f};
    QVL_CUDA_TRY(qvl::launch_rope_append(a, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_qknorm_rope_kv_append(float *q, const float *k_new, const float *v_new, uint16_t *k_pages,
                              uint16_t *v_pages, const int32_t *page_table, const int32_t *seq_ids,
                              const int32_t *positions, size_t nq, const float *rope_cos,
                              const float *rope_sin, const int8_t *q_norm_w, const float *q_norm_s,
                              const int8_t *k_norm_w, const float *k_norm_s, size_t norm_group,
                              float eps, const qvl_attn_dims *dims, void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !k_new || !v_new || !k_pages || !v_pages || !page_table || !seq_ids || !positions ||
        !rope_cos || !rope_sin || !q_norm_w || !q_norm_s || !k_norm_w || !k_norm_s)
        return QVL_ERR_INVALID;
    if (norm_group == 0 || 128 % norm_group || dims->num_heads + dims->num_kv_heads > 64) return QVL_ERR_UNSUPPORTED;
    if (nq == 0) return QVL_OK;
    qvl::RopeArgs a;
    a.q = q; a.k_new = k_new; a.v_new = v_new; a.k_pages = k_pages; a.v_pages = v_pages;
    a.page_table = page_table; a.seq_ids = seq_ids; a.positions = positions; a.nq = nq;
    a.rope_cos = rope_cos; a.rope_sin = rope_sin;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    a.norm = qvl::QkNorm{q_norm_w, q_norm_s, k_norm_w, k_norm_s, (int)norm_group, eps};
    QVL_CUDA_TRY(qvl::launch_rope_append(a, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_rms_norm_i8(const float *x, const int8_t *w, const float *w_scales, float *out,
                    int16_t *q, float *q_scales, size_t rows, size_t hidden, size_t norm_group,
                    float eps, int inplace_form, size_t quant_group, void *stream) {
    if (!x || !w || !w_scales || (!out && !q) || (q && !q_scales)) return QVL_ERR_INVALID;
    if (rows == 0) return QVL_OK;
    if (hidden == 0 || hidden % 16 || hidden > 16384 || norm_group == 0 || hidden % norm_group)
        return QVL_ERR_INVALID;
    if (!aligned(x, 16)) return QVL_ERR_INVALID;
    if (q && (quant_group == 0 || quant_group % 16 || hidden % quant_group || hidden / quant_group > 64))
        return QVL_ERR_UNSUPPORTED;
    QVL_CUDA_TRY(qvl::launch_rmsnorm_quant(x, w, w_scales, out, q, q_scales, (int)rows, (int)hidden,
                                           (int)norm_group, eps, inplace_form != 0,
                                           q ? (int)quant_group : 16, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_rms_norm_i8_planes(const float *x, const int8_t *w, const float *w_scales, float *out, int16_t *q,
                           float *q_scales, int8_t *hi, uint8_t *lo, size_t rows, size_t hidden,
                           size_t norm_group, float eps, int inplace_form, void *stream) {
    if (!x || !w || !w_scales || !q || !q_scales || !hi || !lo) return QVL_ERR_INVALID;
    if (rows == 0) return QVL_OK;
    if (hidden == 0 || hidden % 16 || hidden > 16384 || norm_group == 0 || hidden % norm_group)
        return QVL_ERR_INVALID;
    if (!aligned(x, 16) || !aligned(q, 8) || !aligned(hi, 4) || !aligned(lo, 4)) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_rmsnorm_quant(x, w, w_scales, out, q, q_scales, (int)rows, (int)hidden,
                                           (int)norm_group, eps, inplace_form != 0, (int)hidden,
                                           (cudaStream_t)stream, hi, lo));
    return QVL_OK;
}

int qvl_quantize_rows_planes(const float *x, int16_t *q, float *q_scales, int8_t *hi, uint8_t *lo, size_t M,
                             size_t K, size_t group_size, void *stream) {
    if (!x || !q || !q_scales || !hi || !lo) return QVL_ERR_INVALID;
    if (!aligned(x, 16) || !aligned(q, 8) || !aligned(hi, 4) || !aligned(lo, 4)) return QVL_ERR_INVALID;
    if (M == 0 || K == 0 || group_size == 0 || K % group_size || group_size % 16) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_quantize_rows(x, q, q_scales, (int)M, (int)K, (int)group_size,
                                           (cudaStream_t)stream, hi, lo));
    return QVL_OK;
}

int qvl_swiglu_quantize_rows(const float *gate, const float *up, int16_t *q, float *q_scales,
                             size_t M, size_t I, size_t group_size, void *stream) {
    if (!gate || !up || !q || !q_scales) return QVL_ERR_INVALID;
    if (M == 0) return QVL_OK;
    if (group_size == 0 || group_size % 16 || I % group_size) return QVL_ERR_INVALID;
    if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(q, 8)) return QVL_ERR_INVALID;
    QVL_CUDA_TRY(qvl::launch_swiglu_quant(gate, up, q, q_scales, (int)M, (int)I, (int)group_size,
                                          (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_embedding_lookup_i8(const int8_t *table, const float *row_scales, const int32_t *token_ids,
                            float *out, size_t n_tokens, size_t vocab, size_t hidden, void *stream) {
    if (!table || !row_scales || !token_ids || !out || vocab == 0 || hidden == 0) return QVL_ERR_INVALID;
    if (n_tokens == 0) return QVL_OK;
    QVL_CUDA_TRY(qvl::launch_embedding_i8(table, row_scales, token_ids, out, (int)n_tokens, (int)hidden,
                                          (int)vocab, (cudaStream_t)stream));
    return QVL_OK;
}

size_t qvl_attention_workspace_bytes(size_t nq, int max_ctx, const qvl_attn_dims *dims) {
    if (check_attn_dims(dims) || max_ctx <= 0 || nq == 0) return 0;
    return qvl::attn_scratch_layout(nq, max_ctx, dims->num_heads, dims->num_kv_heads).total;
}

int qvl_attention_decode(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                         const int32_t *page_table, const int32_t *seq_ids,
                         const int32_t *positions, size_t nq, int max_ctx, float *out,
                         const qvl_attn_dims *dims, void *workspace, size_t workspace_bytes,
                         void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !k_pages || !v_pages || !page_table || !seq_ids || !positions || !out) return QVL_ERR_INVALID;
    if (max_ctx <= 0) return QVL_ERR_INVALID;
    if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(q, 16)) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    const size_t need = qvl_attention_workspace_bytes(nq, max_ctx, dims);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    qvl::AttnArgs a = {};
    a.q = q; a.k_pages = k_pages; a.v_pages = v_pages; a.page_table = page_table;
    a.seq_ids = seq_ids; a.positions = positions; a.nq = nq; a.max_ctx = max_ctx; a.out = out;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    QVL_CUDA_TRY(qvl::launch_attention(a, workspace, (cudaStream_t)stream));
    return QVL_OK;
}

size_t qvl_attention_ordered_workspace_bytes(size_t nq, int max_ctx, const qvl_attn_dims *dims) {
    if (check_attn_dims(dims) || max_ctx <= 0) return 0;
    return qvl::attn_ordered_workspace_bytes(nq, max_ctx, dims->num_heads);
}

int qvl_attention_decode_ordered(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                                 const int32_t *page_table, const int32_t *seq_ids, const int32_t *positions,
                                 size_t nq, int max_ctx, float *out, const qvl_attn_dims *dims, void *workspace,
                                 size_t workspace_bytes, void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !k_pages || !v_pages || !page_table || !seq_ids || !positions || !out) return QVL_ERR_INVALID;
    if (max_ctx <= 0) return QVL_ERR_INVALID;
    if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(q, 16)) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    if (nq > 65535) return QVL_ERR_UNSUPPORTED;
    const size_t need = qvl::attn_ordered_workspace_bytes(nq, max_ctx, dims->num_heads);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    qvl::AttnArgs a = {};
    a.q = q; a.k_pages = k_pages; a.v_pages = v_pages; a.page_table = page_table;
    a.seq_ids = seq_ids; a.positions = positions; a.nq = nq; a.max_ctx = max_ctx; a.out = out;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    QVL_CUDA_TRY(qvl::launch_attention_ordered(a, workspace, (cudaStream_t)stream));
    return QVL_OK;
}

int qvl_qknorm_rope_attention_decode_ordered(const float *q, const float *k_new, const float *v_new, uint16_t *k_pages,
                                             uint16_t *v_pages, const int32_t *page_table, const int32_t *seq_ids,
                                             const int32_t *positions, size_t nq, int max_ctx, const float *rope_cos,
                                             const float *rope_sin, const int8_t *q_norm_w, const float *q_norm_s,
                                             const int8_t *k_norm_w, const float *k_norm_s, size_t norm_group,
                                             float eps, float *out, const qvl_attn_dims *dims, void *workspace,
                                             size_t workspace_bytes, void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !k_new || !v_new || !k_pages || !v_pages || !page_table || !seq_ids || !positions || !out ||
        !rope_cos || !rope_sin)
        return QVL_ERR_INVALID;
    const bool has_norm = q_norm_w != nullptr;
    if (has_norm && (!q_norm_s || !k_norm_w || !k_norm_s)) return QVL_ERR_INVALID;
    if (has_norm && (norm_group == 0 || 128 % norm_group)) return QVL_ERR_UNSUPPORTED;
    if (max_ctx <= 0 || max_ctx > dims->max_pos) return QVL_ERR_INVALID;
    if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(q, 16)) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    if (nq > 65535) return QVL_ERR_UNSUPPORTED;
    const size_t need = qvl::attn_ordered_workspace_bytes(nq, max_ctx, dims->num_heads);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    qvl::AttnArgs a = {};
    a.q = q; a.k_pages = k_pages; a.v_pages = v_pages; a.page_table = page_table;
    a.seq_ids = seq_ids; a.positions = positions; a.nq = nq; a.max_ctx = max_ctx; a.out = out;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    qvl::OrdRope rp = {};
    rp.k_new = k_new; rp.v_new = v_new; rp.k_pages = k_pages; rp.v_pages = v_pages;
    rp.rope_cos = rope_cos; rp.rope_sin = rope_sin;
    rp.norm = qvl::QkNorm{q_norm_w, q_norm_s, k_norm_w, k_norm_s, has_norm ? (int)norm_group : 1, eps};
    QVL_CUDA_TRY(qvl::launch_attention_ordered(a, workspace, (cudaStream_t)stream, &rp));
    return QVL_OK;
}

int qvl_attention_decode_q16(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                             const int32_t *page_table, const int32_t *seq_ids, const int32_t *positions,
                             size_t nq, int max_ctx, float *out, int16_t *q_out, float *q_out_scales,
                             int *counter, const qvl_attn_dims *dims, void *workspace, size_t workspace_bytes,
                             void *stream) {
    int rc = check_attn_dims(dims);
    if (rc) return rc;
    if (!q || !k_pages || !v_pages || !page_table || !seq_ids || !positions || !out || !q_out ||
        !q_out_scales || !counter)
        return QVL_ERR_INVALID;
    if (max_ctx <= 0) return QVL_ERR_INVALID;
    if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(q, 16) || !aligned(out, 16)) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    const size_t need = qvl_attention_workspace_bytes(nq, max_ctx, dims);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256)) return QVL_ERR_WORKSPACE;
    qvl::AttnArgs a = {};
    a.q = q; a.k_pages = k_pages; a.v_pages = v_pages; a.page_table = page_table;
    a.seq_ids = seq_ids; a.positions = positions; a.nq = nq; a.max_ctx = max_ctx; a.out = out;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    const bool fused = qvl::attn_use_cluster(nq, max_ctx, a.NKV);
    if (fused) {
        a.q_out = q_out; a.q_out_scales = q_out_scales; a.counter = counter;
    }
    cudaStream_t st = (cudaStream_t)stream;
    QVL_CUDA_TRY(qvl::launch_attention(a, workspace, st));
    if (!fused) {
        const int H = dims->num_heads * dims->head_dim;
        QVL_CUDA_TRY(qvl::launch_quantize_rows(out, q_out, q_out_scales, (int)nq, H, H, st));
    }
    return QVL_OK;
}

int qvl_argmax_rows(const float *logits, int32_t *idx, size_t rows, size_t n, void *stream) {
    if (!logits || !idx || n == 0 || n > (size_t)INT32_MAX) return QVL_ERR_INVALID;
    if (rows == 0) return QVL_OK;
    QVL_CUDA_TRY(qvl::launch_argmax_rows(logits, idx, (long)rows, (long)n, (cudaStream_t)stream));
    return QVL_OK;
}

}  // extern "C"
