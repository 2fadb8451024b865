/* qvl_b200.h -- C ABI of the B200 (sm_100a) INT8 hot path of the Qwen3-VL-2B
 * inference engine (drop-in for dangtruong-github/qwen3-vl-2b-inference's
 * matmul/ INT8 kernels, SwiGLU MLP and GQA attention).
 *
 * Conventions for every entry point
 *   - All tensor pointers are DEVICE pointers unless the name ends in _host.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Calls are asynchronous on `stream`; they return a status code and never
 *     call exit() or trap.  The reference's error convention (fprintf + exit(1)
 *     on an unsupported dtype combination, matmul/src/cpu_wrapper.cpp:394-395)
 *     is kept only by the C++ `linear()` shim in qvl_b200_linear.hpp.
 *   - Nothing allocates device memory on the hot path: scratch is a caller-
 *     provided `workspace` whose size the matching *_workspace_bytes()
 *     function reports.
 *   - Weights use the reference's packed layout unchanged
 *     (export_bin/export_qwen_bin.py:242-275, 297-357): int8 row-major [N, K]
 *     (HF [out, in]); fp32 scales [N * K / group_size] with row n, group gi at
 *     n * (K / group_size) + gi.  Per-output-row quantisation is
 *     group_size == K.
 */
#ifndef QVL_B200_H
#define QVL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define QVL_OK 0
#define QVL_ERR_INVALID 1       /* bad pointer, size or alignment            */
#define QVL_ERR_UNSUPPORTED 2   /* shape/dtype combination not implemented    */
#define QVL_ERR_CUDA 3          /* a CUDA runtime call failed                  */
#define QVL_ERR_WORKSPACE 4     /* workspace missing or too small              */

/* Reference dtype enum (utils/include/tensor.hpp:25-27), same values. */
#define QVL_DTYPE_FP32 0
#define QVL_DTYPE_INT32 1
#define QVL_DTYPE_FP16 2
#define QVL_DTYPE_INT8 3
#define QVL_DTYPE_INT4 4

/* Floating-point summation semantics of the INT8 products.
 * The integer group sums are exact in all modes; the modes differ only in how
 * the fp32 result is assembled from them, mirroring the reference kernels:
 *   QVL_SEM_REFERENCE: what f32a_i8f32sb_f32c_avx2_kernel does for this shape
 *       (cpu_f32a_i8f32sb_f32c_avx2.cpp:464-475): LANE8 when M == 1 &&
 *       N >= 1024 && K >= 1024, TILED otherwise.
 *   QVL_SEM_LANE8: every row is an independent M=1 decode GEMV (:122-224 and
 *       :327-455): 8 int32 lanes per group (k mod 16 in {2l, 2l+1}), each lane
 *       fused into an fp32 lane accumulator, lanes reduced (l, l+4) pairwise.
 *       Use this for a batch of independent decode requests.
 *   QVL_SEM_TILED: the M>1 kernel (:538-653): per group the whole int32 sum
 *       is converted and accumulated as fma(float(S) * a_s, w_s, acc). */
/* OR-ed into `semantics`: add the product into C (C += A.B^T) instead of
 * overwriting it -- the residual add_vector after o_proj/down_proj
 * (model/src/forward.cpp:604, :661), same rounding as a separate add. */
#define QVL_SEM_ACCUMULATE 0x100
#define QVL_SEM_REFERENCE 0
#define QVL_SEM_LANE8 1
#define QVL_SEM_TILED 2

const char *qvl_status_string(int status);
/* Tensor-core timeout word of the current device.  The tensor-core path
 * (M >= 16 products) bounds every wait; a wait that gives up sets the word,
 * and while it is set every tensor-core launch on that device leaves without
 * computing.  Launches are asynchronous, so the call that timed out still
 * returned QVL_OK: this synchronises `stream`, stores 1 in *timed_out if the
 * word is set (the outputs since it was last cleared are invalid) and, with
 * `clear`, resets it so that the path computes again.  No counterpart in the
 * reference (its operators are synchronous and cannot time out). */
int qvl_tc_timeout_status(int *timed_out, int clear, void *stream);
/* Last CUDA error code recorded by a QVL_ERR_CUDA return (0 if none). */
int qvl_last_cuda_error(void);
/* Library version, e.g. "qvl_b200 0.1". */
const char *qvl_version(void);

/* ---- activation quantisation (inlined in every reference INT8 kernel,
 *      cpu_f32a_i8f32sb_f32c_avx2.cpp:135-177, :348-390, :488-530) ---------
 * x fp32 [M, K] -> q int16 [M, K], q_scales fp32 [M, K / group_size]:
 * s = sqrtf(sum(x^2) / g + 1e-6) / 127 per group, q = sat16(rne(x / s)).
 * Requires K % group_size == 0, group_size % 16 == 0, x 16-byte and q
 * 8-byte aligned. */
int qvl_quantize_rows(const float *x, int16_t *q, float *q_scales,
                      size_t M, size_t K, size_t group_size, void *stream);
/* qvl_quantize_rows that also writes the hi/lo planes of q (see
 * qvl_linear_planes_i8_batched); hi/lo 4-byte aligned. */
int qvl_quantize_rows_planes(const float *x, int16_t *q, float *q_scales, int8_t *hi, uint8_t *lo, size_t M,
                             size_t K, size_t group_size, void *stream);

/* ---- INT8 linear: C[M,N] = A[M,K] . dequant(B[N,K])^T, fp32 in/out -------
 * Replaces linear()'s INT8 branch (matmul/src/cpu_wrapper.cpp:339-357) and
 * the kernels behind it (f32a_i8f32sb_f32c_avx2_kernel,
 * matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:665-702).
 * group_quantized == 0 means per-output-row scales (group_size := K); the
 * reference's own row-quant branch reads B as [K, N] (cpu_wrapper.cpp:172-215)
 * and is not reproduced.  Workspace holds the quantised activations. */
size_t qvl_linear_i8_workspace_bytes(size_t M, size_t K, size_t group_size);
int qvl_linear_i8(const float *A, const int8_t *B, const float *B_scales, float *C,
                  size_t M, size_t N, size_t K, int group_quantized, size_t group_size,
                  int semantics, void *workspace, size_t workspace_bytes, void *stream);

/* Same product from already-quantised activations (qvl_quantize_rows output),
 * so q/k/v or gate/up share one quantisation of their common input. */
int qvl_linear_q16_i8(const int16_t *q, const float *q_scales, const int8_t *B,
                      const float *B_scales, float *C, size_t M, size_t N, size_t K,
                      size_t group_size, int semantics, void *stream);

/* Several products of the same activations in one launch (q/k/v from the
 * normalised hidden state, or gate/up): C[i] = q . dequant(B[i])^T for
 * i < n_mats <= 3, each B[i] int8 [N[i], K] with its own scales.  Host arrays
 * of device pointers.  Results equal n_mats separate qvl_linear_q16_i8 calls. */
int qvl_linear_q16_i8_multi(const int16_t *q, const float *q_scales, size_t n_mats,
                            const int8_t *const *B, const float *const *B_scales, float *const *C,
                            const size_t *N, size_t M, size_t K, size_t group_size, int semantics,
                            void *stream);

/* gate/up projections with SwiGLU in the epilogue (model/src/forward.cpp:
 * 621-642): h[M, I] = swiglu(q . dequant(Wg)^T, q . dequant(Wu)^T) without
 * writing gate or up.  One launch when M <= 4 and group_size >= 128; other
 * shapes run the two products and swiglu separately and need up_scratch
 * (fp32 [M, I]; nullable otherwise).  Values equal the unfused sequence. */
int qvl_gate_up_swiglu_q16_i8(const int16_t *q, const float *q_scales, const int8_t *Wg,
                              const float *sg, const int8_t *Wu, const float *su, float *h,
                              float *up_scratch, size_t M, size_t I, size_t K, size_t group_size,
                              int semantics, void *stream);

/* Fused tail of a product: after the last output of the launch is written,
 * the row(s) of C[0] (length N[0]) are RMS-normalised (norm_w != NULL;
 * qvl_rms_norm_i8 arithmetic) and/or quantised for the next linear --
 * e.g. o_proj + residual -> post-attention rms_norm -> gate/up input, or
 * down_proj + residual -> next layer's input rms_norm -> q/k/v input.
 * `counter` is a device int that must be 0 before the first call; each call
 * leaves it 0 again (calls that overlap on the GPU need distinct counters). */
typedef struct {
    int *counter;
    const int8_t *norm_w;     /* NULL: quantise C[0] as is */
    const float *norm_s;
    size_t norm_group;
    float eps;
    int inplace_form;         /* 1: rms_norm_inplace rounding */
    float *norm_out;          /* normalised copy of C[0] (nullable, may alias C[0]) */
    int16_t *q;               /* quantised activations for the next linear */
    float *q_scales;
    size_t quant_group;
} qvl_row_tail;

/* qvl_linear_q16_i8_multi (or, with swiglu_pair = 1 and two matrices, the
 * gate/up + SwiGLU product of qvl_gate_up_swiglu_q16_i8 writing C[0]) plus
 * the fused row tail.  One launch when M <= 4 and group_size >= 128; other
 * shapes run the same steps as separate launches. */
int qvl_linear_q16_i8_tail(const int16_t *q, const float *q_scales, size_t n_mats,
                           const int8_t *const *B, const float *const *B_scales, float *const *C,
                           const size_t *N, size_t M, size_t K, size_t group_size, int semantics,
                           int swiglu_pair, const qvl_row_tail *tail, void *stream);

/* Batched products on the tensor cores (tcgen05 kind::i8), the reference's
 * M>1 (TILED) order: the int16 activations q [M, K] (qvl_quantize_rows /
 * qvl_rms_norm_i8 output, per-row quantisation: one scale per row) are split
 * once into the workspace (qvl_linear_q16_i8_batched_workspace_bytes) and
 * reused by every matrix; per-row weight scales (group = K), K % 128 == 0,
 * N[i] >= 128, M >= 16.  QVL_SEM_ACCUMULATE adds into C.  swiglu_pair = 1:
 * two matrices (gate, up) and C[0] = swiglu(gate, up) with up in up_scratch. */
size_t qvl_linear_q16_i8_batched_workspace_bytes(size_t M, size_t K);
int qvl_linear_q16_i8_batched(const int16_t *q, const float *q_scales, size_t n_mats,
                              const int8_t *const *B, const float *const *B_scales, float *const *C,
                              const size_t *N, size_t M, size_t K, int semantics, int swiglu_pair,
                              float *up_scratch, void *workspace, size_t workspace_bytes, void *stream);

/* The same products from activations already split into the tensor cores'
 * hi/lo planes (hi = q >> 8 int8, lo = q & 255 uint8, [M, K] each, 16-byte
 * aligned) -- as the *_planes producers below write them -- in one launch
 * over all n_mats (<= 3) matrices.  TILED order, per-output-row scales. */
int qvl_linear_planes_i8_batched(const int8_t *hi, const uint8_t *lo, const float *q_scales, size_t n_mats,
                                 const int8_t *const *B, const float *const *B_scales, float *const *C,
                                 const size_t *N, size_t M, size_t K, int semantics, void *stream);

/* ---- SwiGLU (layers/src/text_layer.cpp:420-434) ------------------------
 * gate[i] = gate[i] / (1 + exp(-gate[i])) * up[i], in place, n elements. */
int qvl_swiglu(float *gate, const float *up, size_t n, void *stream);

/* swiglu followed by the down projection's activation quantisation, without
 * materialising the fp32 SwiGLU output: q/q_scales = quantize_rows(
 * swiglu(gate, up)) for M rows of I values (gate/up are not modified;
 * gate/up 16-byte and q 8-byte aligned). */
int qvl_swiglu_quantize_rows(const float *gate, const float *up, int16_t *q, float *q_scales,
                             size_t M, size_t I, size_t group_size, void *stream);


/* Fused MLP chain: out[M,H] = down(swiglu(gate(x), up(x))), the sequence of
 * model/src/forward.cpp:621-654 (gate/up linear, swiglu, down linear).
 * Wg, Wu: int8 [I, H]; Wd: int8 [H, I]; scales in the reference layout.
 * group_size 0 = per-output-row scales for all three (gate/up [I], down [H]:
 * the group is each product's K); otherwise one group size for all three.
 * Workspace: qvl_swiglu_mlp_workspace_bytes(M, H, I, group_size). */
size_t qvl_swiglu_mlp_workspace_bytes(size_t M, size_t H, size_t I, size_t group_size);
int qvl_swiglu_mlp_i8(const float *x, const int8_t *Wg, const float *sg,
                      const int8_t *Wu, const float *su, const int8_t *Wd,
                      const float *sd, float *out, size_t M, size_t H, size_t I,
                      size_t group_size, int semantics, void *workspace,
                      size_t workspace_bytes, void *stream);

/* ---- GQA attention over a paged FP16 KV cache --------------------------
 * Replaces apply_rotary / apply_rotary_cache / the v-cache copy
 * (layers/src/text_layer.cpp:712-824, model/src/forward.cpp:545-562) and
 * attn_scores_all_heads + softmax + attn_weighted_sum_all_heads
 * (layers/src/text_layer.cpp:436-710).
 *
 * KV layout (per layer): k_pages, v_pages fp16 [num_pages, NKV, page_size, D].
 * page_table int32 [num_seqs, max_pages_per_seq]: logical page p of sequence s
 * lives at physical page page_table[s * max_pages_per_seq + p].
 * Query i belongs to sequence seq_ids[i] at position positions[i] and attends
 * causally over positions [0, positions[i]].
 * rope_cos/rope_sin fp32 [max_pos, D/2]: the text section of the reference's
 * table (model/src/load_model.cpp:413-490), computed on the host.
 *
 * qvl_rope_kv_append: q fp32 [nq, NH, D] rotated in place; k_new, v_new fp32
 * [nq, NKV, D]: k rotated, both rounded to fp16 and written at their position.
 * qvl_attention_decode: out fp32 [nq, NH, D]. */
/* Host function (no device work): the RoPE table the attention entry points
 * take, computed as the reference's qwen_rope_precompute computes its text
 * section (model/src/load_model.cpp:413-490) with the host's single-precision
 * libm: cos/sin of pos / powf(theta, 2i/head_dim); theta is an integer there
 * (the header stores rope_theta as int, :71).  cos_out, sin_out: host
 * float [rows, head_dim/2]. */
int qvl_rope_table(int theta, int head_dim, int rows, float *cos_out, float *sin_out);

typedef struct {
    int num_heads;          /* NH  (16 for Qwen3-VL-2B)                 */
    int num_kv_heads;       /* NKV (8)                                  */
    int head_dim;           /* D   (128; only 128 is implemented)       */
    int page_size;          /* tokens per page (multiple of 16)         */
    int max_pages_per_seq;  /* row stride of page_table                 */
    int max_pos;            /* rows of rope_cos / rope_sin              */
} qvl_attn_dims;

int qvl_rope_kv_append(float *q, const float *k_new, const float *v_new,
                       uint16_t *k_pages, uint16_t *v_pages, const int32_t *page_table,
                       const int32_t *seq_ids, const int32_t *positions, size_t nq,
                       const float *rope_cos, const float *rope_sin,
                       const qvl_attn_dims *dims, void *stream);
size_t qvl_attention_workspace_bytes(size_t nq, int max_ctx, const qvl_attn_dims *dims);
int qvl_attention_decode(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                         const int32_t *page_table, const int32_t *seq_ids,
                         const int32_t *positions, size_t nq, int max_ctx, float *out,
                         const qvl_attn_dims *dims, void *workspace,
                         size_t workspace_bytes, void *stream);

/* qvl_attention_decode in the reference's own summation order, bit for bit
 * given the same fp16-valued cache: each score in the order of
 * attn_scores_all_heads (the 8-position unrolled loop and its 0-7 tail,
 * layers/src/text_layer.cpp:575-650), softmax's 8 float lanes plus double
 * tail (:436-535), and one fma chain over t ascending per output element
 * (attn_weighted_sum_all_heads, :655-710).  The chains run sequentially, so
 * this is slower than qvl_attention_decode at long contexts; it is the
 * attention of the decoder's reference-order mode.  workspace:
 * qvl_attention_ordered_workspace_bytes(nq, max_ctx, dims) bytes (scores,
 * 256-byte aligned); nq <= 65535. */
size_t qvl_attention_ordered_workspace_bytes(size_t nq, int max_ctx, const qvl_attn_dims *dims);
int qvl_attention_decode_ordered(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                                 const int32_t *page_table, const int32_t *seq_ids,
                                 const int32_t *positions, size_t nq, int max_ctx, float *out,
                                 const qvl_attn_dims *dims, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* One decode step's QK-norm + RoPE + KV append (qvl_qknorm_rope_kv_append,
 * model/src/forward.cpp:531-562) fused into qvl_attention_decode_ordered
 * (layers/src/text_layer.cpp:436-710): q fp32 [nq, NH, D], k_new/v_new fp32
 * [nq, NKV, D] are the raw projections (q is not modified); k (rotated) and v
 * are rounded to fp16 and written at each query's position, and out equals
 * qvl_qknorm_rope_kv_append followed by qvl_attention_decode_ordered bit for
 * bit.  Every query must belong to a different sequence (a decode batch),
 * and the cache rows before each query's position must be complete when the
 * call is made (the P.V pass may fetch them while the score pass still runs);
 * max_ctx <= dims->max_pos.  q_norm_w NULL: no QK-norm (all four NULL).
 * Workspace as qvl_attention_decode_ordered. */
int qvl_qknorm_rope_attention_decode_ordered(const float *q, const float *k_new, const float *v_new, uint16_t *k_pages,
                                             uint16_t *v_pages, const int32_t *page_table, const int32_t *seq_ids,
                                             const int32_t *positions, size_t nq, int max_ctx, const float *rope_cos,
                                             const float *rope_sin, const int8_t *q_norm_w, const float *q_norm_s,
                                             const int8_t *k_norm_w, const float *k_norm_s, size_t norm_group,
                                             float eps, float *out, const qvl_attn_dims *dims, void *workspace,
                                             size_t workspace_bytes, void *stream);

/* qvl_attention_decode followed by the activation quantisation of each
 * output row (one scale per row, the o_proj input): q_out int16 [nq, NH*D],
 * q_out_scales fp32 [nq].  Fused into the attention launch when it runs as
 * one launch; `counter` is a device int that must be 0 before the first call
 * and is left 0. */
int qvl_attention_decode_q16(const float *q, const uint16_t *k_pages, const uint16_t *v_pages,
                             const int32_t *page_table, const int32_t *seq_ids, const int32_t *positions,
                             size_t nq, int max_ctx, float *out, int16_t *q_out, float *q_out_scales,
                             int *counter, const qvl_attn_dims *dims, void *workspace, size_t workspace_bytes,
                             void *stream);

/* QK-norm + RoPE + KV append in one launch: rms_norm_inplace of every q and
 * k head with the layer's INT8 q_norm / k_norm weights (model/src/forward.cpp:
 * 531-538; layers/src/text_layer.cpp:234-272), then qvl_rope_kv_append.
 * q_norm_w/k_norm_w int8 [D], *_s fp32 [D / norm_group]. */
int qvl_qknorm_rope_kv_append(float *q, const float *k_new, const float *v_new, uint16_t *k_pages,
                              uint16_t *v_pages, const int32_t *page_table, const int32_t *seq_ids,
                              const int32_t *positions, size_t nq, const float *rope_cos,
                              const float *rope_sin, const int8_t *q_norm_w, const float *q_norm_s,
                              const int8_t *k_norm_w, const float *k_norm_s, size_t norm_group,
                              float eps, const qvl_attn_dims *dims, void *stream);

/* ---- RMSNorm and embedding (layers/src/text_layer.cpp:3-300) ------------
 * qvl_rms_norm_i8: rows x hidden fp32 -> out (nullable) and/or its
 * activation quantisation q/q_scales (nullable) for the next linear.
 * Weight: INT8 [hidden] with fp32 scales [hidden / norm_group] (norm weights
 * are always group-quantised by the exporter).  inplace_form selects the
 * rms_norm_inplace rounding (1.0f/sqrtf) instead of rms_norm's
 * (float)(1.0/sqrtf); the result is written to `out` either way.
 * hidden <= 16384, hidden / quant_group <= 64. */
int qvl_rms_norm_i8(const float *x, const int8_t *w, const float *w_scales, float *out,
                    int16_t *q, float *q_scales, size_t rows, size_t hidden, size_t norm_group,
                    float eps, int inplace_form, size_t quant_group, void *stream);
/* qvl_rms_norm_i8 with per-row quantisation (group = hidden) that also
 * writes the hi/lo planes of q for qvl_linear_planes_i8_batched. */
int qvl_rms_norm_i8_planes(const float *x, const int8_t *w, const float *w_scales, float *out, int16_t *q,
                           float *q_scales, int8_t *hi, uint8_t *lo, size_t rows, size_t hidden,
                           size_t norm_group, float eps, int inplace_form, void *stream);
/* embedding_lookup for an INT8 table with per-row scales (the tied
 * embedding / LM-head matrix): out[t] = table[ids[t]] * row_scales[ids[t]]. */
int qvl_embedding_lookup_i8(const int8_t *table, const float *row_scales, const int32_t *token_ids,
                            float *out, size_t n_tokens, size_t vocab, size_t hidden, void *stream);

/* ---- attention without a caller workspace -----------------------------
 * No counterpart in the reference.  Same inputs, outputs and result as
 * qvl_attention_decode, but the split-K scratch lives in a fixed device array
 * compiled into this library instead of a caller-provided workspace.  It is
 * for hosts that cannot allocate device memory when they call in: a plugin
 * running inside a framework that owns all device memory through its own
 * allocator, or a caller that must not allocate on its serving path.
 * Limits and rules:
 *   - The scratch is QVL_ATTN_STATIC_SCRATCH_BYTES per GPU that loads this
 *     library, held until process exit.  A call that needs more
 *     (qvl_attention_workspace_bytes(nq, max_ctx, dims) larger than that)
 *     returns QVL_ERR_WORKSPACE and launches nothing.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress with that device current); make that first call
 *     before any stream capture on the device.
 *   - Every call on a device shares the one array, so calls whose kernels may
 *     overlap on the GPU (different streams without ordering) race; order
 *     them on one stream.  No scratch entry is read before the same call
 *     writes it, so nothing needs clearing between calls.
 *   - Calls no allocator (no cudaMalloc/cudaFree). */
#define QVL_ATTN_STATIC_SCRATCH_BYTES (32u << 20)
int qvl_attention_decode_static(const float *q, const uint16_t *k_pages,
                                const uint16_t *v_pages, const int32_t *page_table,
                                const int32_t *seq_ids, const int32_t *positions, size_t nq,
                                int max_ctx, float *out, const qvl_attn_dims *dims,
                                void *stream);

/* ---- greedy decode (tokenizer/src/utils.cpp:34-44) ---------------------
 * idx[r] = first index of the maximum of logits[r, :n] (strict >, from
 * -FLT_MAX; NaN never wins; all-NaN/-inf rows give 0). */
int qvl_argmax_rows(const float *logits, int32_t *idx, size_t rows, size_t n, void *stream);

/* ---- one whole decode token in one launch (batch 1) ---------------------
 * Replaces, for one request, the per-token text decoder of forward_text
 * (model/src/forward.cpp:458-720) followed by greedy_decode
 * (tokenizer/src/utils.cpp:34-44): embedding lookup of *token, 28 x (input
 * rms_norm, q/k/v linear, q/k rms_norm_inplace + RoPE, KV append, attention,
 * o_proj + residual, post rms_norm, gate/up + SwiGLU, down + residual), final
 * rms_norm_inplace, LM head (tied embedding) into `logits`, greedy token into
 * *token, *pos += 1.  `token` and `pos` stay on the device, so consecutive
 * calls (or a captured graph of them) decode without host round trips.
 *
 * One cooperative kernel: every CTA stays resident for the whole token and
 * the phases meet at a grid barrier whose waits are bounded (2 s); a timeout
 * sets an abort word in the workspace (qvl_text_decode_abort_flag) and every
 * CTA leaves.  A call whose *pos is outside [0, max_ctx) or whose *token is
 * outside [0, vocab) decodes nothing: it sets the abort word to 2 (position)
 * or 3 (token) and leaves token, pos, x, logits and the KV cache unchanged.
 * rope_cos / rope_sin need max_ctx rows.  Arithmetic per operation is that of the separate entry points
 * with QVL_SEM_LANE8 (M=1 GEMV order); the attention splits each context into
 * 16 slices, so its fp32 partial sums are grouped differently.
 *
 * Supported: Qwen3-VL-2B text dims (hidden 2048, intermediate 6144, 16 heads,
 * 8 KV heads, head_dim 128), per-output-row INT8 linear weights (group_size
 * == K), vocab a multiple of 16, page_size a multiple of 16, max_ctx <= 8192;
 * weight matrices and their scale arrays 16-byte aligned.  Weights are stacked over layers: w_q [L, 2048,
 * 2048] etc., s_q [L, 2048]; norm weights int8 [L, n] with fp32 group scales
 * [L, n / norm_group].  KV pages [L][pages, 8, page_size, 128] fp16, layer l at
 * l * kv_layer_stride elements; page_table [ceil(max_ctx / page_size)].
 * workspace: qvl_text_decode_workspace_bytes() bytes, ZERO-FILLED before the
 * first call and then kept (it holds the barrier words); calls sharing one
 * workspace must be ordered on one stream. */
typedef struct {
    const int8_t *w_q, *w_k, *w_v, *w_o, *w_gate, *w_up, *w_down;
    const float *s_q, *s_k, *s_v, *s_o, *s_gate, *s_up, *s_down;
    const int8_t *in_norm, *post_norm, *q_norm, *k_norm;
    const float *in_norm_s, *post_norm_s, *q_norm_s, *k_norm_s;
    const int8_t *final_norm;
    const float *final_norm_s;
    const int8_t *embed;          /* [vocab, hidden], also the LM head */
    const float *embed_s;         /* [vocab] */
    int layers, vocab, hidden, intermediate, heads, kv_heads, head_dim, norm_group;
    float eps;
} qvl_text_weights;

size_t qvl_text_decode_workspace_bytes(void);
int qvl_text_decode_step(const qvl_text_weights *w, float *x, float *logits, int32_t *token,
                         int32_t *pos, uint16_t *k_pages, uint16_t *v_pages, long kv_layer_stride,
                         const int32_t *page_table, int page_size, const float *rope_cos,
                         const float *rope_sin, int max_ctx, void *workspace,
                         size_t workspace_bytes, void *stream);
/* qvl_text_decode_step with flags.  QVL_DECODE_REFERENCE_ORDER: attention in
 * the reference's own summation order (see qvl_attention_decode_ordered), so
 * that the whole token -- logits and greedy id -- is bit-identical to the
 * reference's operators on the same fp16-valued cache; the softmax sum and
 * the P.V chains then run sequentially over the context in one CTA per KV
 * head, which costs a few microseconds per layer. */
#define QVL_DECODE_REFERENCE_ORDER 1
int qvl_text_decode_step_ex(const qvl_text_weights *w, float *x, float *logits, int32_t *token,
                            int32_t *pos, uint16_t *k_pages, uint16_t *v_pages, long kv_layer_stride,
                            const int32_t *page_table, int page_size, const float *rope_cos,
                            const float *rope_sin, int max_ctx, void *workspace,
                            size_t workspace_bytes, int flags, void *stream);
/* Device address of the abort word inside `workspace` (int): 0 healthy, 1 a
 * bounded wait gave up, 2 position out of range, 3 token out of range. */
int *qvl_text_decode_abort_flag(void *workspace);
/* Device address of the phase trace inside `workspace`: 256 uint64
 * global-timer stamps (ns) of the last call -- [0] kernel start, [1 + i] the
 * opening of grid barrier i (5 per layer + 1 barriers per token). */
const uint64_t *qvl_text_decode_trace(const void *workspace);

/* ---- vision tower (FP16 weights; forward_img, model/src/forward.cpp:3-456)
 * fp16 tensors are passed as uint16_t.  Token-major layouts throughout:
 * activations [T, features], attention q/k/v/out [T, heads, head_dim] (the
 * reference's transposes to head-major, tensor_transpose, are folded into the
 * attention's indexing).  Parity with the reference is by tolerance. */

/* Host functions (no device work).  qvl_vision_rot_table: the per-patch 2-D
 * rotary tables of qwen_vision_rope_precompute + vision_rot_pos_emb
 * (model/src/load_model.cpp:492-540, layers/src/vision_layer.cpp:506-623)
 * with the host libm, fp16, in merge order: cos/sin [grid_h*grid_w,
 * head_dim].  qvl_vision_pos_interp: the 4 taps (indices into the
 * num_grid_per_side^2 learned table) and bilinear weights of each patch in
 * merge order, as vision_pos_embed computes them (vision_layer.cpp:219-504):
 * idx int32 [T, 4], w float [T, 4]. */
int qvl_vision_rot_table(float theta, int head_dim, int grid_h, int grid_w, int merge, uint16_t *cos_out,
                         uint16_t *sin_out);
int qvl_vision_pos_interp(int grid_h, int grid_w, int num_grid_per_side, int merge, int32_t *idx_out,
                          float *w_out);

/* conv_3d (vision_layer.cpp:3-217) as a product: x fp32 [T, VH] =
 * patches fp32 [T, Kp] . w fp16 [VH, Kp]^T + b fp16 [VH]. */
int qvl_vision_patch_embed(const float *patches, const uint16_t *w, const uint16_t *b, float *x, int T, int VH,
                           int Kp, void *stream);
/* vision_pos_embed + add_vector: x[t] += fp16(sum_k pos_w[idx[t][k]] * w[t][k]). */
int qvl_vision_pos_add(float *x, const uint16_t *pos_w, const int32_t *idx, const float *wts, int T, int VH,
                       void *stream);
/* layer_norm (vision_layer.cpp:625-724): rows of H values, fp32 or fp16 in
 * and out (x_f16, out_f16), fp16 gamma / beta. */
int qvl_layer_norm(const void *x, int x_f16, const uint16_t *gamma, const uint16_t *beta, void *out, int out_f16,
                   int rows, int H, float eps, void *stream);
/* FP16 tensor-core product with bias, replacing linear() with FP16 weights
 * (matmul/src/cpu_fp16_full_avx2.cpp, cpu_wrapper.cpp:359-390):
 * C[M, N] = A[M, K] . W[N, K]^T + bias, fp32 accumulation; mode 0: C fp16,
 * 1: C fp16 after gelu_tanh of the fp16 value (the in-place gelu_tanh that
 * follows the vision MLP's first linear), 2: C fp32, 3: C fp32 += the fp16
 * value (linear then add_vector into the residual stream).  N >= 128,
 * K % 64 == 0, 16-byte aligned rows. */
int qvl_gemm_f16(const uint16_t *A, const uint16_t *W, const uint16_t *bias, void *C, size_t M, size_t N, size_t K,
                 int mode, void *stream);
/* vision_apply_rotary_inplace (vision_layer.cpp:726-776) on x [T, NH, HD]. */
int qvl_vision_rotary(uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t, int T, int NH, int HD,
                      void *stream);
/* vision_att (vision_layer.cpp:821-867): full attention per head, fp32
 * scores times `scale`, exp256_ps softmax, fp16 out; HD = 64, T <= 2048. */
int qvl_vision_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out, int T, int NH,
                         int HD, float scale, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QVL_B200_H */
