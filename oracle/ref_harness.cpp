// Test infrastructure only (not shipped, not on any product path).
//
// A plain C ABI over the reference engine's own compiled CPU operators, so
// the Python tests can call them through ctypes on the same seeded buffers
// that the CUDA path receives.  Nothing here re-implements arithmetic: every
// function forwards to the reference symbol named in its comment.
//
// Reference Tensor objects are built as non-owning wrappers around caller
// memory.  The reference destructor munmaps non-owning buffers
// (utils/src/tensor.cpp:71-110), so each wrapper's pointers are cleared
// before it goes out of scope.
#include <cstddef>
#include <cstdint>
#include <vector>
#include <cstdio>
#include <unistd.h>
#include "matmul/module.hpp"
#include "utils/module.hpp"
#include "layers/include/text_layer.hpp"

namespace {
struct Wrap {
    Tensor t;
    Wrap(const std::vector<size_t> &shape, void *buf) : t(shape, buf, DType::FP32) {}
    ~Wrap() { t.buf = nullptr; t.scale_buf = nullptr; }
};

// The reference prints a line per Tensor construction; keep test logs quiet.
struct QuietStdout {
    int saved = -1;
    QuietStdout() {
        fflush(stdout);
        saved = dup(1);
        FILE *null = fopen("/dev/null", "w");
        if (null) { dup2(fileno(null), 1); fclose(null); }
    }
    ~QuietStdout() {
        fflush(stdout);
        if (saved >= 0) { dup2(saved, 1); close(saved); }
    }
};
}  // namespace

extern "C" {

// matmul/src/cpu_f32a_i8f32sb_f32c_avx2.cpp:665 (transposed B = [N,K] row-major).
// M==1 && N>=1024 && K>=1024 -> gemv (:122) or gemv_decode (:327); else tiled (:458).
void ref_i8_kernel(const float *x, const int8_t *w, const float *ws, float *y,
                   size_t M, size_t N, size_t K, size_t group_size) {
    f32a_i8f32sb_f32c_avx2_kernel(x, w, ws, y, M, N, K, true, group_size);
}

// matmul/src/cpu_wrapper.cpp:308 `linear` with FP32 A/C, INT8 B, FP32 scales.
void ref_linear_i8(const float *x, const int8_t *w, const float *ws, float *y,
                   size_t M, size_t N, size_t K, int group_quantized, size_t group_size) {
    linear(x, w, ws, nullptr, nullptr, y, M, N, K, true, DType::FP32, DType::INT8,
           DType::FP32, DType::FP32, group_quantized != 0, group_size);
}

// layers/src/text_layer.cpp:420
void ref_swiglu(float *gate, const float *up, size_t n) {
    QuietStdout q;
    Wrap g({n}, gate), u({n}, const_cast<float *>(up));
    swiglu(&g.t, &u.t, n);
}

// layers/src/text_layer.cpp:437
void ref_softmax(float *x, size_t n) { softmax(x, n); }

// layers/src/text_layer.cpp:712; cos/sin tables are [S, head_dim/2] rows.
void ref_apply_rotary(float *x, const float *cos_tab, const float *sin_tab,
                      size_t S, int n_heads, int head_dim, int pos) {
    QuietStdout q;
    Wrap xt({(size_t)n_heads * head_dim}, x);
    Wrap c({S, (size_t)head_dim / 2}, const_cast<float *>(cos_tab));
    Wrap s({S, (size_t)head_dim / 2}, const_cast<float *>(sin_tab));
    apply_rotary(&xt.t, &c.t, &s.t, n_heads, head_dim, pos);
}

// layers/src/text_layer.cpp:767; writes head h at k_out + h*sh_off.
void ref_apply_rotary_cache(const float *k_in, float *k_out, const float *cos_tab,
                            const float *sin_tab, size_t S, int n_heads, int head_dim,
                            int pos, size_t sh_off) {
    QuietStdout q;
    Wrap xt({(size_t)n_heads * head_dim}, const_cast<float *>(k_in));
    Wrap c({S, (size_t)head_dim / 2}, const_cast<float *>(cos_tab));
    Wrap s({S, (size_t)head_dim / 2}, const_cast<float *>(sin_tab));
    apply_rotary_cache(&xt.t, k_out, &c.t, &s.t, n_heads, head_dim, pos, sh_off);
}

// layers/src/text_layer.cpp:575 + :655 for one layer of one request.
// key_cache / value_cache: [NKV, S, D] fp32; q: [NH, D]; att scratch: [NH, S];
// out: [NH, D].
void ref_attention(const float *key_cache, const float *value_cache, const float *q,
                   float *att, float *out, int NH, int NKV, int D, size_t S, int pos) {
    QuietStdout qs;
    Wrap qt({1, (size_t)NH, (size_t)D}, const_cast<float *>(q));
    Wrap at({1, (size_t)NH, S}, att);
    Wrap ot({1, (size_t)NH * D}, out);
    const int kv_mul = NH / NKV;
    attn_scores_all_heads(key_cache, &qt.t, &at.t, NH, kv_mul, D, NKV * D, S * D, pos);
    attn_weighted_sum_all_heads(value_cache, &at.t, &ot.t, NH, kv_mul, D, NKV * D, S * D, pos);
}

}  // extern "C"

extern "C" {

// layers/src/text_layer.cpp:52 `rms_norm`, INT8 group-quantised norm weight
// (the exporter always group-quantises norms, export_qwen_bin.py:325).
void ref_rms_norm_i8(const float *x, const int8_t *wq, const float *ws, float *out,
                     size_t hidden, size_t group_size, float eps, size_t batches) {
    QuietStdout qs;
    Wrap xt({batches, hidden}, const_cast<float *>(x));
    Wrap ot({batches, hidden}, out);
    Tensor w({hidden}, const_cast<int8_t *>(wq), const_cast<float *>(ws), group_size, true,
             DType::INT8, DType::FP32);
    rms_norm(&xt.t, &w, &ot.t, eps, batches, 0);
    w.buf = nullptr;
    w.scale_buf = nullptr;
}

// layers/src/text_layer.cpp:177 `rms_norm_inplace`, INT8 group-quantised weight.
void ref_rms_norm_inplace_i8(float *x, const int8_t *wq, const float *ws, size_t hidden,
                             size_t group_size, float eps, size_t batches) {
    QuietStdout qs;
    Wrap xt({batches, hidden}, x);
    Tensor w({hidden}, const_cast<int8_t *>(wq), const_cast<float *>(ws), group_size, true,
             DType::INT8, DType::FP32);
    rms_norm_inplace(&xt.t, &w, eps, batches, 0);
    w.buf = nullptr;
    w.scale_buf = nullptr;
}

// layers/src/text_layer.cpp:3 `embedding_lookup` for an INT8 table with
// per-row scales (group_quantized = false).
void ref_embedding_i8(const int8_t *table, const float *scales, float *out, size_t vocab,
                      size_t hidden, size_t token) {
    QuietStdout qs;
    Wrap ot({hidden}, out);
    Tensor e({vocab, hidden}, const_cast<int8_t *>(table), const_cast<float *>(scales), hidden, false,
             DType::INT8, DType::FP32);
    embedding_lookup(&e, &ot.t, token, hidden);
    e.buf = nullptr;
    e.scale_buf = nullptr;
}

}  // extern "C"
