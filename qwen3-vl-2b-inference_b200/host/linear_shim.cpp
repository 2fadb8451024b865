// Drop-in replacement for the reference's INT8 `linear()` branch
// (matmul/include/cpu_wrapper.hpp:10-16, matmul/src/cpu_wrapper.cpp:308-396)
// on top of the C ABI of libqvl_b200.so.  Same signature, same argument
// meaning, same error convention (message on stderr + exit(1) for an
// unsupported dtype combination, cpu_wrapper.cpp:394-395).
//
// Buffers are the reference's host buffers.  Weight buffers (B and its
// scales) are uploaded to the device once per host pointer and reused -- the
// reference maps its weights once at load time (model/src/load_model.cpp:
// 146-181) and never changes them; activations and results are copied on
// every call.  The workspace is allocated once and grown when needed, at the
// first call of a size, never on a repeated shape.
//
// The definition is the reference's own symbol: global `linear` with the
// reference's `struct DType { enum Type ... }` (utils/include/tensor.hpp:25-27)
// mangles to the same name, so an object linked in place of the reference's
// (or ahead of a weakened copy of it) serves every call site unchanged --
// forward_text (model/src/forward.cpp:506-654) and classifier_gemm
// (layers/src/text_layer.cpp:309-313) included.
//
// Build:
//   g++ -std=c++17 -O2 -fPIC -I include -c linear_shim.cpp
//   ... -L qwen3-vl-2b-inference_b200/lib -lqvl_b200 -lcudart
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <cuda_runtime.h>
#include "qvl_b200.h"

// The reference's DType (utils/include/tensor.hpp:25-27): same name, same
// enumerators and values, so `linear` below has the reference's mangled name.
struct DType { enum Type { FP32 = QVL_DTYPE_FP32, INT32 = QVL_DTYPE_INT32, FP16 = QVL_DTYPE_FP16,
                           INT8 = QVL_DTYPE_INT8, INT4 = QVL_DTYPE_INT4 }; };

namespace qvl_shim {

std::mutex g_mu;
struct Mirror {
    void *dev;
    size_t bytes;
};
std::unordered_map<const void *, Mirror> g_mirror;   // host weight buffer -> device copy
namespace {
void *g_ws = nullptr, *g_a = nullptr, *g_c = nullptr;
size_t g_ws_bytes = 0, g_a_bytes = 0, g_c_bytes = 0;

[[noreturn]] void die(const char *what, int rc) {
    fprintf(stderr, "%s: %s (CUDA error %d)\n", what, qvl_status_string(rc), qvl_last_cuda_error());
    exit(1);
}
void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
        exit(1);
    }
}
// Device copy of a weight buffer.  Weights are immutable for the life of the
// process in the reference (mmapped once); a host address seen again with a
// different size is a different buffer and is uploaded afresh.
void *mirror(const void *host, size_t bytes) {
    auto it = g_mirror.find(host);
    if (it != g_mirror.end()) {
        if (it->second.bytes == bytes) return it->second.dev;
        cudaFree(it->second.dev);
        g_mirror.erase(it);
    }
    void *d = nullptr;
    check(cudaMalloc(&d, bytes), "upload weights");
    check(cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice), "upload weights");
    g_mirror.emplace(host, Mirror{d, bytes});
    return d;
}
void grow(void **p, size_t *have, size_t need) {
    if (*have >= need) return;
    if (*p) cudaFree(*p);
    check(cudaMalloc(p, need), "workspace");
    *have = need;
}
}  // namespace

}  // namespace qvl_shim

void linear(const void *mat_A, const void *mat_B_in, const void *mat_B_scale, const void *mat_bias_in,
            const void *mat_bias_scale, void *mat_C, size_t M, size_t N, size_t K, bool mat_B_transpose,
            DType::Type type_a, DType::Type type_b, DType::Type type_b_scale, DType::Type type_c,
            bool group_quantized, size_t group_size) {
    using namespace qvl_shim;
    (void)mat_bias_scale;
    if (!(type_a == DType::FP32 && type_c == DType::FP32 && type_b == DType::INT8 &&
          type_b_scale == DType::FP32 && mat_bias_in == nullptr && mat_B_transpose)) {
        fprintf(stderr, "DType matmul not supported: type_a=%d, type_b=%d, type_b_scale=%d, type_c=%d, "
                        "group_quantized=%d\n", (int)type_a, (int)type_b, (int)type_b_scale, (int)type_c,
                group_quantized);
        exit(1);
    }
    std::lock_guard<std::mutex> lock(g_mu);
    const size_t g = group_quantized ? group_size : K;
    if (g == 0 || K % g) {
        fprintf(stderr, "linear: group size %zu does not divide K=%zu\n", g, K);
        exit(1);
    }
    void *dB = mirror(mat_B_in, N * K);
    void *dS = mirror(mat_B_scale, N * (K / g) * sizeof(float));
    grow(&g_a, &g_a_bytes, M * K * sizeof(float));
    grow(&g_c, &g_c_bytes, M * N * sizeof(float));
    grow(&g_ws, &g_ws_bytes, qvl_linear_i8_workspace_bytes(M, K, g));
    check(cudaMemcpy(g_a, mat_A, M * K * sizeof(float), cudaMemcpyHostToDevice), "activations");
    int rc = qvl_linear_i8((const float *)g_a, (const int8_t *)dB, (const float *)dS, (float *)g_c, M, N, K,
                           group_quantized ? 1 : 0, group_size, QVL_SEM_REFERENCE, g_ws, g_ws_bytes, nullptr);
    if (rc != QVL_OK) die("qvl_linear_i8", rc);
    check(cudaMemcpy(mat_C, g_c, M * N * sizeof(float), cudaMemcpyDeviceToHost), "result");
}

// Frees every device weight copy (call when the host weights are unmapped).
extern "C" void qvl_shim_release_weights(void) {
    std::lock_guard<std::mutex> lock(qvl_shim::g_mu);
    for (auto &kv : qvl_shim::g_mirror) cudaFree(kv.second.dev);
    qvl_shim::g_mirror.clear();
}

// C entry used by the tests (ctypes) to drive the C++ shim.
extern "C" void qvl_shim_linear_i8(const float *A, const int8_t *B, const float *Bs, float *C, size_t M,
                                   size_t N, size_t K, int group_quantized, size_t group_size) {
    linear(A, B, Bs, nullptr, nullptr, C, M, N, K, true, DType::FP32, DType::INT8, DType::FP32, DType::FP32,
           group_quantized != 0, group_size);
}
