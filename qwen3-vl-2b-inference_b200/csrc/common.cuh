// Shared device helpers for the sm_100a INT8 hot path.
//
// Exactness notes.  Every floating-point step that has to reproduce the
// reference CPU engine bit for bit is written with an explicit
// round-to-nearest intrinsic (__fmaf_rn, __fmul_rn, __fadd_rn, __fdiv_rn,
// __fsqrt_rn, __int2float_rn, __float2int_rn) so the compiler can neither fuse
// nor reassociate it.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "../../include/qvl_b200.h"

namespace qvl {

constexpr int kWarp = 32;

__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// Horizontal sum of 8 fp32 lanes in the order of the reference's
// add_reduce_mm_256 (matmul/include/simd_utils.hpp:5-19):
// u_i = v_i + v_{i+4}, then (u0 + u1) + (u2 + u3).
__device__ __forceinline__ float reduce8_ref(const float v[8]) {
    float u0 = add_rn(v[0], v[4]), u1 = add_rn(v[1], v[5]);
    float u2 = add_rn(v[2], v[6]), u3 = add_rn(v[3], v[7]);
    return add_rn(add_rn(u0, u1), add_rn(u2, u3));
}

// One lane of the reference's exp256_ps (layers/include/simd_utils.hpp:7-47):
// clamp to +-88.3762626647949, n = floor(x*log2e), g = x - n*ln2 (fused),
// 4th-order Taylor polynomial with fused adds, times 2^n built from the
// exponent bits.  Restated from the algorithm; constants are the reference's.
__device__ __forceinline__ float exp_ref(float x) {
    const float max_x = 88.3762626647949f;
    x = fminf(x, max_x);
    x = fmaxf(x, -max_x);
    const float ln2 = 0.69314718056f, inv_ln2 = 1.44269504089f;
    float fx = floorf(mul_rn(x, inv_ln2));
    int e = (int)fx;
    float g = fma_rn(-fx, ln2, x);
    float y = fma_rn(g, 1.0f, 1.0f);
    float g2 = mul_rn(g, g);
    y = fma_rn(g2, 0.5f, y);
    float g3 = mul_rn(g2, g);
    y = fma_rn(g3, 1.0f / 6.0f, y);
    float g4 = mul_rn(g3, g);
    y = fma_rn(g4, 1.0f / 24.0f, y);
    float p = __int_as_float((int)((unsigned)(e + 127) << 23));
    return mul_rn(y, p);
}

// SwiGLU of one element, layers/src/text_layer.cpp:430-432:
// (x / (1 + expf(-x))) * u.  exp is evaluated in double precision and rounded
// once to fp32 -- the correctly rounded expf value (glibc's expf, used by the
// reference, is correctly rounded for all but a vanishing set of inputs).
__device__ __forceinline__ float swiglu_one(float x, float u) {
    float e = (float)exp(-(double)x);
    float silu = __fdiv_rn(x, add_rn(1.0f, e));
    return mul_rn(silu, u);
}

// 128-bit streaming load that bypasses L1 (weights are read exactly once).
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (weight prefetch) while this one finishes, and wait for the
// previous kernel's results before touching them.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Integer dot of an int16 pair with two int8 bytes: the _mm256_madd_epi16
// lane (a.lo*b0 + a.hi*b1 + c), via dp2a.
__device__ __forceinline__ int dp2a_lo(int a16x2, int b8x4, int c) { return __dp2a_lo(a16x2, b8x4, c); }
__device__ __forceinline__ int dp2a_hi(int a16x2, int b8x4, int c) { return __dp2a_hi(a16x2, b8x4, c); }

}  // namespace qvl

#define QVL_CUDA_TRY(expr)                                  \
    do {                                                    \
        cudaError_t _e = (expr);                            \
        if (_e != cudaSuccess) {                            \
            qvl_internal_set_cuda_error((int)_e);           \
            return QVL_ERR_CUDA;                            \
        }                                                   \
    } while (0)

extern "C" void qvl_internal_set_cuda_error(int err);
