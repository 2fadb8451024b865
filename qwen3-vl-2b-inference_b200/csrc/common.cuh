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

// expf as the reference's host C library computes it, bit for bit.  The
// reference's swiglu (layers/src/text_layer.cpp:430) calls the scalar expf of
// glibc (2.28 and later), whose method is the table-driven exp of ARM's
// optimized-routines (Szabolcs Nagy, 2017; MIT licence): in double precision,
// k = round(x * 32/ln2), r = x * 32/ln2 - k, 2^(r/32) by a degree-3
// polynomial times the table value 2^((k mod 32)/32) with k/32 added to its
// exponent, one rounding to float at the end.  On x86-64 glibc selects the
// build compiled with FMA contraction, so every multiply-add here is fused the
// same way.  The table is 2^(i/32) rounded to double; the polynomial
// coefficients are the published ones.  Checked on the GPU against the host's
// expf over every float (tests/test_gpu_parity.py).  Overflow (x > 88.72...)
// gives +inf, underflow (x < -103.97...) +0, NaN stays NaN.
// 2^(i/32), i = 0..31, rounded to double
static __constant__ double kExpTab[32] = {
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0,
};

__device__ __forceinline__ float expf_host(float x) {
    constexpr double kInvLn2N = 0x1.71547652b82fep0 * 32.0;
    constexpr double kShift = 0x1.8p+52;
    constexpr double kC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    if (!(x <= 0x1.62e42ep6f)) return x != x ? x : __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p6f) return 0.0f;
    const double xd = (double)x;
    double kd = __fma_rn(kInvLn2N, xd, kShift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, kShift);
    const double r = __fma_rn(kInvLn2N, xd, -kd);
    const unsigned long long t =
        (unsigned long long)__double_as_longlong(kExpTab[ki & 31]) - ((ki & 31) << 47) + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double z = __fma_rn(kC0, r, kC1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(kC2, r, 1.0);
    y = __fma_rn(z, r2, y);
    return __double2float_rn(__dmul_rn(y, s));
}

// SwiGLU of one element, layers/src/text_layer.cpp:430-432:
// (x / (1 + expf(-x))) * u with the host library's expf (expf_host).
__device__ __forceinline__ float swiglu_one(float x, float u) {
    const float e = expf_host(-x);
    const float silu = __fdiv_rn(x, add_rn(1.0f, e));
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
