#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace qvl {
// Tensor-core (tcgen05 kind::i8) INT8 GEMM with TILED summation semantics.
// TILED summation, K % 128 == 0, M >= 16; per-output-row weight scales
// (g == K) or group-wise ones with g in {32, 64} or a multiple of 128.
bool gemm_tc_supported(size_t M, size_t N, size_t K, size_t g);
// group sizes (g < K) the group-wise tensor-core kernel takes
bool gemm_tc_grouped_size(size_t g, size_t K);
// device address (current device) of the kernel's timeout word, or nullptr
int *gemm_tc_timeout_word();
// bytes of the hi/lo activation planes the GEMM needs in the caller's workspace
size_t gemm_tc_planes_bytes(size_t M, size_t K);
cudaError_t launch_gemm_i8_tc(const int16_t *q, const float *qs, int8_t *hi, uint8_t *lo, const int8_t *W,
                              const float *ws, float *C, int M, int N, int K, cudaStream_t stream);
// hi/lo planes from int16 activations, and the GEMM on planes already split
// (so several products of the same activations split once).  acc: C += result.
cudaError_t launch_split_hi_lo(const int16_t *q, int8_t *hi, uint8_t *lo, int M, int K, cudaStream_t stream);
cudaError_t launch_gemm_i8_tc_planes(const int8_t *hi, const uint8_t *lo, const float *qs, const int8_t *W,
                                     const float *ws, float *C, int M, int N, int K, int acc,
                                     cudaStream_t stream, int g = 0);   // g: group size, 0 = K
// One launch over up to three weight matrices [N_i, K] of the same hi/lo
// activation planes (per-output-row scales): C_i = product_i (C_i += with acc).
cudaError_t launch_gemm_i8_tc_planes_multi(const int8_t *hi, const uint8_t *lo, const float *qs, int n_mats,
                                           const int8_t *const *W, const float *const *ws, float *const *C,
                                           const int *N, int M, int K, int acc, cudaStream_t stream);
}  // namespace qvl
