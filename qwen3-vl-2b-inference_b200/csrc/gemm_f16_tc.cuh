#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstddef>

namespace qvl {
// Epilogues of the FP16 tensor-core GEMM (gemm_f16_tc.cu).
enum { GEMM_F16_OUT_F16 = 0, GEMM_F16_OUT_F16_GELU = 1, GEMM_F16_OUT_F32 = 2, GEMM_F16_ADD_F32 = 3 };
// C[M, N] = A[M, K] . W[N, K]^T + bias, fp16 operands, fp32 accumulation.
// N >= 128, K % 64 == 0, A and W 16-byte aligned rows.
bool gemm_f16_supported(size_t M, size_t N, size_t K);
// device address (current device) of the kernel's timeout word, or nullptr
int *gemm_f16_timeout_word();
cudaError_t launch_gemm_f16_tc(const __half *A, const __half *W, const __half *bias, void *C, int M, int N, int K,
                               int mode, cudaStream_t stream);
}  // namespace qvl
