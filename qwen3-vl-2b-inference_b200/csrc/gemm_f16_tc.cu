// FP16 GEMM with bias on the 5th-generation tensor cores (tcgen05,
// kind::f16, fp32 accumulation in tensor memory), for the vision tower's
// linear layers (model/src/forward.cpp:97-339 and the FP16 kernels they reach
// through linear(), matmul/src/cpu_fp16_full_avx2.cpp):
//
//   C[M, N] = A[M, K] (fp16) . W[N, K]^T (fp16, the exporter's [out, in]
//             layout) + bias[N] (fp16)
//
// with one of four epilogues:
//   F16        C fp16 = round(acc + bias)
//   F16_GELU   C fp16 = round(gelu_tanh(round(acc + bias)))   (linear, then the
//              in-place gelu_tanh on the fp16 tensor, layers/src/vision_layer.cpp:869-911)
//   F32        C fp32 = acc + bias
//   ADD_F32    C fp32 += float(round(acc + bias))             (linear into an
//              fp16 tensor, then add_vector into the fp32 residual stream)
//
// Tiling as in the INT8 kernel (gemm_i8_tc.cu): 128 weight rows are the MMA's
// M dimension (TMEM lanes), NT activation rows its N dimension; one thread
// issues TMA loads of 64-element (128-byte) K slices into a ring of stages
// with 128-byte swizzle, one thread issues 4 MMAs of K = 16 per stage, four
// warps drain the accumulator.  Every wait is bounded; a timeout sets this
// kernel's timeout word and the kernel computes nothing while it is set.
#include <cuda_fp16.h>
#include "tc_common.cuh"
#include "gemm_f16_tc.cuh"

namespace qvl {

// Set when a bounded wait of this kernel gave up; while set the kernel
// computes nothing (read and cleared through qvl_tc_timeout_status).
__device__ int g_gemm_f16_timeout = 0;

namespace {
constexpr int kBM = 128;            // weight rows per CTA
constexpr int kBKe = 64;            // K elements per stage (128 bytes)
constexpr int kThreads = 128;
constexpr int kUmmaK = 16;          // K per kind::f16 MMA

template <int NT>
struct F16Smem {
    static constexpr int kA = kBM * 128;          // 16 KB of weights per stage
    static constexpr int kB = NT * 128;           // activations per stage
    static constexpr int kStage = kA + kB;
    static constexpr int kSt = 4;                 // 128 KB (NT 128) / 96 KB (NT 64: two CTAs per SM)
    static constexpr int kBytes = kSt * kStage + 1024 + 256;
};

// Instruction descriptor, kind::f16: D = F32, A = B = F16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// gelu_tanh of layers/src/vision_layer.cpp:898-905 on one value (float
// arithmetic in the reference's operation order; tanhf of the device).
__device__ __forceinline__ float gelu_tanh_one(float x) {
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}
}  // namespace

// grid (ceil(M / NT), ceil(N / 128)); block 128.
template <int NT, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                   const __half *__restrict bias, void *__restrict Cv, int M, int N, int K) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    using L = F16Smem<NT>;
    constexpr int kStages = L::kSt;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * L::kStage);
    const uint32_t full0 = tc::smem_u32(bars);
    const uint32_t empty0 = tc::smem_u32(bars + kStages);
    const uint32_t accbar = tc::smem_u32(bars + 2 * kStages);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kStages + 1);
    __shared__ int timed_out_at_entry;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.y * kBM;
    const int m0 = blockIdx.x * NT;
    const int nk = K / kBKe;
    constexpr uint32_t kCols = NT < 32 ? 32 : NT;

    if (threadIdx.x == 0) {
        timed_out_at_entry = *reinterpret_cast<volatile int *>(&g_gemm_f16_timeout) != 0;
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, 1);
        }
        tc::mbar_init(accbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tc::prefetch_tmap(&tm_w);
        tc::prefetch_tmap(&tm_a);
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
    if (timed_out_at_entry) {
        tc::tc_fence_before();
        __syncthreads();
        if (warp == 1) tc::tmem_dealloc(tmem, kCols);
        return;
    }

    bool ok = true;
    int issued = 0;
    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % kStages;
            if (kb >= kStages) ok = tc::mbar_wait(empty0 + 8 * s, ((kb / kStages) - 1) & 1, &g_gemm_f16_timeout);
            if (!ok) break;
            unsigned char *st = smem + s * L::kStage;
            tc::mbar_expect_tx(full0 + 8 * s, L::kStage);
            tc::tma_load_2d(tc::smem_u32(st), &tm_w, kb * kBKe, n0, full0 + 8 * s);
            if (kb == 0) pdl_wait();   // activations come from the previous kernel
            tc::tma_load_2d(tc::smem_u32(st + L::kA), &tm_a, kb * kBKe, m0, full0 + 8 * s);
            issued = kb + 1;
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t id = idesc_f16(kBM, NT);
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % kStages;
            ok = tc::mbar_wait(full0 + 8 * s, (kb / kStages) & 1, &g_gemm_f16_timeout);
            if (!ok) break;
            tc::tc_fence_after();
            const uint32_t a_base = tc::smem_u32(smem + s * L::kStage);
            const uint32_t b_base = a_base + L::kA;
#pragma unroll
            for (int k = 0; k < kBKe / kUmmaK; ++k)
                mma_f16(tmem, tc::sdesc_k_sw128(a_base + k * 32), tc::sdesc_k_sw128(b_base + k * 32), id,
                        (kb > 0 || k > 0) ? 1u : 0u);
            tc::tc_commit(empty0 + 8 * s);
        }
        tc::tc_commit(accbar);
    }
    __syncwarp();

    pdl_wait();
    const bool acc_ok = tc::mbar_wait(accbar, 0, &g_gemm_f16_timeout);
    tc::tc_fence_after();
    if (acc_ok) {
        const int n = n0 + warp * 32 + lane;
        const float b = (n < N && bias) ? __half2float(bias[n]) : 0.0f;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
        for (int c0 = 0; c0 < NT; c0 += 16) {
            uint32_t r[16];
            tc::tmem_ld16(tmem + lane_off + c0, r);
            tc::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = m0 + c0 + j;
                if (m < M && n < N) {
                    const float v = __fadd_rn(__uint_as_float(r[j]), b);
                    const size_t o = (size_t)m * N + n;
                    if constexpr (MODE == GEMM_F16_OUT_F16) {
                        reinterpret_cast<__half *>(Cv)[o] = __float2half_rn(v);
                    } else if constexpr (MODE == GEMM_F16_OUT_F16_GELU) {
                        const float h = __half2float(__float2half_rn(v));
                        reinterpret_cast<__half *>(Cv)[o] = __float2half_rn(gelu_tanh_one(h));
                    } else if constexpr (MODE == GEMM_F16_OUT_F32) {
                        reinterpret_cast<float *>(Cv)[o] = v;
                    } else {
                        float *cp = reinterpret_cast<float *>(Cv) + o;
                        *cp = __fadd_rn(*cp, __half2float(__float2half_rn(v)));
                    }
                }
            }
        }
    }
    if (warp == 0 && lane == 0 && !ok) {
        for (int kb = issued - 1; kb >= 0 && kb >= issued - kStages; --kb)
            tc::mbar_wait(full0 + 8 * (kb % kStages), (kb / kStages) & 1, nullptr);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, kCols);
}

// ---------------------------------------------------------------- host side
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

// fp16 [rows, cols] (cols contiguous), box {64 elements, box_rows}, 128-byte swizzle.
bool map_f16(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBKe, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int MODE>
cudaError_t launch_mode(const CUtensorMap &mw, const CUtensorMap &ma, const __half *bias, void *C, int M, int N,
                        int K, cudaStream_t st) {
    auto kern = gemm_f16_tc_kernel<NT, MODE>;
    const int smem = F16Smem<NT>::kBytes;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + NT - 1) / NT, (N + kBM - 1) / kBM);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, mw, ma, bias, C, M, N, K);
}

template <int NT>
cudaError_t launch_nt(const CUtensorMap &mw, const CUtensorMap &ma, const __half *bias, void *C, int M, int N,
                      int K, int mode, cudaStream_t st) {
    switch (mode) {
    case GEMM_F16_OUT_F16: return launch_mode<NT, GEMM_F16_OUT_F16>(mw, ma, bias, C, M, N, K, st);
    case GEMM_F16_OUT_F16_GELU: return launch_mode<NT, GEMM_F16_OUT_F16_GELU>(mw, ma, bias, C, M, N, K, st);
    case GEMM_F16_OUT_F32: return launch_mode<NT, GEMM_F16_OUT_F32>(mw, ma, bias, C, M, N, K, st);
    default: return launch_mode<NT, GEMM_F16_ADD_F32>(mw, ma, bias, C, M, N, K, st);
    }
}
}  // namespace

int *gemm_f16_timeout_word() {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_f16_timeout) != cudaSuccess) return nullptr;
    return static_cast<int *>(p);
}

bool gemm_f16_supported(size_t M, size_t N, size_t K) {
    return M >= 1 && N >= (size_t)kBM && K % kBKe == 0 && K > 0 && (N + kBM - 1) / kBM <= 65535 &&
           encode_fn() != nullptr;
}

cudaError_t launch_gemm_f16_tc(const __half *A, const __half *W, const __half *bias, void *C, int M, int N, int K,
                               int mode, cudaStream_t stream) {
    // 128-row activation tiles only when they alone fill the GPU; otherwise
    // 64-row tiles (twice the CTAs, two per SM)
    const long tiles128 = (long)((M + 127) / 128) * ((N + kBM - 1) / kBM);
    const int NT = (M >= 512 && tiles128 >= 2 * 148) ? 128 : 64;
    CUtensorMap mw, ma;
    if (!map_f16(&mw, W, N, K, kBM) || !map_f16(&ma, A, M, K, NT)) return cudaErrorInvalidValue;
    if (NT == 128) return launch_nt<128>(mw, ma, bias, C, M, N, K, mode, stream);
    return launch_nt<64>(mw, ma, bias, C, M, N, K, mode, stream);
}

}  // namespace qvl
