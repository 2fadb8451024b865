// Greedy decode on device, tokenizer/src/utils.cpp:34-44: the first index of
// the maximum (strict >, starting from -FLT_MAX, so NaN and -FLT_MAX never
// win and an all-losing row yields 0).
//
// One thread-block cluster of kClusterCtas CTAs per row: each CTA scans a
// contiguous slice of the row, the CTAs' (value, index) winners meet in CTA 0
// through distributed shared memory, and CTA 0 writes 4 bytes.  No global
// scratch and no second launch.
#include <cfloat>
#include <climits>
#include <cooperative_groups.h>
#include "common.cuh"
#include "argmax.cuh"

namespace cg = cooperative_groups;

namespace qvl {

constexpr int kClusterCtas = 8;

__device__ __forceinline__ void better(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

// Block-wide (value, index) reduction; result valid in thread 0.
__device__ __forceinline__ void block_best(float &v, int &bi) {
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        better(v, bi, v2, i2);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv[w] = v; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        v = (threadIdx.x < nw) ? sv[threadIdx.x] : -FLT_MAX;
        bi = (threadIdx.x < nw) ? si[threadIdx.x] : INT_MAX;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            better(v, bi, v2, i2);
        }
    }
}

// grid: (kClusterCtas, rows), cluster (kClusterCtas, 1, 1); block 1024.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float *__restrict logits,
                                                           int32_t *__restrict idx, long n) {
    __shared__ float best_v;
    __shared__ int best_i;
    cg::cluster_group cluster = cg::this_cluster();
    pdl_launch_dependents();
    pdl_wait();
    const unsigned rank = cluster.block_rank();
    const float *row = logits + (long)blockIdx.y * n;
    const long per = (n + kClusterCtas - 1) / kClusterCtas;
    const long j0 = rank * per, j1 = min(n, j0 + per);
    float v = -FLT_MAX;
    int bi = INT_MAX;
    for (long j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
        const float x = row[j];
        if (x > v) { v = x; bi = (int)j; }   // ascending j: strict > keeps the first
    }
    block_best(v, bi);
    if (threadIdx.x == 0) { best_v = v; best_i = bi; }
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        float fv = -FLT_MAX;
        int fi = INT_MAX;
        for (int r = 0; r < kClusterCtas; ++r) {
            const float rv = *cluster.map_shared_rank(&best_v, r);
            const int ri = *cluster.map_shared_rank(&best_i, r);
            better(fv, fi, rv, ri);
        }
        idx[blockIdx.y] = (fi == INT_MAX) ? 0 : fi;
    }
    cluster.sync();   // keep every CTA's shared memory alive until CTA 0 has read it
}

cudaError_t launch_argmax_rows(const float *logits, int32_t *idx, long rows, long n,
                               cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kClusterCtas, (unsigned)rows);
    cfg.blockDim = dim3(1024);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kClusterCtas;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, argmax_rows_kernel, logits, idx, n);
}

}  // namespace qvl
