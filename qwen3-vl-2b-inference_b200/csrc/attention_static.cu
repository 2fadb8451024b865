// Attention decode with its split-K scratch in a fixed device array, for
// callers that cannot allocate device memory at call time (see
// qvl_attention_decode_static in include/qvl_b200.h).  Same kernels and
// results as qvl_attention_decode; only where the scratch lives differs.
#include <mutex>
#include "common.cuh"
#include "attention.cuh"

namespace {

// One copy per device that loads the library.
static __device__ __align__(256) unsigned char g_attn_scratch[QVL_ATTN_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_attn_scratch on the current device.  The symbol name
// in host code only stands for the array; the address must come from the
// runtime, looked up once per device with that device current.
int scratch_for_current_device(void **out) {
    int dev = 0;
    QVL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return QVL_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        QVL_CUDA_TRY(cudaGetSymbolAddress(&p, g_attn_scratch));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return QVL_OK;
}

}  // namespace

extern "C" int qvl_attention_decode_static(const float *q, const uint16_t *k_pages,
                                           const uint16_t *v_pages, const int32_t *page_table,
                                           const int32_t *seq_ids, const int32_t *positions,
                                           size_t nq, int max_ctx, float *out,
                                           const qvl_attn_dims *dims, void *stream) {
    if (!dims || dims->head_dim != 128) return dims ? QVL_ERR_UNSUPPORTED : QVL_ERR_INVALID;
    if (dims->num_heads <= 0 || dims->num_kv_heads <= 0 || dims->num_heads % dims->num_kv_heads)
        return QVL_ERR_INVALID;
    const int kvm = dims->num_heads / dims->num_kv_heads;
    if (kvm != 1 && kvm != 2 && kvm != 4) return QVL_ERR_UNSUPPORTED;
    if (dims->page_size <= 0 || dims->max_pages_per_seq <= 0 || dims->max_pos <= 0) return QVL_ERR_INVALID;
    if (!q || !k_pages || !v_pages || !page_table || !seq_ids || !positions || !out) return QVL_ERR_INVALID;
    if (max_ctx <= 0) return QVL_ERR_INVALID;
    if (((uintptr_t)k_pages | (uintptr_t)v_pages | (uintptr_t)q) % 16) return QVL_ERR_INVALID;
    if (nq == 0) return QVL_OK;
    const qvl::AttnScratch lay = qvl::attn_scratch_layout(nq, max_ctx, dims->num_heads, dims->num_kv_heads);
    if (lay.total > (size_t)QVL_ATTN_STATIC_SCRATCH_BYTES) return QVL_ERR_WORKSPACE;
    void *scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    qvl::AttnArgs a = {};
    a.q = q; a.k_pages = k_pages; a.v_pages = v_pages; a.page_table = page_table;
    a.seq_ids = seq_ids; a.positions = positions; a.nq = nq; a.max_ctx = max_ctx; a.out = out;
    a.NH = dims->num_heads; a.NKV = dims->num_kv_heads; a.P = dims->page_size;
    a.maxp = dims->max_pages_per_seq; a.max_pos = dims->max_pos;
    QVL_CUDA_TRY(qvl::launch_attention(a, scratch, (cudaStream_t)stream));
    return QVL_OK;
}
