// enx_attn_decode_noalloc: decode attention that needs no caller workspace and allocates nothing.
//
// enx_attn_decode keeps its attention scores in a workspace the caller allocates.
// Some callers cannot allocate device memory at the point where they run attention: code that
// runs inside a host callback or a real-time loop where cudaMalloc's implicit synchronisation is
// not allowed, plugin hosts that hand over only fixed input/output buffers, and embedders with
// their own memory manager that forbids outside allocations.  This variant keeps the scores
// in one file-scope device array instead, sized for the limits below.  Every GPU that loads the
// library holds that array (kScratchFloats * 4 bytes, 512 KB) until the process exits.

#include <mutex>
#include <string>
#include <vector>

#include "enx_internal.cuh"
#include "k_decode.cuh"

namespace enx {

// Capacity: attention scores of up to 32 query heads x 4096 positions.
constexpr uint32_t kNoAllocMaxPositions = 4096;
constexpr size_t kScratchFloats = (size_t)kNoAllocMaxPositions * 32;

static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

// Device address of g_attn_scratch, looked up once per device (with that device current).
static std::mutex g_scratch_mu;
static std::vector<float*> g_scratch_ptr;

static enx_status scratch_for_current_device(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if ((size_t)dev >= g_scratch_ptr.size()) g_scratch_ptr.resize((size_t)dev + 1, nullptr);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_attn_scratch)");
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return ENX_OK;
}

}  // namespace enx

using namespace enx;

extern "C" enx_status enx_attn_decode_noalloc(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                              float* out, const enx_attn_decode_dims* d, void* stream) {
    if (!d || !q || !k_cache || !v_cache || !out) return fail(ENX_ERR_INVALID, "enx_attn_decode_noalloc: null pointer");
    if (d->kv_heads == 0 || d->heads % d->kv_heads != 0 || d->heads / d->kv_heads > 8)
        return fail(ENX_ERR_INVALID, "enx_attn_decode_noalloc: heads must be a multiple of kv_heads, at most 8 per kv head");
    if (d->head_dim == 0 || d->head_dim % 2 != 0 || d->head_dim > 64)
        return fail(ENX_ERR_INVALID, "enx_attn_decode_noalloc: head_dim must be even and <= 64");
    if (d->cache_stride != d->kv_heads * d->head_dim)
        return fail(ENX_ERR_INVALID, "enx_attn_decode_noalloc: cache_stride must be kv_heads*head_dim");
    const uint32_t splits = (d->position + 1 + kAttnChunk - 1) / kAttnChunk;
    const size_t need = (size_t)splits * kAttnChunk * d->heads;
    if (d->position >= kNoAllocMaxPositions || d->heads > 32 || need > kScratchFloats)
        return fail(ENX_ERR_RANGE, "enx_attn_decode_noalloc: position " + std::to_string(d->position) + " / heads " +
                                       std::to_string(d->heads) +
                                       " exceed the built-in scratch (position < 4096, heads <= 32, head_dim <= 64); "
                                       "use enx_attn_decode with a workspace");
    float* scratch = nullptr;
    ENX_TRY(scratch_for_current_device(&scratch));
    // Every score the softmax reads is written first by the score kernel of the same call, so the
    // shared array needs no clearing between calls.
    StepArgs S{};
    S.hidden = d->heads * d->head_dim;
    S.heads = d->heads;
    S.kv_heads = d->kv_heads;
    S.head_dim = d->head_dim;
    S.q = const_cast<float*>(q);
    S.scores = scratch;
    S.score_stride = splits * kAttnChunk;
    S.pos = nullptr;
    S.pos_base = d->position;
    S.seq_fixed = 0;
    S.kcache = const_cast<uint16_t*>(k_cache);
    S.vcache = const_cast<uint16_t*>(v_cache);
    S.layers = 1;
    S.max_context = d->position + 1;
    cudaStream_t st = as_stream(stream);
    ENX_CUDA(launch_attn(S, 0, 1, out, st, false));
    return ENX_OK;
}
