// libenx C ABI: raw kernel entry points, the .enargeia loader, and the model context
// (weights + f16 KV caches + the captured decode step).  Declarations and the reference
// interfaces each function replaces are in include/enx.h.

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <mutex>
#include <vector>

#include "enx_internal.cuh"
#include "k_decode.cuh"
#include "k_gemm_tc.cuh"
#include "k_mega.cuh"
#include "k_small.cuh"
#include "json_lite.h"

// ---------------------------------------------------------------------------------------------
// error state

namespace enx {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

enx_status fail(enx_status code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

enx_status cuda_fail(cudaError_t err, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
    return ENX_ERR_CUDA;
}

}  // namespace enx

using namespace enx;

extern "C" const char* enx_last_error(void) { return g_last_error.c_str(); }
extern "C" const char* enx_version(void) { return "enx 0.1 sm_100a"; }

#define CHECK_ARG(cond, msg) \
    do {                     \
        if (!(cond)) return fail(ENX_ERR_INVALID, msg); \
    } while (0)

// ---------------------------------------------------------------------------------------------
// raw kernels

// Tensor-core GEMMs (M >= kTcMinTokens) need a workspace for the activation limbs.  The raw entry
// points keep one per device, grown on demand (a call that grows it synchronises the device through
// cudaMalloc), with a device error word that a bounded wait raises.
constexpr uint32_t kTcMinTokens = 16;
static std::mutex g_tc_mu;
struct TcWorkspace {
    uint8_t* ptr = nullptr;
    size_t bytes = 0;
    uint32_t* err = nullptr;
};
static std::vector<TcWorkspace> g_tc_ws;

static enx_status tc_workspace(size_t bytes, uint8_t** ws, uint32_t** err) {
    int dev = 0;
    ENX_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_tc_mu);
    if ((size_t)dev >= g_tc_ws.size()) g_tc_ws.resize((size_t)dev + 1);
    TcWorkspace& W = g_tc_ws[dev];
    if (!W.err) {
        ENX_CUDA(cudaMalloc(&W.err, sizeof(uint32_t)));
        ENX_CUDA(cudaMemset(W.err, 0, sizeof(uint32_t)));
    }
    if (W.bytes < bytes) {
        if (W.ptr) cudaFree(W.ptr);
        W.ptr = nullptr;
        W.bytes = 0;
        ENX_CUDA(cudaMalloc(&W.ptr, bytes));
        W.bytes = bytes;
    }
    *ws = W.ptr;
    *err = W.err;
    return ENX_OK;
}

extern "C" enx_status enx_raw_check(void) {
    int dev = 0;
    ENX_CUDA(cudaGetDevice(&dev));
    ENX_CUDA(cudaDeviceSynchronize());
    uint32_t* err = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_tc_mu);
        if ((size_t)dev < g_tc_ws.size()) err = g_tc_ws[dev].err;
    }
    if (!err) return ENX_OK;
    uint32_t code = 0;
    ENX_CUDA(cudaMemcpy(&code, err, 4, cudaMemcpyDeviceToHost));
    if (!code) return ENX_OK;
    ENX_CUDA(cudaMemset(err, 0, 4));
    return fail(ENX_ERR_TIMEOUT, "raw tensor-core GEMM: a bounded device wait gave up (code " +
                                     std::to_string(code) + ")");
}

extern "C" enx_status enx_set_wait_limit(int device, uint32_t spins) {
    int n = 0;
    ENX_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(ENX_ERR_INVALID, "enx_set_wait_limit: no such device");
    int prev = 0;
    ENX_CUDA(cudaGetDevice(&prev));
    ENX_CUDA(cudaSetDevice(device));
    cudaError_t e = mega_set_spin(spins);
    if (e == cudaSuccess) e = tc_set_spin(spins);
    cudaSetDevice(prev);
    ENX_CUDA(e);
    return ENX_OK;
}

extern "C" enx_status enx_matmul_q4(const float* x, const uint32_t* packed, const float* scales,
                                    const uint32_t* zeros, const float* bias, float* out,
                                    const enx_matmul_q4_dims* d, void* stream) {
    CHECK_ARG(d && x && packed && scales && zeros && out, "enx_matmul_q4: null pointer");
    CHECK_ARG(d->block_size == 64, "enx_matmul_q4: block_size must be 64");
    CHECK_ARG(d->k % 64 == 0 && d->k > 0, "enx_matmul_q4: k must be a positive multiple of 64");
    CHECK_ARG(d->blocks_per_row == d->k / 64, "enx_matmul_q4: blocks_per_row != k/64");
    CHECK_ARG(!d->use_bias || bias, "enx_matmul_q4: use_bias set without a bias");
    if (d->m == 0 || d->n == 0) return ENX_OK;
    QW w{packed, scales, zeros, d->n, d->k};
    if (d->m >= kTcMinTokens) {  // tensor cores (exact limb GEMM), library-owned workspace
        uint8_t* ws = nullptr;
        uint32_t* err = nullptr;
        ENX_TRY(tc_workspace(gemm_tc_workspace_bytes(d->m, d->k) + gemm_tc_codes_bytes(d->n, d->k), &ws, &err));
        ENX_CUDA(launch_gemm_tc(4, x, d->k, w, nullptr, d->use_bias ? bias : nullptr, out, d->m, d->out_stride,
                                d->out_offset, ws, err, as_stream(stream)));
        return ENX_OK;
    }
    ENX_CUDA(launch_matmul(4, x, w, d->use_bias ? bias : nullptr, out, d->m, d->out_stride, d->out_offset,
                           as_stream(stream), false));
    return ENX_OK;
}

extern "C" enx_status enx_lm_head_q8(const float* x, const uint32_t* packed, const float* scales,
                                     const uint32_t* zeros, float* out, const enx_embedding_dims* d,
                                     void* stream) {
    CHECK_ARG(d && x && packed && scales && zeros && out, "enx_lm_head_q8: null pointer");
    CHECK_ARG(d->block_size == 64 && d->hidden % 64 == 0 && d->blocks_per_row == d->hidden / 64,
              "enx_lm_head_q8: hidden must be a multiple of 64 with block_size 64");
    if (d->row_count == 0 || d->seq == 0) return ENX_OK;
    const uint32_t stride = d->out_stride ? d->out_stride : d->row_count;
    CHECK_ARG(d->seq == 1 || stride >= d->row_count, "enx_lm_head_q8: out_stride below row_count");
    QW w{packed, scales, zeros, d->row_count, d->hidden};
    if (d->seq >= kTcMinTokens) {
        uint8_t* ws = nullptr;
        uint32_t* err = nullptr;
        ENX_TRY(tc_workspace(gemm_tc_workspace_bytes(d->seq, d->hidden), &ws, &err));
        ENX_CUDA(launch_gemm_tc(8, x, d->hidden, w, nullptr, nullptr, out, d->seq, stride, d->out_offset, ws, err,
                                as_stream(stream)));
        return ENX_OK;
    }
    if (d->seq <= 4 && d->hidden <= 1024 && d->hidden % 128 == 0) {  // decode rows: tensor-core head
        uint8_t* ws = nullptr;
        uint32_t* err = nullptr;
        ENX_TRY(tc_workspace(0, &ws, &err));
        HeadTcArgs h{};
        h.x = x;
        h.w = w;
        h.out = out + d->out_offset;
        h.out_stride = stride;
        h.ntok = d->seq;
        h.err = err;
        ENX_CUDA(launch_head_tc(h, as_stream(stream), false));
        return ENX_OK;
    }
    ENX_CUDA(launch_matmul(8, x, w, nullptr, out, d->seq, stride, d->out_offset, as_stream(stream), false));
    return ENX_OK;
}

extern "C" enx_status enx_embed_gather_q8(const uint32_t* ids, const uint32_t* packed,
                                          const float* scales, const uint32_t* zeros, float* out,
                                          const enx_embedding_dims* d, void* stream) {
    CHECK_ARG(d && ids && packed && scales && zeros && out, "enx_embed_gather_q8: null pointer");
    CHECK_ARG(d->block_size == 64 && d->hidden % 64 == 0, "enx_embed_gather_q8: bad hidden/block");
    if (d->seq == 0) return ENX_OK;
    QW w{packed, scales, zeros, d->row_count, d->hidden};
    ENX_CUDA(launch_embed(ids, w, 8, out, d->seq, d->row_begin, d->row_count, d->hidden, as_stream(stream), false));
    return ENX_OK;
}

extern "C" enx_status enx_sample(float* logits, const uint32_t* history, uint32_t* out,
                                 const enx_sample_dims* d, void* workspace, void* stream) {
    (void)workspace;
    CHECK_ARG(d && logits && out, "enx_sample: null pointer");
    CHECK_ARG(d->history_length == 0 || history, "enx_sample: history_length > 0 without history");
    CHECK_ARG(d->vocab > 0, "enx_sample: empty vocabulary");
    if (d->vocab > sample_max_vocab())
        return fail(ENX_ERR_RANGE, "enx_sample: vocabulary of " + std::to_string(d->vocab) +
                                       " exceeds the on-chip limit of " + std::to_string(sample_max_vocab()));
    SampleRow r{d->temperature, d->top_p, d->repetition_penalty, d->random};
    ENX_CUDA(launch_sample(logits, d->vocab, 1, history, d->history_length, nullptr, nullptr, false, r, out,
                           as_stream(stream), false));
    return ENX_OK;
}

extern "C" enx_status enx_sample_batched(float* logits, uint32_t vocab, uint32_t batch,
                                         const uint32_t* history, uint32_t history_stride,
                                         const uint32_t* history_length,
                                         const enx_sampling_row* rows, uint32_t* out, void* stream) {
    CHECK_ARG(logits && rows && out, "enx_sample_batched: null pointer");
    CHECK_ARG(vocab > 0, "enx_sample_batched: empty vocabulary");
    if (vocab > sample_max_vocab()) return fail(ENX_ERR_RANGE, "enx_sample_batched: vocabulary too large");
    if (batch == 0) return ENX_OK;
    static_assert(sizeof(enx_sampling_row) == sizeof(SampleRow), "row layout");
    ENX_CUDA(launch_sample(logits, vocab, batch, history, history_stride, history_length,
                           reinterpret_cast<const SampleRow*>(rows), false, SampleRow{}, out, as_stream(stream),
                           false));
    return ENX_OK;
}

static uint32_t splits_for(uint32_t positions) { return (positions + kAttnChunk - 1) / kAttnChunk; }
// Score row stride of the many-token attention path: a multiple of kAttnSplit.
static uint32_t split_stride(uint32_t positions) { return (positions + kAttnSplit - 1) / kAttnSplit * kAttnSplit; }

extern "C" size_t enx_attn_decode_workspace_bytes(uint32_t max_context, uint32_t heads, uint32_t head_dim) {
    return (size_t)splits_for(max_context) * kAttnChunk * heads * sizeof(float);
}

extern "C" size_t enx_attn_prefill_workspace_bytes(uint32_t queries, uint32_t keys, uint32_t heads,
                                                   uint32_t head_dim) {
    return (size_t)queries * splits_for(keys) * kAttnChunk * heads * sizeof(float);
}

static enx_status attn_common(const float* q, const uint16_t* kc, const uint16_t* vc, float* out,
                              uint32_t ntok, uint32_t begin, uint32_t heads, uint32_t kv_heads,
                              uint32_t hd, void* ws, cudaStream_t st, const char* who) {
    std::string w = who;
    CHECK_ARG(q && kc && vc && out && ws, (w + ": null pointer").c_str());
    CHECK_ARG(kv_heads > 0 && heads % kv_heads == 0, (w + ": heads must be a multiple of kv_heads").c_str());
    CHECK_ARG(hd % 2 == 0 && hd <= 64 && hd > 0, (w + ": head_dim must be even and <= 64").c_str());
    CHECK_ARG(heads / kv_heads <= 8, (w + ": at most 8 query heads per kv head").c_str());
    if (ntok == 0) return ENX_OK;
    StepArgs S{};
    S.hidden = heads * hd;
    S.heads = heads;
    S.kv_heads = kv_heads;
    S.head_dim = hd;
    S.q = const_cast<float*>(q);
    S.scores = static_cast<float*>(ws);
    S.score_stride = splits_for(begin + ntok) * kAttnChunk;
    S.pos = nullptr;
    S.pos_base = begin;
    S.seq_fixed = 0;
    S.kcache = const_cast<uint16_t*>(kc);
    S.vcache = const_cast<uint16_t*>(vc);
    S.layers = 1;
    S.max_context = begin + ntok;
    ENX_CUDA(launch_attn(S, 0, ntok, out, st, false));
    return ENX_OK;
}

extern "C" enx_status enx_attn_decode(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                      float* out, const enx_attn_decode_dims* d, void* workspace,
                                      void* stream) {
    CHECK_ARG(d, "enx_attn_decode: null dims");
    CHECK_ARG(d->cache_stride == d->kv_heads * d->head_dim, "enx_attn_decode: cache_stride must be kv_heads*head_dim");
    return attn_common(q, k_cache, v_cache, out, 1, d->position, d->heads, d->kv_heads, d->head_dim, workspace,
                       as_stream(stream), "enx_attn_decode");
}

extern "C" enx_status enx_attn_prefill(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                       float* out, uint32_t queries, uint32_t begin, uint32_t heads,
                                       uint32_t kv_heads, uint32_t head_dim, void* workspace,
                                       void* stream) {
    return attn_common(q, k_cache, v_cache, out, queries, begin, heads, kv_heads, head_dim, workspace,
                       as_stream(stream), "enx_attn_prefill");
}

extern "C" enx_status enx_rmsnorm(const float* x, const float* w, float* out, uint32_t seq,
                                  uint32_t features, float eps, void* stream) {
    CHECK_ARG(x && w && out, "enx_rmsnorm: null pointer");
    ENX_CUDA(launch_rmsnorm(x, w, out, seq, features, eps, as_stream(stream)));
    return ENX_OK;
}

extern "C" enx_status enx_rope(const float* x, float* out, const float* ct, const float* sn, uint32_t seq,
                               uint32_t heads, uint32_t hd, uint32_t pos0, uint32_t out_offset, void* stream) {
    CHECK_ARG(x && out && ct && sn, "enx_rope: null pointer");
    CHECK_ARG(hd % 2 == 0, "enx_rope: head_dim must be even");
    ENX_CUDA(launch_rope(x, out, ct, sn, seq, heads, hd, pos0, out_offset, as_stream(stream)));
    return ENX_OK;
}

extern "C" enx_status enx_cache_pack(const float* src, uint16_t* dst, uint32_t count, uint32_t dst_offset,
                                     void* stream) {
    CHECK_ARG(src && dst, "enx_cache_pack: null pointer");
    ENX_CUDA(launch_cache_pack(src, dst, count, dst_offset, as_stream(stream)));
    return ENX_OK;
}

extern "C" enx_status enx_silu_mul(const float* g, const float* u, float* out, uint32_t n, void* stream) {
    CHECK_ARG(g && u && out, "enx_silu_mul: null pointer");
    ENX_CUDA(launch_silu_mul(g, u, out, n, as_stream(stream)));
    return ENX_OK;
}

extern "C" enx_status enx_add(const float* a, const float* b, float* out, uint32_t n, void* stream) {
    CHECK_ARG(a && b && out, "enx_add: null pointer");
    ENX_CUDA(launch_add(a, b, out, n, as_stream(stream)));
    return ENX_OK;
}

// ---------------------------------------------------------------------------------------------
// model context

namespace {

constexpr uint32_t kMaxStepBatch = 4;

struct Tensor {
    int bits = 0;  // 4, 8, or 32 (F32 data in `packed`)
    uint32_t rows = 0, cols = 0;
    void* packed = nullptr;
    float* scales = nullptr;
    uint32_t* zeros = nullptr;
    size_t bytes = 0;
};

// Per-step inputs/outputs, one pinned host copy and one device copy; the captured step copies
// the input half host->device at its start and the ids device->host at its end.
struct StepBlock {
    uint32_t tokens[kMaxStepBatch];
    uint32_t pos[kMaxStepBatch];
    uint32_t hist_len[kMaxStepBatch];
    uint32_t pad;
    SampleRow rows[kMaxStepBatch];
    uint32_t out[kMaxStepBatch];
    uint32_t err;  // sticky device error of the persistent kernel (read back with `out`)
};

// Before each launch of the persistent step kernel (see k_mega.cu, tagged activations): its tag
// epoch (low half of word 0) one more.
__device__ __forceinline__ void mega_prep_counters(unsigned long long* bar) {
    if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(bar) += 1;
}

__global__ void k_bump_epoch(unsigned long long* bar) { mega_prep_counters(bar); }

__global__ void k_step_prep(StepBlock* blk, uint32_t* history, uint32_t max_ctx, uint32_t batch, unsigned long long* bar) {
    uint32_t b = threadIdx.x;
    if (b < batch) history[(size_t)b * max_ctx + blk->pos[b]] = blk->tokens[b];
    mega_prep_counters(bar);
}

// State of a device-fed decode loop: step counter, start positions, first tokens, params.
struct LoopState {
    uint32_t i;
    uint32_t base_pos[kMaxStepBatch];
    uint32_t first[kMaxStepBatch];
    SampleRow params[kMaxStepBatch];  // random field unused: per-step draws come from `randoms`
};

__global__ void k_loop_prep(LoopState* L, StepBlock* blk, const float* randoms, const uint32_t* ids,
                            uint32_t* history, uint32_t max_ctx, uint32_t batch, unsigned long long* bar) {
    uint32_t b = threadIdx.x;
    mega_prep_counters(bar);
    if (b >= batch) return;
    uint32_t i = L->i;
    uint32_t tok = i == 0 ? L->first[b] : ids[(size_t)(i - 1) * batch + b];
    uint32_t pos = L->base_pos[b] + i;
    blk->tokens[b] = tok;
    blk->pos[b] = pos;
    blk->hist_len[b] = pos + 1;
    SampleRow r = L->params[b];
    r.random = randoms[(size_t)i * batch + b];
    blk->rows[b] = r;
    history[(size_t)b * max_ctx + pos] = tok;
}

__global__ void k_loop_post(LoopState* L, const StepBlock* blk, uint32_t* ids, uint32_t batch) {
    uint32_t b = threadIdx.x;
    uint32_t i = L->i;
    if (b < batch) ids[(size_t)i * batch + b] = blk->out[b];
    __syncthreads();
    if (b == 0) L->i = i + 1;
}

// Batched decode (more than kMaxStepBatch sequences per step): one block of u32 arrays for
// `cap` sequences (cap a multiple of 4), offsets below; SampleRow entries are 4 words.
struct BatchLayout {
    uint32_t cap;
    __host__ __device__ uint32_t tok() const { return 0; }
    __host__ __device__ uint32_t pos() const { return cap; }
    __host__ __device__ uint32_t hist() const { return 2 * cap; }
    __host__ __device__ uint32_t rows() const { return 3 * cap; }
    __host__ __device__ uint32_t out() const { return 7 * cap; }
    __host__ __device__ uint32_t err() const { return 8 * cap; }
    __host__ __device__ uint32_t step() const { return 8 * cap + 1; }
    __host__ __device__ uint32_t base() const { return 8 * cap + 4; }
    __host__ __device__ uint32_t first() const { return 9 * cap + 4; }
    __host__ __device__ uint32_t params() const { return 10 * cap + 4; }
    __host__ __device__ uint32_t words() const { return 14 * cap + 4; }
};

__global__ void k_batch_prep(uint32_t* blk, BatchLayout Lb, uint32_t* history, uint32_t max_ctx, uint32_t batch) {
    for (uint32_t b = threadIdx.x; b < batch; b += blockDim.x)
        history[(size_t)b * max_ctx + blk[Lb.pos() + b]] = blk[Lb.tok() + b];
}

__global__ void k_batch_loop_prep(uint32_t* blk, BatchLayout Lb, const float* randoms, const uint32_t* ids,
                                  uint32_t* history, uint32_t max_ctx, uint32_t batch) {
    const uint32_t i = blk[Lb.step()];
    for (uint32_t b = threadIdx.x; b < batch; b += blockDim.x) {
        const uint32_t tok = i == 0 ? blk[Lb.first() + b] : ids[(size_t)(i - 1) * batch + b];
        const uint32_t pos = blk[Lb.base() + b] + i;
        blk[Lb.tok() + b] = tok;
        blk[Lb.pos() + b] = pos;
        blk[Lb.hist() + b] = pos + 1;
        SampleRow r = reinterpret_cast<const SampleRow*>(blk + Lb.params())[b];
        r.random = randoms[(size_t)i * batch + b];
        reinterpret_cast<SampleRow*>(blk + Lb.rows())[b] = r;
        history[(size_t)b * max_ctx + pos] = tok;
    }
}

__global__ void k_batch_loop_post(uint32_t* blk, BatchLayout Lb, uint32_t* ids, uint32_t batch) {
    const uint32_t i = blk[Lb.step()];
    for (uint32_t b = threadIdx.x; b < batch; b += blockDim.x) ids[(size_t)i * batch + b] = blk[Lb.out() + b];
    __syncthreads();
    if (threadIdx.x == 0) blk[Lb.step()] = i + 1;
}

}  // namespace

static enx_status ensure_codes8(enx_ctx* c);

struct enx_ctx {
    enx_model_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::map<std::string, Tensor> tensors;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    bool loaded = false;
    std::vector<LayerArgs> layers;
    HeadArgs head{};
    // KV and per-sequence state
    uint32_t max_ctx = 0, batch = 0;
    uint16_t* kcache = nullptr;
    uint16_t* vcache = nullptr;
    double* rope_cos = nullptr;
    double* rope_sin = nullptr;
    uint32_t* history = nullptr;  // [batch][max_ctx]
    std::vector<uint32_t> filled;
    // decode step buffers
    float *x = nullptr, *q = nullptr, *gated = nullptr, *logits = nullptr, *normed = nullptr,
          *scores = nullptr, *attn_out = nullptr, *x_mid = nullptr;
    StepBlock* d_step = nullptr;
    StepBlock* h_step = nullptr;
    cudaGraphExec_t graph[kMaxStepBatch + 1] = {};
    uint32_t graph_launches[kMaxStepBatch + 1] = {};
    cudaGraphExec_t loop_graph[kMaxStepBatch + 1] = {};
    cudaGraphExec_t loop_graph_n[kMaxStepBatch + 1] = {};  // kLoopGraphSteps loop steps in one graph
    uint32_t loop_launches[kMaxStepBatch + 1] = {};
    LoopState* d_loop = nullptr;
    LoopState* h_loop = nullptr;
    float* d_loop_rand = nullptr;
    uint32_t* d_loop_ids = nullptr;
    uint32_t* h_loop_ids = nullptr;
    uint32_t loop_cap = 0, loop_count = 0;
    unsigned long long* d_bar = nullptr;  // step counters; word 0: tag epoch of the persistent step kernel
    unsigned long long* d_ll = nullptr;   // tagged stage outputs of the persistent step kernel
    double* d_nll = nullptr;              // enx_nll's result
    unsigned long long* d_trace = nullptr;  // stage stamps when tracing is on
    uint32_t trace_len = 0;
    bool graph_mega[kMaxStepBatch + 1] = {};
    bool loop_mega[kMaxStepBatch + 1] = {};
    // persistent step kernel: slice tables per batch size, head-major o-projection, per-head partials
    MegaSlice* d_table[kMaxStepBatch + 1] = {};
    uint32_t* d_nslices[kMaxStepBatch + 1] = {};
    uint32_t table_stride[kMaxStepBatch + 1] = {};
    uint32_t last_launches = 0;
    // prefill buffers (chunk-sized)
    uint32_t pf_chunk = 0;
    float *pf_x = nullptr, *pf_n = nullptr, *pf_q = nullptr, *pf_q2 = nullptr, *pf_k = nullptr,
          *pf_k2 = nullptr, *pf_v = nullptr, *pf_att = nullptr, *pf_t = nullptr, *pf_g = nullptr,
          *pf_u = nullptr, *pf_part = nullptr;
    double* pf_apart = nullptr;  // split partial sums of the many-token attention
    uint8_t* pf_ws = nullptr;  // tensor-core GEMM workspace (activation limbs) for prefill chunks
    // batched decode: more than kMaxStepBatch sequences per step (the tensor-core GEMM path)
    BatchLayout bl{};
    uint32_t* d_bb = nullptr;  // BatchLayout block
    uint32_t* h_bb = nullptr;  // pinned mirror
    double* b_part = nullptr;  // split partial sums of the many-token attention
    float *b_x = nullptr, *b_xn = nullptr, *b_q = nullptr, *b_k = nullptr, *b_v = nullptr, *b_att = nullptr,
          *b_t = nullptr, *b_g = nullptr, *b_u = nullptr, *b_scores = nullptr, *b_rand = nullptr;
    uint32_t* b_ids = nullptr;
    uint8_t* b_ws = nullptr;
    // int4 projection weights as the byte matrices (q - z) the tensor-core GEMM reads, by packed pointer
    std::map<const uint32_t*, uint8_t*> codes8;  // int8 code matrix of each int4 projection (may alias a stack)
    std::vector<void*> codes8_bufs;                // the allocations behind codes8 and the stacks' scales
    struct Stacked {
        QW qkv, gu;               // q|k|v and gate|up rows one after another (stacked scales)
        const uint8_t* qkv_codes;
        const uint8_t* gu_codes;
    };
    std::vector<Stacked> stacked;  // per layer, with codes8
    std::map<uint32_t, cudaGraphExec_t> b_graph, b_loop_graph;
    std::map<uint32_t, uint32_t> b_launches;
    bool loop_batched = false;  // the last enx_decode_loop ran the batched path
    uint32_t* pf_ids = nullptr;
};

namespace {

template <typename T>
enx_status dalloc(T** p, size_t count, const char* what) {
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
    if (e != cudaSuccess) return fail(ENX_ERR_NOMEM, std::string("cudaMalloc(") + what + "): " + cudaGetErrorString(e));
    return ENX_OK;
}


template <typename T>
void dfree(T*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

// ENX_ERR_TIMEOUT with the caller's name and which wait gave up (codes of the device error words:
// 1 grid barrier or readiness counter, 2 weight copy into the ring, 3 tensor-core GEMM pipeline).
static enx_status timeout_error(const char* caller, uint32_t code) {
    const char* what = code == 1 ? "grid barrier" : code == 2 ? "weight copy" : code == 3 ? "tensor-core GEMM wait" : "device wait";
    return fail(ENX_ERR_TIMEOUT, std::string(caller) + ": a bounded device wait gave up (" + what + ")");
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

void free_graphs(enx_ctx* c) {
    for (auto& g : c->graph) {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    }
    for (auto& g : c->loop_graph) {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    }
    for (auto& g : c->loop_graph_n) {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    }
    for (auto& kv : c->b_graph) cudaGraphExecDestroy(kv.second);
    for (auto& kv : c->b_loop_graph) cudaGraphExecDestroy(kv.second);
    c->b_graph.clear();
    c->b_loop_graph.clear();
    for (uint32_t b = 0; b <= kMaxStepBatch; ++b) {
        dfree(c->d_table[b]);
        dfree(c->d_nslices[b]);
        c->table_stride[b] = 0;
    }
}

void free_prefill(enx_ctx* c) {
    dfree(c->pf_x); dfree(c->pf_n); dfree(c->pf_q); dfree(c->pf_q2); dfree(c->pf_k); dfree(c->pf_k2);
    dfree(c->pf_v); dfree(c->pf_att); dfree(c->pf_t); dfree(c->pf_g); dfree(c->pf_u); dfree(c->pf_part); dfree(c->pf_apart);
    dfree(c->pf_ids);
    dfree(c->pf_ws);
    c->pf_chunk = 0;
}

void free_kv(enx_ctx* c) {
    free_graphs(c);
    free_prefill(c);
    dfree(c->kcache); dfree(c->vcache); dfree(c->rope_cos); dfree(c->rope_sin); dfree(c->history);
    dfree(c->x); dfree(c->q); dfree(c->gated); dfree(c->logits); dfree(c->normed); dfree(c->scores); dfree(c->attn_out); dfree(c->x_mid);
    dfree(c->d_step);
    if (c->h_step) cudaFreeHost(c->h_step);
    c->h_step = nullptr;
    dfree(c->d_loop); dfree(c->d_loop_rand); dfree(c->d_loop_ids); dfree(c->d_bar); dfree(c->d_ll); dfree(c->d_nll);
    if (c->h_loop) cudaFreeHost(c->h_loop);
    if (c->h_loop_ids) cudaFreeHost(c->h_loop_ids);
    c->h_loop = nullptr;
    c->h_loop_ids = nullptr;
    c->loop_cap = c->loop_count = 0;
    dfree(c->d_bb); dfree(c->b_x); dfree(c->b_xn); dfree(c->b_q); dfree(c->b_k); dfree(c->b_v); dfree(c->b_att);
    dfree(c->b_t); dfree(c->b_g); dfree(c->b_u); dfree(c->b_scores); dfree(c->b_rand); dfree(c->b_ids); dfree(c->b_ws); dfree(c->b_part);
    if (c->h_bb) cudaFreeHost(c->h_bb);
    c->h_bb = nullptr;
    c->bl = BatchLayout{};
    c->max_ctx = c->batch = 0;
    c->filled.clear();
}

const Tensor* find(enx_ctx* c, const std::string& name, int bits, uint32_t rows, uint32_t cols,
                   std::string& err) {
    auto it = c->tensors.find(name);
    if (it == c->tensors.end()) { err = "missing tensor " + name; return nullptr; }
    const Tensor& t = it->second;
    if ((bits == 32) != (t.bits == 32) || (bits != 32 && bits != 0 && t.bits != bits)) {
        err = name + ": unexpected dtype";
        return nullptr;
    }
    if (t.rows != rows || t.cols != cols) {
        err = name + ": shape [" + std::to_string(t.rows) + ", " + std::to_string(t.cols) + "] expected [" +
              std::to_string(rows) + ", " + std::to_string(cols) + "]";
        return nullptr;
    }
    return &t;
}

QW qw(const Tensor* t) {
    return QW{static_cast<const uint32_t*>(t->packed), t->scales, t->zeros, t->rows, t->cols};
}

enx_status bind_model(enx_ctx* c) {
    const enx_model_config& C = c->cfg;
    const uint32_t H = C.hidden, kv = C.kv_heads * C.head_dim, I = C.intermediate;
    std::string err;
    c->layers.assign(C.layers, LayerArgs{});
    for (uint32_t l = 0; l < C.layers; ++l) {
        std::string p = "model.layers." + std::to_string(l) + ".";
        LayerArgs& L = c->layers[l];
        L.layer = l;
        const Tensor* t;
#define NEED(var, name, bits, r, cl)                                 \
    t = find(c, p + name, bits, r, cl, err);                        \
    if (!t) return fail(ENX_ERR_FORMAT, err);                        \
    var = t;
        const Tensor *tin, *tpost, *tq, *tk, *tv, *to, *tg, *tu, *td, *bq, *bk, *bv;
        NEED(tin, "input_layernorm.weight", 32, H, 1);
        NEED(tpost, "post_attention_layernorm.weight", 32, H, 1);
        NEED(tq, "self_attn.q_proj.weight", 4, H, H);
        NEED(tk, "self_attn.k_proj.weight", 4, kv, H);
        NEED(tv, "self_attn.v_proj.weight", 4, kv, H);
        NEED(to, "self_attn.o_proj.weight", 4, H, H);
        NEED(tg, "mlp.gate_proj.weight", 4, I, H);
        NEED(tu, "mlp.up_proj.weight", 4, I, H);
        NEED(td, "mlp.down_proj.weight", 4, H, I);
        NEED(bq, "self_attn.q_proj.bias", 32, H, 1);
        NEED(bk, "self_attn.k_proj.bias", 32, kv, 1);
        NEED(bv, "self_attn.v_proj.bias", 32, kv, 1);
#undef NEED
        L.norm_in = static_cast<const float*>(tin->packed);
        L.norm_post = static_cast<const float*>(tpost->packed);
        L.wq = qw(tq); L.wk = qw(tk); L.wv = qw(tv); L.wo = qw(to); L.wg = qw(tg); L.wu = qw(tu); L.wd = qw(td);
        L.bq = static_cast<const float*>(bq->packed);
        L.bk = static_cast<const float*>(bk->packed);
        L.bv = static_cast<const float*>(bv->packed);
    }
    const Tensor* e = find(c, "model.embed_tokens.weight", 0, C.vocab, H, err);
    if (!e) return fail(ENX_ERR_FORMAT, err);
    if (e->bits != 4 && e->bits != 8) return fail(ENX_ERR_FORMAT, "embedding must be Q4 or Q8");
    const Tensor* fn = find(c, "model.norm.weight", 32, H, 1, err);
    if (!fn) return fail(ENX_ERR_FORMAT, err);
    c->head.embed = qw(e);
    c->head.bits = e->bits;
    c->head.norm = static_cast<const float*>(fn->packed);
    return ENX_OK;
}

}  // namespace


extern "C" enx_status enx_create(const enx_model_config* cfg, int device, enx_ctx** out) {
    CHECK_ARG(cfg && out, "enx_create: null pointer");
    const enx_model_config& C = *cfg;
    CHECK_ARG(C.layers > 0 && C.hidden > 0 && C.heads > 0 && C.kv_heads > 0 && C.vocab > 0, "enx_create: empty config");
    CHECK_ARG(C.heads % C.kv_heads == 0, "enx_create: heads must be a multiple of kv_heads");
    CHECK_ARG(C.heads * C.head_dim == C.hidden, "enx_create: heads*head_dim must equal hidden");
    CHECK_ARG(C.head_dim % 2 == 0 && C.head_dim <= 64, "enx_create: head_dim must be even and <= 64");
    CHECK_ARG(C.heads / C.kv_heads <= 8, "enx_create: at most 8 query heads per kv head");
    CHECK_ARG(C.hidden % 64 == 0 && C.intermediate % 64 == 0, "enx_create: hidden/intermediate must be multiples of 64");
    CHECK_ARG(C.vocab <= sample_max_vocab(), "enx_create: vocabulary exceeds the sampler's on-chip limit");
    int n = 0;
    ENX_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(ENX_ERR_INVALID, "enx_create: no CUDA device " + std::to_string(device));
    DeviceGuard g(device);
    std::unique_ptr<enx_ctx> c(new enx_ctx());
    c->cfg = C;
    c->device = device;
    ENX_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    *out = c.release();
    return ENX_OK;
}

extern "C" enx_status enx_destroy(enx_ctx* c) {
    if (!c) return ENX_OK;
    {
        DeviceGuard g(c->device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        free_kv(c);
        dfree(c->d_trace);
        for (void* b : c->codes8_bufs) cudaFree(b);
        if (c->arena) cudaFree(c->arena);
        if (c->stream) cudaStreamDestroy(c->stream);
    }
    delete c;
    return ENX_OK;
}

extern "C" enx_status enx_load_enargeia_memory(enx_ctx* c, const void* data, size_t size) {
    CHECK_ARG(c && data, "enx_load_enargeia: null pointer");
    const uint8_t* raw = static_cast<const uint8_t*>(data);
    if (size < 16) return fail(ENX_ERR_FORMAT, "need at least 16 bytes to read the header length");
    if (std::memcmp(raw, "ENARGEIA", 8) != 0) return fail(ENX_ERR_FORMAT, "not a .enargeia file: bad magic");
    uint32_t version, hlen;
    std::memcpy(&version, raw + 8, 4);
    std::memcpy(&hlen, raw + 12, 4);
    if (version != 1) return fail(ENX_ERR_FORMAT, "unsupported .enargeia version " + std::to_string(version) + ", expected 1");
    if (hlen > 64u * 1024 * 1024 || 16 + (size_t)hlen > size) return fail(ENX_ERR_FORMAT, "header length out of range");
    size_t data_off = 16 + (size_t)hlen;
    data_off += (256 - data_off % 256) % 256;
    json::Value root;
    std::string perr;
    if (!json::parse(std::string(reinterpret_cast<const char*>(raw + 16), hlen), root, perr))
        return fail(ENX_ERR_FORMAT, "header JSON: " + perr);
    const json::Value* tensors = root.get("tensors");
    if (!tensors || !tensors->is_object()) return fail(ENX_ERR_FORMAT, "header has no tensors object");

    struct Range { size_t b, e; };
    struct Plan { Tensor t; Range r[3]; int nr; };
    std::map<std::string, Plan> plan;
    size_t total = 0;
    auto range = [&](const json::Value* v, Range& r) -> bool {
        if (!v || !v->is_array() || v->arr.size() != 2) return false;
        r.b = (size_t)v->arr[0].num;
        r.e = (size_t)v->arr[1].num;
        return r.e >= r.b && data_off + r.e <= size && r.b % 256 == 0;
    };
    for (auto& kvp : tensors->obj) {
        const std::string& name = kvp.first;
        const json::Value& e = kvp.second;
        const json::Value* dt = e.get("dtype");
        const json::Value* sh = e.get("shape");
        const json::Value* of = e.get("offsets");
        if (!dt || !sh || !of || !sh->is_array()) return fail(ENX_ERR_FORMAT, name + ": incomplete entry");
        Plan p{};
        if (dt->str == "Q4" || dt->str == "Q8") {
            if (sh->arr.size() != 2) return fail(ENX_ERR_FORMAT, name + ": quantised tensor must be 2-D");
            p.t.bits = dt->str == "Q4" ? 4 : 8;
            p.t.rows = (uint32_t)sh->arr[0].num;
            p.t.cols = (uint32_t)sh->arr[1].num;
            const json::Value* bs = e.get("blockSize");
            if (bs && (uint32_t)bs->num != 64) return fail(ENX_ERR_FORMAT, name + ": block size must be 64");
            if (p.t.cols % 64) return fail(ENX_ERR_FORMAT, name + ": reduction axis not a multiple of 64");
            if (!range(of->get("packed"), p.r[0]) || !range(of->get("scales"), p.r[1]) || !range(of->get("zeros"), p.r[2]))
                return fail(ENX_ERR_FORMAT, name + ": bad byte range");
            size_t elems = (size_t)p.t.rows * p.t.cols, blocks = elems / 64, per = 32 / p.t.bits;
            if (p.r[0].e - p.r[0].b != elems / per * 4 || p.r[1].e - p.r[1].b != blocks * 4 ||
                p.r[2].e - p.r[2].b != (blocks + per - 1) / per * 4)
                return fail(ENX_ERR_FORMAT, name + ": range sizes do not match the shape");
            p.nr = 3;
        } else if (dt->str == "F32") {
            p.t.bits = 32;
            size_t n = 1;
            for (auto& d : sh->arr) n *= (size_t)d.num;
            p.t.rows = sh->arr.empty() ? 1 : (uint32_t)sh->arr[0].num;
            p.t.cols = sh->arr.size() >= 2 ? (uint32_t)(n / p.t.rows) : 1;
            if (!range(of->get("data"), p.r[0]) || p.r[0].e - p.r[0].b != n * 4)
                return fail(ENX_ERR_FORMAT, name + ": bad data range");
            p.nr = 1;
        } else {
            return fail(ENX_ERR_FORMAT, name + ": dtype " + dt->str + " unsupported on this path");
        }
        for (int i = 0; i < p.nr; ++i) total += (p.r[i].e - p.r[i].b + 255) / 256 * 256 + 256;
        plan[name] = p;
    }
    DeviceGuard g(c->device);
    if (c->arena) { cudaFree(c->arena); c->arena = nullptr; }
    for (void* b : c->codes8_bufs) cudaFree(b);
    c->codes8_bufs.clear();
    c->codes8.clear();
    c->stacked.clear();
    c->tensors.clear();
    c->loaded = false;
    free_graphs(c);
    ENX_TRY(dalloc(reinterpret_cast<uint8_t**>(&c->arena), total, "weights"));
    c->arena_bytes = total;
    uint8_t* cur = static_cast<uint8_t*>(c->arena);
    // Ranges go to the device verbatim; every range starts 256-aligned and keeps 16 bytes of
    // slack after it so 16-byte vector loads at the tail never leave the allocation.
    for (auto& kvp : plan) {
        Plan& p = kvp.second;
        void* dst[3];
        for (int i = 0; i < p.nr; ++i) {
            size_t n = p.r[i].e - p.r[i].b;
            ENX_CUDA(cudaMemcpyAsync(cur, raw + data_off + p.r[i].b, n, cudaMemcpyHostToDevice, c->stream));
            dst[i] = cur;
            cur += (n + 255) / 256 * 256 + 256;
        }
        p.t.packed = dst[0];
        if (p.nr == 3) {
            p.t.scales = static_cast<float*>(dst[1]);
            p.t.zeros = static_cast<uint32_t*>(dst[2]);
        }
        p.t.bytes = 0;
        for (int i = 0; i < p.nr; ++i) p.t.bytes += p.r[i].e - p.r[i].b;
        c->tensors[kvp.first] = p.t;
    }
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    ENX_TRY(bind_model(c));
    c->loaded = true;
    if (c->pf_ws || (c->d_bb && c->batch >= kTcMinTokens)) ENX_TRY(ensure_codes8(c));  // buffers set up before the load
    return ENX_OK;
}

extern "C" enx_status enx_load_enargeia(enx_ctx* c, const char* path) {
    CHECK_ARG(c && path, "enx_load_enargeia: null pointer");
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) return fail(ENX_ERR_FORMAT, std::string("cannot open ") + path);
    size_t n = (size_t)f.tellg();
    f.seekg(0);
    void* host = nullptr;
    // pinned staging so the upload runs at full PCIe rate
    if (cudaMallocHost(&host, n) != cudaSuccess) return fail(ENX_ERR_NOMEM, "cudaMallocHost for the model file");
    f.read(static_cast<char*>(host), (std::streamsize)n);
    enx_status s = f ? enx_load_enargeia_memory(c, host, n) : fail(ENX_ERR_FORMAT, "short read");
    cudaFreeHost(host);
    return s;
}

extern "C" enx_status enx_kv_alloc(enx_ctx* c, uint32_t max_context, uint32_t batch) {
    CHECK_ARG(c, "enx_kv_alloc: null context");
    CHECK_ARG(max_context > 0 && batch > 0, "enx_kv_alloc: empty cache");
    const enx_model_config& C = c->cfg;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    free_kv(c);
    const size_t kv = (size_t)C.kv_heads * C.head_dim;
    const size_t per = (size_t)batch * C.layers * max_context * kv;
    ENX_TRY(dalloc(&c->kcache, per, "k cache"));
    ENX_TRY(dalloc(&c->vcache, per, "v cache"));
    ENX_CUDA(cudaMemsetAsync(c->kcache, 0, per * 2, c->stream));
    ENX_CUDA(cudaMemsetAsync(c->vcache, 0, per * 2, c->stream));
    // RoPE table: f64 angle, cos and sin rounded once to f32 (src/kernels/rope.wgsl:42-46)
    const uint32_t half = C.head_dim / 2;
    std::vector<double> ct((size_t)max_context * half), st((size_t)max_context * half);
    for (uint32_t p = 0; p < max_context; ++p)
        for (uint32_t i = 0; i < half; ++i) {
            double freq = 1.0 / std::pow((double)C.rope_theta, (2.0 * i) / (double)C.head_dim);
            double a = (double)p * freq;
            ct[(size_t)p * half + i] = std::cos(a);
            st[(size_t)p * half + i] = std::sin(a);
        }
    ENX_TRY(dalloc(&c->rope_cos, ct.size(), "rope cos"));
    ENX_TRY(dalloc(&c->rope_sin, st.size(), "rope sin"));
    ENX_CUDA(cudaMemcpy(c->rope_cos, ct.data(), ct.size() * 8, cudaMemcpyHostToDevice));
    ENX_CUDA(cudaMemcpy(c->rope_sin, st.data(), st.size() * 8, cudaMemcpyHostToDevice));
    ENX_TRY(dalloc(&c->history, (size_t)batch * max_context, "history"));
    const uint32_t B = batch < kMaxStepBatch ? batch : kMaxStepBatch;
    ENX_TRY(dalloc(&c->x, (size_t)B * C.hidden, "x"));
    ENX_TRY(dalloc(&c->q, (size_t)B * C.hidden, "q"));
    ENX_TRY(dalloc(&c->gated, (size_t)B * C.intermediate, "gated"));
    ENX_TRY(dalloc(&c->logits, (size_t)batch * C.vocab, "logits"));
    ENX_TRY(dalloc(&c->normed, (size_t)batch * C.hidden, "normed"));
    ENX_TRY(dalloc(&c->scores, (size_t)B * splits_for(max_context) * kAttnChunk * C.heads, "attention scores"));
    ENX_TRY(dalloc(&c->attn_out, (size_t)B * C.hidden, "attention output"));
    ENX_TRY(dalloc(&c->x_mid, (size_t)B * C.hidden, "residual after attention"));
    ENX_TRY(dalloc(&c->d_step, 1, "step block"));
    if (cudaMallocHost(&c->h_step, sizeof(StepBlock)) != cudaSuccess) return fail(ENX_ERR_NOMEM, "pinned step block");
    std::memset(c->h_step, 0, sizeof(StepBlock));
    // device-fed loop: room for every step the caches can hold
    c->loop_cap = max_context * B;
    ENX_TRY(dalloc(&c->d_nll, 1, "nll result"));
    ENX_TRY(dalloc(&c->d_bar, kMegaBarWords, "step counters"));
    ENX_CUDA(cudaMemsetAsync(c->d_bar, 0, kMegaBarWords * sizeof(unsigned long long), c->stream));
    ENX_CUDA(cudaMemsetAsync(c->d_step, 0, sizeof(StepBlock), c->stream));
    ENX_TRY(dalloc(&c->d_loop, 1, "loop state"));
    ENX_TRY(dalloc(&c->d_loop_rand, c->loop_cap, "loop randoms"));
    ENX_TRY(dalloc(&c->d_loop_ids, c->loop_cap, "loop ids"));
    if (cudaMallocHost(&c->h_loop, sizeof(LoopState)) != cudaSuccess) return fail(ENX_ERR_NOMEM, "pinned loop state");
    if (cudaMallocHost(&c->h_loop_ids, (size_t)c->loop_cap * 4) != cudaSuccess) return fail(ENX_ERR_NOMEM, "pinned loop ids");
    if (batch > kMaxStepBatch) {  // batched decode buffers
        const size_t Bn = batch, H = C.hidden, kvd = (size_t)C.kv_heads * C.head_dim, I = C.intermediate;
        c->bl.cap = (batch + 3) & ~3u;
        ENX_TRY(dalloc(&c->d_bb, c->bl.words(), "batch block"));
        ENX_CUDA(cudaMemset(c->d_bb, 0, (size_t)c->bl.words() * 4));
        if (cudaMallocHost(&c->h_bb, (size_t)c->bl.words() * 4) != cudaSuccess) return fail(ENX_ERR_NOMEM, "pinned batch block");
        std::memset(c->h_bb, 0, (size_t)c->bl.words() * 4);
        ENX_TRY(dalloc(&c->b_x, Bn * H, "batch x"));
        ENX_TRY(dalloc(&c->b_xn, Bn * H, "batch normed"));
        ENX_TRY(dalloc(&c->b_q, Bn * H, "batch q"));
        ENX_TRY(dalloc(&c->b_k, Bn * kvd, "batch k"));
        ENX_TRY(dalloc(&c->b_v, Bn * kvd, "batch v"));
        ENX_TRY(dalloc(&c->b_att, Bn * H, "batch attention"));
        ENX_TRY(dalloc(&c->b_t, Bn * H, "batch projection"));
        ENX_TRY(dalloc(&c->b_g, Bn * I, "batch gate"));
        ENX_TRY(dalloc(&c->b_u, Bn * I, "batch up"));
        ENX_TRY(dalloc(&c->b_scores, Bn * split_stride(max_context) * C.heads, "batch scores"));
        ENX_TRY(dalloc(&c->b_part, Bn * (split_stride(max_context) / kAttnSplit) * H, "batch attention splits"));
        ENX_TRY(dalloc(&c->b_rand, Bn * max_context, "batch loop randoms"));
        ENX_TRY(dalloc(&c->b_ids, Bn * max_context, "batch loop ids"));
        ENX_TRY(dalloc(&c->b_ws, gemm_tc_workspace_bytes(batch, (uint32_t)(I > H ? I : H)), "batch GEMM workspace"));
        if (batch >= kTcMinTokens) ENX_TRY(ensure_codes8(c));
    }
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    c->max_ctx = max_context;
    c->batch = batch;
    c->filled.assign(batch, 0);
    return ENX_OK;
}

extern "C" enx_status enx_kv_reset(enx_ctx* c, uint32_t seq) {
    CHECK_ARG(c, "enx_kv_reset: null context");
    if (seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_kv_reset: sequence " + std::to_string(seq) + " outside the cache");
    c->filled[seq] = 0;
    return ENX_OK;
}

extern "C" enx_status enx_kv_filled(enx_ctx* c, uint32_t seq, uint32_t* filled) {
    CHECK_ARG(c && filled, "enx_kv_filled: null pointer");
    if (seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_kv_filled: sequence outside the cache");
    *filled = c->filled[seq];
    return ENX_OK;
}

static StepArgs step_args(enx_ctx* c) {
    const enx_model_config& C = c->cfg;
    StepArgs S{};
    S.hidden = C.hidden;
    S.heads = C.heads;
    S.kv_heads = C.kv_heads;
    S.head_dim = C.head_dim;
    S.intermediate = C.intermediate;
    S.eps = C.rms_norm_eps;
    S.x = c->x;
    S.q = c->q;
    S.gated = c->gated;
    S.logits = c->logits;
    S.normed = c->normed;
    S.scores = c->scores;
    S.attn_out = c->attn_out;
    S.score_stride = splits_for(c->max_ctx) * kAttnChunk;
    S.pos = nullptr;
    S.pos_base = 0;
    S.seq_fixed = 0xFFFFFFFFu;
    S.rope_cos = c->rope_cos;
    S.rope_sin = c->rope_sin;
    S.kcache = c->kcache;
    S.vcache = c->vcache;
    S.layers = C.layers;
    S.max_context = c->max_ctx;
    return S;
}

// The byte matrices of every int4 projection weight for the tensor-core GEMM, prepared once
// (before any graph capture) and reused by prefill and batched decode.  q|k|v and gate|up share
// their input, so their matrices are laid out one after another (with a stacked copy of their
// scales) and each runs as one GEMM over the stack; the single weights' code pointers point into
// the stack.
static enx_status ensure_codes8(enx_ctx* c) {
    if (!c->codes8.empty()) return ENX_OK;
    auto stack = [&](std::initializer_list<const QW*> ws, QW& sw, const uint8_t*& codes) -> enx_status {
        uint32_t rows = 0;
        const uint32_t K = (*ws.begin())->cols, bpr = K / kBlock;
        for (const QW* w : ws) rows += w->rows;
        uint8_t* buf = nullptr;
        float* sc = nullptr;
        ENX_TRY(dalloc(&buf, gemm_tc_codes_bytes(rows, K), "GEMM code matrix"));
        c->codes8_bufs.push_back(buf);
        ENX_TRY(dalloc(&sc, (size_t)rows * bpr, "GEMM stacked scales"));
        c->codes8_bufs.push_back(sc);
        uint32_t r = 0;
        for (const QW* w : ws) {
            c->codes8[w->packed] = buf + (size_t)r * K;
            ENX_CUDA(launch_codes_i8(*w, buf + (size_t)r * K, c->stream));
            ENX_CUDA(cudaMemcpyAsync(sc + (size_t)r * bpr, w->scales, (size_t)w->rows * bpr * 4, cudaMemcpyDeviceToDevice,
                                     c->stream));
            r += w->rows;
        }
        sw = QW{nullptr, sc, nullptr, rows, K};
        codes = buf;
        return ENX_OK;
    };
    c->stacked.assign(c->layers.size(), enx_ctx::Stacked{});
    for (size_t l = 0; l < c->layers.size(); ++l) {
        const LayerArgs& L = c->layers[l];
        enx_ctx::Stacked& S = c->stacked[l];
        ENX_TRY(stack({&L.wq, &L.wk, &L.wv}, S.qkv, S.qkv_codes));
        ENX_TRY(stack({&L.wg, &L.wu}, S.gu, S.gu_codes));
        for (const QW* w : {&L.wo, &L.wd}) {
            if (c->codes8.count(w->packed)) continue;
            uint8_t* buf = nullptr;
            ENX_TRY(dalloc(&buf, gemm_tc_codes_bytes(w->rows, w->cols), "GEMM code matrix"));
            c->codes8_bufs.push_back(buf);
            c->codes8[w->packed] = buf;
            ENX_CUDA(launch_codes_i8(*w, buf, c->stream));
        }
    }
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return ENX_OK;
}

// One tensor-core GEMM over layer l's q|k|v stack (outputs q, k, v with their biases) or its
// gate|up stack (outputs g, u): the stacked rows' input is normalised x, m rows.
static cudaError_t proj_qkv(enx_ctx* c, uint32_t l, const float* x, float* q, float* k, float* v, uint32_t m,
                            uint8_t* ws, uint32_t* err, cudaStream_t st) {
    const LayerArgs& L = c->layers[l];
    const uint32_t H = L.wq.rows, kv = L.wk.rows;
    TcSeg seg{};
    seg.out[0] = q, seg.out[1] = k, seg.out[2] = v;
    seg.bias[0] = L.bq, seg.bias[1] = L.bk, seg.bias[2] = L.bv;
    seg.stride[0] = H, seg.stride[1] = kv, seg.stride[2] = kv;
    seg.end[0] = H, seg.end[1] = H + kv, seg.end[2] = H + 2 * kv;
    seg.n = 3;
    const enx_ctx::Stacked& S = c->stacked[l];
    return launch_gemm_tc(4, x, S.qkv.cols, S.qkv, S.qkv_codes, nullptr, nullptr, m, 0, 0, ws, err, st, false, nullptr, &seg);
}
static cudaError_t proj_gu(enx_ctx* c, uint32_t l, const float* x, float* g, float* u, uint32_t m, uint8_t* ws,
                           uint32_t* err, cudaStream_t st) {
    const uint32_t I = c->layers[l].wg.rows;
    TcSeg seg{};
    seg.out[0] = g, seg.out[1] = u;
    seg.stride[0] = I, seg.stride[1] = I;
    seg.end[0] = I, seg.end[1] = 2 * I;
    seg.n = 2;
    const enx_ctx::Stacked& S = c->stacked[l];
    return launch_gemm_tc(4, x, S.gu.cols, S.gu, S.gu_codes, nullptr, nullptr, m, 0, 0, ws, err, st, false, nullptr, &seg);
}

static const uint8_t* codes_of(const enx_ctx* c, const QW& w) {
    const auto it = c->codes8.find(w.packed);
    return it == c->codes8.end() ? nullptr : it->second;
}

// A projection of m prefill rows: tensor cores for m >= kTcMinTokens, CUDA cores below.
// out += float(x W^T): the residual add fused into the tensor-core GEMM's output (its epilogue or
// split-K combine); below the tensor-core size, the projection into tmp and a separate add.
static cudaError_t proj_add(enx_ctx* c, const float* x, const QW& w, float* out, float* tmp, uint32_t m, uint32_t n,
                            cudaStream_t st, bool tc, uint8_t* ws, uint32_t* err) {
    if (tc) return launch_gemm_tc(4, x, w.cols, w, codes_of(c, w), nullptr, out, m, n, 0, ws, err, st, false, out);
    cudaError_t e = launch_matmul(4, x, w, nullptr, tmp, m, n, 0, st, false);
    return e == cudaSuccess ? launch_add(out, tmp, out, m * n, st) : e;
}

static cudaError_t proj(enx_ctx* c, int bits, const float* x, const QW& w, const float* bias, float* out, uint32_t m,
                        uint32_t stride, uint32_t offset, cudaStream_t st, bool same_x = false) {
    if (m >= kTcMinTokens && c->pf_ws && bits == 4 && !codes_of(c, w)) return cudaErrorInvalidValue;  // never prepared
    if (m >= kTcMinTokens && c->pf_ws)
        return launch_gemm_tc(bits, x, w.cols, w, bits == 4 ? codes_of(c, w) : nullptr, bias, out, m, stride, offset,
                              c->pf_ws, &c->d_step->err, st, same_x);
    return launch_matmul(bits, x, w, bias, out, m, stride, offset, st, false);
}

static enx_status ensure_prefill(enx_ctx* c, uint32_t chunk) {
    if (c->pf_chunk >= chunk) return ENX_OK;
    free_prefill(c);
    const enx_model_config& C = c->cfg;
    const size_t H = C.hidden, kv = (size_t)C.kv_heads * C.head_dim, I = C.intermediate;
    ENX_TRY(dalloc(&c->pf_x, chunk * H, "prefill x"));
    ENX_TRY(dalloc(&c->pf_n, chunk * H, "prefill normed"));
    ENX_TRY(dalloc(&c->pf_q, chunk * H, "prefill q"));
    ENX_TRY(dalloc(&c->pf_q2, chunk * H, "prefill q rope"));
    ENX_TRY(dalloc(&c->pf_k, chunk * kv, "prefill k"));
    ENX_TRY(dalloc(&c->pf_k2, chunk * kv, "prefill k rope"));
    ENX_TRY(dalloc(&c->pf_v, chunk * kv, "prefill v"));
    ENX_TRY(dalloc(&c->pf_att, chunk * H, "prefill attn"));
    ENX_TRY(dalloc(&c->pf_t, chunk * H, "prefill tmp"));
    ENX_TRY(dalloc(&c->pf_g, chunk * I, "prefill gate"));
    ENX_TRY(dalloc(&c->pf_u, chunk * I, "prefill up"));
    ENX_TRY(dalloc(&c->pf_part, (size_t)chunk * split_stride(c->max_ctx) * C.heads, "prefill scores"));
    ENX_TRY(dalloc(&c->pf_apart, (size_t)chunk * (split_stride(c->max_ctx) / kAttnSplit) * H, "prefill attention splits"));
    ENX_TRY(dalloc(&c->pf_ids, chunk, "prefill ids"));
    if (chunk >= kTcMinTokens) {
        ENX_TRY(dalloc(&c->pf_ws, gemm_tc_workspace_bytes(chunk, (uint32_t)(I > H ? I : H)), "prefill GEMM workspace"));
        ENX_TRY(ensure_codes8(c));
    }
    c->pf_chunk = chunk;
    return ENX_OK;
}

static enx_status device_error(enx_ctx* c, const char* caller);

extern "C" enx_status enx_prefill(enx_ctx* c, uint32_t seq, const uint32_t* ids, uint32_t n, uint32_t chunk) {
    CHECK_ARG(c && ids, "enx_prefill: null pointer");
    if (!c->loaded) return fail(ENX_ERR_STATE, "enx_prefill: no model loaded");
    if (!c->kcache) return fail(ENX_ERR_STATE, "enx_prefill: call enx_kv_alloc first");
    if (seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_prefill: sequence outside the cache");
    if (n < 1) return fail(ENX_ERR_RANGE, "prompt length 0 must be at least 1");
    const uint32_t remaining = c->max_ctx - c->filled[seq];
    if (n > remaining)
        return fail(ENX_ERR_RANGE, "prompt of " + std::to_string(n) + " exceeds the remaining context of " +
                                       std::to_string(remaining));
    const enx_model_config& C = c->cfg;
    for (uint32_t i = 0; i < n; ++i)
        if (ids[i] >= C.vocab) return fail(ENX_ERR_INVALID, "token id " + std::to_string(ids[i]) + " outside the vocabulary");
    if (chunk == 0 || chunk > n) chunk = n;
    DeviceGuard g(c->device);
    ENX_TRY(ensure_prefill(c, chunk));
    cudaStream_t st = c->stream;
    const uint32_t H = C.hidden, kv = C.kv_heads * C.head_dim, I = C.intermediate;
    const uint32_t filled0 = c->filled[seq];
    StepArgs S = step_args(c);
    S.seq_fixed = seq;
    S.q = c->pf_q2;
    S.scores = c->pf_part;
    S.score_stride = split_stride(c->max_ctx);
    S.attn_part = c->pf_apart;
    for (uint32_t begin0 = 0; begin0 < n; begin0 += chunk) {
        const uint32_t m = n - begin0 < chunk ? n - begin0 : chunk;
        const uint32_t begin = c->filled[seq];
        ENX_CUDA(cudaMemcpyAsync(c->pf_ids, ids + begin0, m * 4, cudaMemcpyHostToDevice, st));
        ENX_CUDA(cudaMemcpyAsync(c->history + (size_t)seq * c->max_ctx + begin, c->pf_ids, m * 4,
                                 cudaMemcpyDeviceToDevice, st));
        ENX_CUDA(launch_embed(c->pf_ids, c->head.embed, c->head.bits, c->pf_x, m, 0, C.vocab, H, st, false));
        S.pos_base = begin;
        for (uint32_t l = 0; l < C.layers; ++l) {
            const LayerArgs& L = c->layers[l];
            ENX_CUDA(launch_rmsnorm(c->pf_x, L.norm_in, c->pf_n, m, H, C.rms_norm_eps, st));
            const bool stk = m >= kTcMinTokens && c->pf_ws && l < c->stacked.size();  // one GEMM over q|k|v
            if (stk) {
                ENX_CUDA(proj_qkv(c, l, c->pf_n, c->pf_q, c->pf_k, c->pf_v, m, c->pf_ws, &c->d_step->err, st));
            } else {
                ENX_CUDA(proj(c, 4, c->pf_n, L.wq, L.bq, c->pf_q, m, H, 0, st));
                ENX_CUDA(proj(c, 4, c->pf_n, L.wk, L.bk, c->pf_k, m, kv, 0, st, true));  // limbs of pf_n reused
                ENX_CUDA(proj(c, 4, c->pf_n, L.wv, L.bv, c->pf_v, m, kv, 0, st, true));
            }
            ENX_CUDA(launch_rope_d(c->pf_q, c->pf_q2, c->rope_cos, c->rope_sin, m, C.heads, C.head_dim, begin, 0, st));
            ENX_CUDA(launch_rope_d(c->pf_k, c->pf_k2, c->rope_cos, c->rope_sin, m, C.kv_heads, C.head_dim, begin, 0, st));
            ENX_CUDA(launch_cache_pack(c->pf_k2, c->kcache + S.cache_offset(seq, l, begin), m * kv, 0, st));
            ENX_CUDA(launch_cache_pack(c->pf_v, c->vcache + S.cache_offset(seq, l, begin), m * kv, 0, st));
            ENX_CUDA(launch_attn(S, l, m, c->pf_att, st, false));
            const bool tc = m >= kTcMinTokens && c->pf_ws && codes_of(c, L.wo);
            ENX_CUDA(proj_add(c, c->pf_att, L.wo, c->pf_x, c->pf_t, m, H, st, tc, c->pf_ws, &c->d_step->err));
            ENX_CUDA(launch_rmsnorm(c->pf_x, L.norm_post, c->pf_n, m, H, C.rms_norm_eps, st));
            if (stk) {
                ENX_CUDA(proj_gu(c, l, c->pf_n, c->pf_g, c->pf_u, m, c->pf_ws, &c->d_step->err, st));
            } else {
                ENX_CUDA(proj(c, 4, c->pf_n, L.wg, nullptr, c->pf_g, m, I, 0, st));
                ENX_CUDA(proj(c, 4, c->pf_n, L.wu, nullptr, c->pf_u, m, I, 0, st, true));
            }
            ENX_CUDA(launch_silu_mul(c->pf_g, c->pf_u, c->pf_g, m * I, st));
            ENX_CUDA(proj_add(c, c->pf_g, L.wd, c->pf_x, c->pf_t, m, H, st, tc, c->pf_ws, &c->d_step->err));
        }
        c->filled[seq] += m;
        if (begin0 + m >= n) {
            // tail on the last chunk only: final norm of the last row, then the tied head
            float* last = c->normed + (size_t)seq * H;
            ENX_CUDA(launch_rmsnorm(c->pf_x + (size_t)(m - 1) * H, c->head.norm, last, 1, H, C.rms_norm_eps, st));
            ENX_CUDA(launch_matmul(c->head.bits, last, c->head.embed, nullptr, c->logits + (size_t)seq * C.vocab, 1,
                                   C.vocab, 0, st, false));
        }
    }
    ENX_CUDA(cudaStreamSynchronize(st));
    // the tensor-core GEMMs' bounded waits report through the step's error word; on a timeout the
    // cache rows this call wrote are not valid, so the sequence keeps its fill from before the call
    const enx_status e = device_error(c, "enx_prefill");
    if (e != ENX_OK) c->filled[seq] = filled0;
    return e;
}

extern "C" enx_status enx_sample_prefill(enx_ctx* c, uint32_t seq, const enx_sampling* params, float random,
                                         uint32_t* out_id) {
    CHECK_ARG(c && params && out_id, "enx_sample_prefill: null pointer");
    if (!c->kcache) return fail(ENX_ERR_STATE, "enx_sample_prefill: no cache");
    if (seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_sample_prefill: sequence outside the cache");
    if (c->filled[seq] == 0) return fail(ENX_ERR_STATE, "enx_sample_prefill: nothing prefilled");
    DeviceGuard g(c->device);
    SampleRow r{params->temperature, params->top_p, params->repetition_penalty, random};
    ENX_CUDA(launch_sample(c->logits + (size_t)seq * c->cfg.vocab, c->cfg.vocab, 1,
                           c->history + (size_t)seq * c->max_ctx, c->filled[seq], nullptr, nullptr, false, r,
                           c->d_step->out, c->stream, false));
    ENX_CUDA(cudaMemcpyAsync(out_id, c->d_step->out, 4, cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return ENX_OK;
}

// The persistent step kernel runs when it fits: its ring gets at least two slots in shared memory
// for this many tokens (in practice 1 or 2 for config 0), the scores of every cached position fit
// its activation area, the shape is within its fixed capacities (mega_geometry), and
// ENX_DECODE_PATH is not "kernels".  Otherwise the six-launches-per-layer path runs.
static bool mega_eligible(enx_ctx* c, uint32_t B, const StepArgs& S, MegaArgs& A, MegaGeometry& geo) {
    const char* env = std::getenv("ENX_DECODE_PATH");
    if (env && std::string(env) == "kernels") return false;
    const enx_model_config& C = c->cfg;
    if ((B != 1 && B != 2 && B != 4) || C.layers > kMaxLayers || C.head_dim % 8 != 0 || C.head_dim > 64 ||
        C.heads / C.kv_heads > 8 || C.hidden > 1024)
        return false;
    std::memset(&A, 0, sizeof(A));
    A.hidden = C.hidden;
    A.heads = C.heads;
    A.kv_heads = C.kv_heads;
    A.head_dim = C.head_dim;
    A.intermediate = C.intermediate;
    A.vocab = C.vocab;
    A.layers = C.layers;
    A.eps = C.rms_norm_eps;
    for (uint32_t l = 0; l < C.layers; ++l) A.layer[l] = c->layers[l];
    A.head = c->head.embed;
    A.head_bits = c->head.bits;
    A.final_norm = c->head.norm;
    A.S = S;
    A.tokens = c->d_step->tokens;
    if (!c->d_ll) {  // tagged stage outputs, zero tags (never a live tag: epochs start at 1)
        const size_t words = mega_ll_words(kMegaMaxTokens, C.hidden, C.kv_heads * C.head_dim, C.intermediate);
        if (dalloc(&c->d_ll, words, "tagged stage outputs") != ENX_OK ||
            cudaMemsetAsync(c->d_ll, 0, words * 8, c->stream) != cudaSuccess) {
            dfree(c->d_ll);
            return false;
        }
    }
    A.ll = c->d_ll;
    A.ll_epoch = reinterpret_cast<const uint32_t*>(c->d_bar);
    A.err = &c->d_step->err;
    A.trace = c->d_trace;
    if (const char* tc = std::getenv("ENX_TRACE_CTA")) A.trace_cta = (uint32_t)std::atoi(tc);  // default CTA 0
    geo = mega_geometry(B, A);
    if (geo.nslots < 2 || c->max_ctx > geo.max_positions) return false;
    A.nslots = geo.nslots;
    A.slot_bytes = geo.slot_bytes;
    A.x4_floats = geo.x4_floats;
    if (!c->d_table[B]) {
        std::vector<MegaSlice> table;
        std::vector<uint32_t> counts;
        uint32_t stride = 0;
        mega_build_table(B, A, geo, table, counts, stride);
        if (dalloc(&c->d_table[B], table.size(), "mega table") != ENX_OK ||
            dalloc(&c->d_nslices[B], counts.size(), "mega counts") != ENX_OK ||
            cudaMemcpy(c->d_table[B], table.data(), table.size() * sizeof(MegaSlice), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(c->d_nslices[B], counts.data(), counts.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            dfree(c->d_table[B]);
            dfree(c->d_nslices[B]);
            return false;
        }
        c->table_stride[B] = stride;
    }
    A.table = c->d_table[B];
    A.nslices = c->d_nslices[B];
    A.table_stride = c->table_stride[B];
    return true;
}

// A projection of B batched tokens: tensor cores from kTcMinTokens tokens, CUDA cores below.
static cudaError_t proj_b(enx_ctx* c, int bits, const float* x, const QW& w, const float* bias, float* out, uint32_t B,
                          uint32_t stride, cudaStream_t st, bool same_x = false) {
    if (B >= kTcMinTokens && bits == 4 && !codes_of(c, w)) return cudaErrorInvalidValue;  // never prepared
    if (B >= kTcMinTokens)
        return launch_gemm_tc(bits, x, w.cols, w, bits == 4 ? codes_of(c, w) : nullptr, bias, out, B, stride, 0, c->b_ws,
                              c->d_bb + c->bl.err(), st, same_x);
    return launch_matmul(bits, x, w, bias, out, B, stride, 0, st, false);
}

// One batched decode step of sequences 0..B-1 (each at its own position) as graph nodes: embed,
// per layer RMSNorm, q|k|v projections, RoPE + cache rows, attention over each sequence's cache,
// o projection + residual, RMSNorm, gate/up, SiLU, down + residual; final norm, tied head and the
// batched sampler.  The reference runs each sequence through the same per-token step.
static cudaError_t batch_body(enx_ctx* c, uint32_t B, cudaStream_t st) {
    const enx_model_config& C = c->cfg;
    const uint32_t H = C.hidden, kvd = C.kv_heads * C.head_dim, I = C.intermediate;
    uint32_t* blk = c->d_bb;
    StepArgs S = step_args(c);
    S.q = c->b_q;
    S.scores = c->b_scores;
    S.score_stride = split_stride(c->max_ctx);
    S.attn_part = c->b_part;
    S.pos = blk + c->bl.pos();
    cudaError_t e = launch_embed(blk + c->bl.tok(), c->head.embed, c->head.bits, c->b_x, B, 0, C.vocab, H, st, false);
    for (uint32_t l = 0; l < C.layers && e == cudaSuccess; ++l) {
        const LayerArgs& L = c->layers[l];
        e = launch_rmsnorm(c->b_x, L.norm_in, c->b_xn, B, H, C.rms_norm_eps, st);
        const bool stk = B >= kTcMinTokens && l < c->stacked.size();  // one GEMM over q|k|v, one over gate|up
        if (e == cudaSuccess && stk) e = proj_qkv(c, l, c->b_xn, c->b_q, c->b_k, c->b_v, B, c->b_ws, c->d_bb + c->bl.err(), st);
        if (e == cudaSuccess && !stk) e = proj_b(c, 4, c->b_xn, L.wq, L.bq, c->b_q, B, H, st);
        if (e == cudaSuccess && !stk) e = proj_b(c, 4, c->b_xn, L.wk, L.bk, c->b_k, B, kvd, st, true);  // limbs of b_xn reused
        if (e == cudaSuccess && !stk) e = proj_b(c, 4, c->b_xn, L.wv, L.bv, c->b_v, B, kvd, st, true);
        if (e == cudaSuccess) e = launch_rope_cache_batch(S, l, c->b_q, c->b_k, c->b_v, B, st);
        if (e == cudaSuccess) e = launch_attn(S, l, B, c->b_att, st, false);
        const bool tc = B >= kTcMinTokens && codes_of(c, L.wo);
        if (e == cudaSuccess) e = proj_add(c, c->b_att, L.wo, c->b_x, c->b_t, B, H, st, tc, c->b_ws, c->d_bb + c->bl.err());
        if (e == cudaSuccess) e = launch_rmsnorm(c->b_x, L.norm_post, c->b_xn, B, H, C.rms_norm_eps, st);
        if (e == cudaSuccess && stk) e = proj_gu(c, l, c->b_xn, c->b_g, c->b_u, B, c->b_ws, c->d_bb + c->bl.err(), st);
        if (e == cudaSuccess && !stk) e = proj_b(c, 4, c->b_xn, L.wg, nullptr, c->b_g, B, I, st);
        if (e == cudaSuccess && !stk) e = proj_b(c, 4, c->b_xn, L.wu, nullptr, c->b_u, B, I, st, true);
        if (e == cudaSuccess) e = launch_silu_mul(c->b_g, c->b_u, c->b_g, B * I, st);
        if (e == cudaSuccess) e = proj_add(c, c->b_g, L.wd, c->b_x, c->b_t, B, H, st, tc, c->b_ws, c->d_bb + c->bl.err());
    }
    if (e == cudaSuccess) e = launch_rmsnorm(c->b_x, c->head.norm, c->normed, B, H, C.rms_norm_eps, st);
    if (e == cudaSuccess) e = proj_b(c, c->head.bits, c->normed, c->head.embed, nullptr, c->logits, B, C.vocab, st);
    if (e == cudaSuccess)
        e = launch_sample(c->logits, C.vocab, B, c->history, c->max_ctx, blk + c->bl.hist(),
                          reinterpret_cast<const SampleRow*>(blk + c->bl.rows()), false, SampleRow{}, blk + c->bl.out(), st,
                          false);
    return e;
}

// The batched step body once, outside any graph, with events between its sections; adds each
// section's time (ms) to ms[k]: 0 embed, 1 RMSNorms, 2 q|k|v GEMMs, 3 RoPE + cache rows,
// 4 attention, 5 o GEMM + residual, 6 gate/up GEMMs + SiLU, 7 down GEMM + residual, 8 head GEMM,
// 9 sampler.  It reruns the last step's rows (same cache rows and logits).
static enx_status batch_profile(enx_ctx* c, uint32_t B, float* ms, uint32_t count) {
    const enx_model_config& C = c->cfg;
    const uint32_t H = C.hidden, kvd = C.kv_heads * C.head_dim, I = C.intermediate;
    cudaStream_t st = c->stream;
    uint32_t* blk = c->d_bb;
    StepArgs S = step_args(c);
    S.q = c->b_q;
    S.scores = c->b_scores;
    S.score_stride = split_stride(c->max_ctx);
    S.attn_part = c->b_part;
    S.pos = blk + c->bl.pos();
    cudaEvent_t ev[2];
    ENX_CUDA(cudaEventCreate(&ev[0]));
    ENX_CUDA(cudaEventCreate(&ev[1]));
    auto section = [&](int k, auto&& work) -> cudaError_t {
        cudaEventRecord(ev[0], st);
        cudaError_t e = work();
        cudaEventRecord(ev[1], st);
        cudaEventSynchronize(ev[1]);
        float t = 0.f;
        cudaEventElapsedTime(&t, ev[0], ev[1]);
        ms[k] += t;
        return e;
    };
    cudaError_t e = section(0, [&] { return launch_embed(blk + c->bl.tok(), c->head.embed, c->head.bits, c->b_x, B, 0, C.vocab, H, st, false); });
    for (uint32_t l = 0; l < C.layers && e == cudaSuccess; ++l) {
        const LayerArgs& L = c->layers[l];
        e = section(1, [&] { return launch_rmsnorm(c->b_x, L.norm_in, c->b_xn, B, H, C.rms_norm_eps, st); });
        if (e == cudaSuccess) e = section(2, [&] {
            if (B >= kTcMinTokens && l < c->stacked.size())
                return proj_qkv(c, l, c->b_xn, c->b_q, c->b_k, c->b_v, B, c->b_ws, c->d_bb + c->bl.err(), st);
            cudaError_t r = proj_b(c, 4, c->b_xn, L.wq, L.bq, c->b_q, B, H, st);
            if (r == cudaSuccess) r = proj_b(c, 4, c->b_xn, L.wk, L.bk, c->b_k, B, kvd, st, true);
            return r == cudaSuccess ? proj_b(c, 4, c->b_xn, L.wv, L.bv, c->b_v, B, kvd, st, true) : r;
        });
        if (e == cudaSuccess) e = section(3, [&] { return launch_rope_cache_batch(S, l, c->b_q, c->b_k, c->b_v, B, st); });
        if (e == cudaSuccess) {
            if (count >= 14 && attn_split_path(S, B)) {  // attention stage by stage
                for (int k = 0; k < 4 && e == cudaSuccess; ++k)
                    e = section(10 + k, [&] { return launch_attn(S, l, B, c->b_att, st, false, k); });
                ms[4] = ms[10] + ms[11] + ms[12] + ms[13];
            } else {
                e = section(4, [&] { return launch_attn(S, l, B, c->b_att, st, false); });
            }
        }
        if (e == cudaSuccess) e = section(5, [&] {
            return proj_add(c, c->b_att, L.wo, c->b_x, c->b_t, B, H, st, B >= kTcMinTokens && codes_of(c, L.wo), c->b_ws,
                            c->d_bb + c->bl.err());
        });
        if (e == cudaSuccess) e = section(1, [&] { return launch_rmsnorm(c->b_x, L.norm_post, c->b_xn, B, H, C.rms_norm_eps, st); });
        if (e == cudaSuccess) e = section(6, [&] {
            cudaError_t r = cudaSuccess;
            if (B >= kTcMinTokens && l < c->stacked.size()) {
                r = proj_gu(c, l, c->b_xn, c->b_g, c->b_u, B, c->b_ws, c->d_bb + c->bl.err(), st);
            } else {
                r = proj_b(c, 4, c->b_xn, L.wg, nullptr, c->b_g, B, I, st);
                if (r == cudaSuccess) r = proj_b(c, 4, c->b_xn, L.wu, nullptr, c->b_u, B, I, st, true);
            }
            return r == cudaSuccess ? launch_silu_mul(c->b_g, c->b_u, c->b_g, B * I, st) : r;
        });
        if (e == cudaSuccess) e = section(7, [&] {
            return proj_add(c, c->b_g, L.wd, c->b_x, c->b_t, B, H, st, B >= kTcMinTokens && codes_of(c, L.wd), c->b_ws,
                            c->d_bb + c->bl.err());
        });
    }
    if (e == cudaSuccess) e = section(1, [&] { return launch_rmsnorm(c->b_x, c->head.norm, c->normed, B, H, C.rms_norm_eps, st); });
    if (e == cudaSuccess) e = section(8, [&] { return proj_b(c, c->head.bits, c->normed, c->head.embed, nullptr, c->logits, B, C.vocab, st); });
    if (e == cudaSuccess) e = section(9, [&] {
        return launch_sample(c->logits, C.vocab, B, c->history, c->max_ctx, blk + c->bl.hist(),
                             reinterpret_cast<const SampleRow*>(blk + c->bl.rows()), false, SampleRow{}, blk + c->bl.out(), st,
                             false);
    });
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
    if (e != cudaSuccess) return cuda_fail(e, "batched step profile");
    return ENX_OK;
}

static enx_status capture_batch(enx_ctx* c, uint32_t B, bool loop) {
    cudaStream_t st = c->stream;
    const BatchLayout& Lb = c->bl;
    ENX_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    if (loop) {
        k_batch_loop_prep<<<1, 256, 0, st>>>(c->d_bb, Lb, c->b_rand, c->b_ids, c->history, c->max_ctx, B);
        e = cudaGetLastError();
    } else {
        // this step's inputs: B entries of each array (ids, positions, history lengths, sampling rows)
        const uint32_t offs[3] = {Lb.tok(), Lb.pos(), Lb.hist()};
        for (uint32_t k = 0; k < 3 && e == cudaSuccess; ++k)
            e = cudaMemcpyAsync(c->d_bb + offs[k], c->h_bb + offs[k], (size_t)B * 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->d_bb + Lb.rows(), c->h_bb + Lb.rows(), (size_t)B * 16, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) {
            k_batch_prep<<<1, 256, 0, st>>>(c->d_bb, Lb, c->history, c->max_ctx, B);
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess) e = batch_body(c, B, st);
    if (e == cudaSuccess) {
        if (loop) {
            k_batch_loop_post<<<1, 256, 0, st>>>(c->d_bb, Lb, c->b_ids, B);
            e = cudaGetLastError();
        } else {
            e = cudaMemcpyAsync(c->h_bb + Lb.out(), c->d_bb + Lb.out(), (size_t)B * 4, cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(c->h_bb + Lb.err(), c->d_bb + Lb.err(), 4, cudaMemcpyDeviceToHost, st);
        }
    }
    cudaGraph_t graph = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(st, &graph);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return cuda_fail(e, "capturing the batched decode step");
    }
    size_t nodes = 0;
    cudaGraphGetNodes(graph, nullptr, &nodes);
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "instantiating the batched decode step");
    (loop ? c->b_loop_graph : c->b_graph)[B] = exec;
    c->b_launches[B] = (uint32_t)nodes;
    return ENX_OK;
}

static enx_status batch_error(enx_ctx* c, uint32_t code) {
    c->h_bb[c->bl.err()] = 0;
    cudaMemsetAsync(c->d_bb + c->bl.err(), 0, 4, c->stream);
    return fail(ENX_ERR_TIMEOUT, "batched decode: a bounded device wait gave up (code " + std::to_string(code) + ")");
}

// enx_decode_step for more than kMaxStepBatch sequences.
static enx_status decode_batch(enx_ctx* c, uint32_t B, const uint32_t* tokens, const enx_sampling* params,
                               uint32_t params_count, const float* randoms, uint32_t* out_ids) {
    if (!c->d_bb) return fail(ENX_ERR_STATE, "batched decode: enx_kv_alloc with more than 4 sequences first");
    auto it = c->b_graph.find(B);
    if (it == c->b_graph.end()) {
        ENX_TRY(capture_batch(c, B, false));
        it = c->b_graph.find(B);
    }
    uint32_t* h = c->h_bb;
    const BatchLayout& Lb = c->bl;
    for (uint32_t b = 0; b < B; ++b) {
        const enx_sampling& p = params[params_count == 1 ? 0 : b];
        h[Lb.tok() + b] = tokens[b];
        h[Lb.pos() + b] = c->filled[b];
        h[Lb.hist() + b] = c->filled[b] + 1;
        reinterpret_cast<SampleRow*>(h + Lb.rows())[b] = SampleRow{p.temperature, p.top_p, p.repetition_penalty, randoms[b]};
    }
    ENX_CUDA(cudaGraphLaunch(it->second, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    if (h[Lb.err()]) return batch_error(c, h[Lb.err()]);
    for (uint32_t b = 0; b < B; ++b) {
        out_ids[b] = h[Lb.out() + b];
        c->filled[b] += 1;
    }
    c->last_launches = c->b_launches[B];
    return ENX_OK;
}

// enx_decode_loop for more than kMaxStepBatch sequences.
static enx_status decode_batch_loop(enx_ctx* c, uint32_t B, const uint32_t* first, const enx_sampling* params,
                                    uint32_t params_count, uint32_t steps, const float* randoms, uint32_t* out_ids,
                                    int sync) {
    if (!c->d_bb) return fail(ENX_ERR_STATE, "batched decode: enx_kv_alloc with more than 4 sequences first");
    auto it = c->b_loop_graph.find(B);
    if (it == c->b_loop_graph.end()) {
        ENX_TRY(capture_batch(c, B, true));
        it = c->b_loop_graph.find(B);
    }
    uint32_t* h = c->h_bb;
    const BatchLayout& Lb = c->bl;
    h[Lb.step()] = 0;
    for (uint32_t b = 0; b < B; ++b) {
        const enx_sampling& p = params[params_count == 1 ? 0 : b];
        h[Lb.base() + b] = c->filled[b];
        h[Lb.first() + b] = first[b];
        reinterpret_cast<SampleRow*>(h + Lb.params())[b] = SampleRow{p.temperature, p.top_p, p.repetition_penalty, 0.f};
    }
    ENX_CUDA(cudaMemcpyAsync(c->d_bb + Lb.step(), h + Lb.step(), ((size_t)Lb.words() - Lb.step()) * 4,
                             cudaMemcpyHostToDevice, c->stream));
    ENX_CUDA(cudaMemcpyAsync(c->b_rand, randoms, (size_t)steps * B * 4, cudaMemcpyHostToDevice, c->stream));
    for (uint32_t i = 0; i < steps; ++i) ENX_CUDA(cudaGraphLaunch(it->second, c->stream));
    for (uint32_t b = 0; b < B; ++b) c->filled[b] += steps;
    c->loop_count = steps * B;
    c->last_launches = c->b_launches[B];
    if (!sync) return ENX_OK;
    ENX_CUDA(cudaMemcpyAsync(out_ids, c->b_ids, (size_t)steps * B * 4, cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaMemcpyAsync(h + Lb.err(), c->d_bb + Lb.err(), 4, cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    if (h[Lb.err()]) return batch_error(c, h[Lb.err()]);
    return ENX_OK;
}

// The final RMSNorm and the tied head of a persistent step (after k_mega, which leaves the last
// layer's x in S.x): the tensor-core head for an int8 table (its weight stream starts while k_mega
// drains), the CUDA-core head kernel otherwise.
static cudaError_t launch_step_head(enx_ctx* c, uint32_t B, const StepArgs& S, cudaStream_t st) {
    if (c->head.bits == 8 && c->cfg.hidden % 128 == 0 && c->cfg.hidden <= 1024) {
        HeadTcArgs h{};
        h.x = c->x;
        h.gain = c->head.norm;
        h.eps = c->cfg.rms_norm_eps;
        h.normed_out = c->normed;
        h.w = c->head.embed;
        h.out = c->logits;
        h.out_stride = c->cfg.vocab;
        h.ntok = B;
        h.err = &c->d_step->err;
        return launch_head_tc(h, st, true);
    }
    return launch_head(B, c->head.bits, c->head, S, st);
}

// Decode-loop steps per graph launch (the rest of a loop runs one-step graphs): consecutive steps
// inside one graph start without a graph launch between them.
constexpr uint32_t kLoopGraphSteps = 8;

// Captures the decode step of B sequences (loop: the device-fed loop step) as a CUDA graph; reps
// loop steps one after another in one graph when reps > 1.
static enx_status capture_step(enx_ctx* c, uint32_t B, bool loop, uint32_t reps = 1) {
    cudaStream_t st = c->stream;
    StepArgs S = step_args(c);
    S.pos = c->d_step->pos;
    const size_t in_bytes = offsetof(StepBlock, out);
    // decided (and the slice table uploaded) before capture: no synchronous copies inside it
    MegaArgs A;
    MegaGeometry geo{};
    const bool mega = mega_eligible(c, B, S, A, geo);
    ENX_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    for (uint32_t rep = 0; rep < (loop ? reps : 1u) && e == cudaSuccess; ++rep) {
        if (loop) {
            k_loop_prep<<<1, 32, 0, st>>>(c->d_loop, c->d_step, c->d_loop_rand, c->d_loop_ids, c->history, c->max_ctx, B,
                                          c->d_bar);
            e = cudaGetLastError();
        } else {
            e = cudaMemcpyAsync(c->d_step, c->h_step, in_bytes, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) {
                k_step_prep<<<1, 32, 0, st>>>(c->d_step, c->history, c->max_ctx, B, c->d_bar);
                e = cudaGetLastError();
            }
        }
        if (e == cudaSuccess) {
            if (mega) {
                e = launch_mega(B, A, geo, st);  // the prep kernel above bumped the tag epoch
                if (e == cudaSuccess) e = launch_step_head(c, B, S, st);
            } else {
                e = launch_embed(c->d_step->tokens, c->head.embed, c->head.bits, c->x, B, 0, c->cfg.vocab, c->cfg.hidden,
                                 st, true);
                for (uint32_t l = 0; l < c->cfg.layers && e == cudaSuccess; ++l) e = launch_layer(B, c->layers[l], S, st);
                if (e == cudaSuccess) e = launch_head(B, c->head.bits, c->head, S, st);
            }
        }
        (loop ? c->loop_mega : c->graph_mega)[B] = mega;
        if (e == cudaSuccess)
            e = launch_sample(c->logits, c->cfg.vocab, B, c->history, c->max_ctx, c->d_step->hist_len, c->d_step->rows,
                              false, SampleRow{}, c->d_step->out, st, true);
        if (e == cudaSuccess) {
            if (loop) {
                k_loop_post<<<1, 32, 0, st>>>(c->d_loop, c->d_step, c->d_loop_ids, B);
                e = cudaGetLastError();
            } else {
                // the ids and the sticky error word travel back together
                e = cudaMemcpyAsync(c->h_step->out, c->d_step->out, sizeof(StepBlock) - offsetof(StepBlock, out),
                                    cudaMemcpyDeviceToHost, st);
            }
        }
    }
    cudaGraph_t graph = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return cuda_fail(e, "capturing the decode step");
    }
    if (e2 != cudaSuccess) return cuda_fail(e2, "cudaStreamEndCapture");
    size_t nn = 0;
    cudaGraphGetNodes(graph, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    cudaGraphGetNodes(graph, nodes.data(), &nn);
    uint32_t kernels = 0;
    for (auto& nd : nodes) {
        cudaGraphNodeType t;
        cudaGraphNodeGetType(nd, &t);
        if (t == cudaGraphNodeTypeKernel) ++kernels;
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate(decode step)");
    if (loop && reps > 1) {
        c->loop_graph_n[B] = exec;
        return ENX_OK;
    }
    (loop ? c->loop_graph : c->graph)[B] = exec;
    (loop ? c->loop_launches : c->graph_launches)[B] = kernels;
    return ENX_OK;
}

extern "C" enx_status enx_decode_step(enx_ctx* c, uint32_t batch, const uint32_t* tokens,
                                      const enx_sampling* params, uint32_t params_count,
                                      const float* randoms, uint32_t* out_ids) {
    CHECK_ARG(c && tokens && params && randoms && out_ids, "enx_decode_step: null pointer");
    if (!c->loaded) return fail(ENX_ERR_STATE, "enx_decode_step: no model loaded");
    if (!c->kcache) return fail(ENX_ERR_STATE, "enx_decode_step: call enx_kv_alloc first");
    if (batch == 0) return ENX_OK;
    if (batch > c->batch) return fail(ENX_ERR_RANGE, "enx_decode_step: batch exceeds the allocated sequences");
    CHECK_ARG(params_count == 1 || params_count == batch, "enx_decode_step: params_count must be 1 or batch");
    for (uint32_t b = 0; b < batch; ++b) {
        if (tokens[b] >= c->cfg.vocab) return fail(ENX_ERR_INVALID, "token id outside the vocabulary");
        if (c->filled[b] >= c->max_ctx)
            return fail(ENX_ERR_RANGE, "context exhausted: " + std::to_string(c->filled[b]) + " + 1 exceeds " +
                                           std::to_string(c->max_ctx));
    }
    DeviceGuard g(c->device);
    if (batch > kMaxStepBatch) return decode_batch(c, batch, tokens, params, params_count, randoms, out_ids);
    if (!c->graph[batch]) ENX_TRY(capture_step(c, batch, false));
    StepBlock* h = c->h_step;
    for (uint32_t b = 0; b < batch; ++b) {
        const enx_sampling& p = params[params_count == 1 ? 0 : b];
        h->tokens[b] = tokens[b];
        h->pos[b] = c->filled[b];
        h->hist_len[b] = c->filled[b] + 1;  // the fed token joins the history before sampling
        h->rows[b] = SampleRow{p.temperature, p.top_p, p.repetition_penalty, randoms[b]};
    }
    ENX_CUDA(cudaGraphLaunch(c->graph[batch], c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    if (h->err) {
        const uint32_t code = h->err;
        h->err = 0;
        cudaMemsetAsync(&c->d_step->err, 0, 4, c->stream);
        return timeout_error("enx_decode_step", code);
    }
    for (uint32_t b = 0; b < batch; ++b) {
        out_ids[b] = h->out[b];
        c->filled[b] += 1;
    }
    c->last_launches = c->graph_launches[batch];
    return ENX_OK;
}

static enx_status device_error(enx_ctx* c, const char* caller);

extern "C" enx_status enx_decode_loop(enx_ctx* c, uint32_t batch, const uint32_t* first_tokens,
                                      const enx_sampling* params, uint32_t params_count, uint32_t steps,
                                      const float* randoms, uint32_t* out_ids, int sync) {
    CHECK_ARG(c && first_tokens && params && randoms, "enx_decode_loop: null pointer");
    CHECK_ARG(!sync || out_ids, "enx_decode_loop: sync without out_ids");
    if (!c->loaded) return fail(ENX_ERR_STATE, "enx_decode_loop: no model loaded");
    if (!c->kcache) return fail(ENX_ERR_STATE, "enx_decode_loop: call enx_kv_alloc first");
    if (batch == 0 || steps == 0) return ENX_OK;
    if (batch > c->batch) return fail(ENX_ERR_RANGE, "enx_decode_loop: batch too large");
    CHECK_ARG(params_count == 1 || params_count == batch, "enx_decode_loop: params_count must be 1 or batch");
    for (uint32_t b = 0; b < batch; ++b) {
        if (first_tokens[b] >= c->cfg.vocab) return fail(ENX_ERR_INVALID, "token id outside the vocabulary");
        if ((uint64_t)c->filled[b] + steps > c->max_ctx)
            return fail(ENX_ERR_RANGE, "context exhausted: " + std::to_string(c->filled[b]) + " + " +
                                           std::to_string(steps) + " exceeds " + std::to_string(c->max_ctx));
    }
    DeviceGuard g(c->device);
    c->loop_batched = batch > kMaxStepBatch;
    if (batch > kMaxStepBatch)
        return decode_batch_loop(c, batch, first_tokens, params, params_count, steps, randoms, out_ids, sync);
    if (!c->loop_graph[batch]) ENX_TRY(capture_step(c, batch, true));
    if (steps >= kLoopGraphSteps && !c->loop_graph_n[batch]) ENX_TRY(capture_step(c, batch, true, kLoopGraphSteps));
    ENX_CUDA(cudaStreamSynchronize(c->stream));  // the pinned loop state may still be in flight
    LoopState* L = c->h_loop;
    L->i = 0;
    for (uint32_t b = 0; b < batch; ++b) {
        const enx_sampling& p = params[params_count == 1 ? 0 : b];
        L->base_pos[b] = c->filled[b];
        L->first[b] = first_tokens[b];
        L->params[b] = SampleRow{p.temperature, p.top_p, p.repetition_penalty, 0.f};
    }
    ENX_CUDA(cudaMemcpyAsync(c->d_loop, L, sizeof(LoopState), cudaMemcpyHostToDevice, c->stream));
    ENX_CUDA(cudaMemcpyAsync(c->d_loop_rand, randoms, (size_t)steps * batch * 4, cudaMemcpyHostToDevice, c->stream));
    uint32_t i = 0;
    for (; i + kLoopGraphSteps <= steps && c->loop_graph_n[batch]; i += kLoopGraphSteps)
        ENX_CUDA(cudaGraphLaunch(c->loop_graph_n[batch], c->stream));
    for (; i < steps; ++i) ENX_CUDA(cudaGraphLaunch(c->loop_graph[batch], c->stream));
    ENX_CUDA(cudaMemcpyAsync(c->h_loop_ids, c->d_loop_ids, (size_t)steps * batch * 4, cudaMemcpyDeviceToHost,
                             c->stream));
    for (uint32_t b = 0; b < batch; ++b) c->filled[b] += steps;
    c->loop_count = steps * batch;
    c->last_launches = c->loop_launches[batch];
    if (sync) {
        ENX_CUDA(cudaStreamSynchronize(c->stream));
        ENX_TRY(device_error(c, "enx_decode_loop"));
        std::memcpy(out_ids, c->h_loop_ids, (size_t)steps * batch * 4);
    }
    return ENX_OK;
}

// Reads (and clears) the sticky device error word after the stream has drained.
static enx_status device_error(enx_ctx* c, const char* caller) {
    uint32_t code = 0;
    ENX_CUDA(cudaMemcpy(&code, &c->d_step->err, 4, cudaMemcpyDeviceToHost));
    if (!code) return ENX_OK;
    ENX_CUDA(cudaMemset(&c->d_step->err, 0, 4));
    return timeout_error(caller, code);
}

extern "C" enx_status enx_synchronize(enx_ctx* c) {
    CHECK_ARG(c, "enx_synchronize: null context");
    DeviceGuard g(c->device);
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    if (c->d_bb) {
        uint32_t code = 0;
        ENX_CUDA(cudaMemcpy(&code, c->d_bb + c->bl.err(), 4, cudaMemcpyDeviceToHost));
        if (code) return batch_error(c, code);
    }
    return c->d_step ? device_error(c, "enx_synchronize") : ENX_OK;
}

extern "C" enx_status enx_loop_ids(enx_ctx* c, uint32_t* out_ids, uint32_t count) {
    CHECK_ARG(c && out_ids, "enx_loop_ids: null pointer");
    if (count > c->loop_count) return fail(ENX_ERR_RANGE, "enx_loop_ids: more ids than the last loop produced");
    if (c->loop_batched) {  // the batched loop leaves its ids on the device
        DeviceGuard g(c->device);
        ENX_CUDA(cudaMemcpyAsync(out_ids, c->b_ids, (size_t)count * 4, cudaMemcpyDeviceToHost, c->stream));
        ENX_CUDA(cudaStreamSynchronize(c->stream));
        return ENX_OK;
    }
    std::memcpy(out_ids, c->h_loop_ids, (size_t)count * 4);
    return ENX_OK;
}

extern "C" enx_status enx_logits(enx_ctx* c, uint32_t seq, float* out) {
    CHECK_ARG(c && out, "enx_logits: null pointer");
    if (!c->logits || seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_logits: sequence outside the cache");
    DeviceGuard g(c->device);
    ENX_CUDA(cudaMemcpyAsync(out, c->logits + (size_t)seq * c->cfg.vocab, (size_t)c->cfg.vocab * 4,
                             cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return ENX_OK;
}

extern "C" enx_status enx_nll(enx_ctx* c, uint32_t seq, uint32_t target, double* out) {
    CHECK_ARG(c && out, "enx_nll: null pointer");
    if (!c->logits || seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_nll: sequence outside the cache");
    if (target >= c->cfg.vocab) return fail(ENX_ERR_INVALID, "enx_nll: target id outside the vocabulary");
    DeviceGuard g(c->device);
    ENX_CUDA(launch_nll(c->logits + (size_t)seq * c->cfg.vocab, c->cfg.vocab, target, c->d_nll, c->stream));
    ENX_CUDA(cudaMemcpyAsync(out, c->d_nll, 8, cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return ENX_OK;
}

extern "C" enx_status enx_hidden(enx_ctx* c, uint32_t seq, float* out) {
    CHECK_ARG(c && out, "enx_hidden: null pointer");
    if (!c->normed || seq >= c->batch) return fail(ENX_ERR_RANGE, "enx_hidden: sequence outside the cache");
    DeviceGuard g(c->device);
    ENX_CUDA(cudaMemcpyAsync(out, c->normed + (size_t)seq * c->cfg.hidden, (size_t)c->cfg.hidden * 4,
                             cudaMemcpyDeviceToHost, c->stream));
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return ENX_OK;
}

extern "C" enx_status enx_kv_view(enx_ctx* c, uint32_t seq, uint32_t layer, const uint16_t** k, const uint16_t** v) {
    CHECK_ARG(c && k && v, "enx_kv_view: null pointer");
    if (!c->kcache || seq >= c->batch || layer >= c->cfg.layers) return fail(ENX_ERR_RANGE, "enx_kv_view: out of range");
    StepArgs S = step_args(c);
    *k = c->kcache + S.cache_offset(seq, layer, 0);
    *v = c->vcache + S.cache_offset(seq, layer, 0);
    return ENX_OK;
}

extern "C" enx_status enx_tensor_view(enx_ctx* c, const char* name, int32_t* bits, uint32_t* rows, uint32_t* cols,
                                      const void** packed, const float** scales, const uint32_t** zeros) {
    CHECK_ARG(c && name && bits && rows && cols && packed && scales && zeros, "enx_tensor_view: null pointer");
    auto it = c->tensors.find(name);
    if (it == c->tensors.end()) return fail(ENX_ERR_INVALID, std::string("no tensor ") + name);
    const Tensor& t = it->second;
    *bits = t.bits;
    *rows = t.rows;
    *cols = t.cols;
    *packed = t.packed;
    *scales = t.scales;
    *zeros = t.zeros;
    return ENX_OK;
}

extern "C" enx_status enx_set_tracing(enx_ctx* c, int on) {
    CHECK_ARG(c, "enx_set_tracing: null context");
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    free_graphs(c);
    dfree(c->d_trace);
    c->trace_len = 0;
    if (on) {
        c->trace_len = 3 * (kMegaStages * c->cfg.layers + 1) + kMegaTraceDetail * c->cfg.layers + 2;
        ENX_TRY(dalloc(&c->d_trace, c->trace_len, "trace"));
        ENX_CUDA(cudaMemset(c->d_trace, 0, (size_t)c->trace_len * 8));
    }
    return ENX_OK;
}

extern "C" enx_status enx_trace(enx_ctx* c, uint64_t* out, uint32_t capacity, uint32_t* count) {
    CHECK_ARG(c && out && count, "enx_trace: null pointer");
    if (!c->d_trace) return fail(ENX_ERR_STATE, "enx_trace: tracing is off");
    DeviceGuard g(c->device);
    const uint32_t n = capacity < c->trace_len ? capacity : c->trace_len;
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    ENX_CUDA(cudaMemcpy(out, c->d_trace, (size_t)n * 8, cudaMemcpyDeviceToHost));
    *count = n;
    return ENX_OK;
}

extern "C" enx_status enx_stream(enx_ctx* c, void** stream) {
    CHECK_ARG(c && stream, "enx_stream: null pointer");
    *stream = c->stream;
    return ENX_OK;
}

extern "C" enx_status enx_step_launches(enx_ctx* c, uint32_t* launches) {
    CHECK_ARG(c && launches, "enx_step_launches: null pointer");
    *launches = c->last_launches;
    return ENX_OK;
}

extern "C" enx_status enx_launch_step_kernel(enx_ctx* c, uint32_t batch, uint32_t count) {
    CHECK_ARG(c, "enx_launch_step_kernel: null context");
    if (batch == 0 || batch > kMaxStepBatch || !c->d_step || !(c->graph_mega[batch] || c->loop_mega[batch]))
        return fail(ENX_ERR_STATE, "enx_launch_step_kernel: no decode step of this batch ran on the persistent kernel");
    DeviceGuard g(c->device);
    StepArgs S = step_args(c);
    S.pos = c->d_step->pos;
    MegaArgs A;
    MegaGeometry geo{};
    if (!mega_eligible(c, batch, S, A, geo)) return fail(ENX_ERR_STATE, "enx_launch_step_kernel: not eligible");
    for (uint32_t i = 0; i < count; ++i) {
        k_bump_epoch<<<1, 32, 0, c->stream>>>(c->d_bar);
        ENX_CUDA(cudaGetLastError());
        ENX_CUDA(launch_mega(batch, A, geo, c->stream));
        ENX_CUDA(launch_step_head(c, batch, S, c->stream));
    }
    return ENX_OK;
}

extern "C" enx_status enx_batch_profile(enx_ctx* c, uint32_t batch, float* ms, uint32_t count) {
    CHECK_ARG(c && ms && count >= 10, "enx_batch_profile: need room for 10 section times");
    if (!c->d_bb || batch <= kMaxStepBatch || batch > c->batch)
        return fail(ENX_ERR_STATE, "enx_batch_profile: needs a batched context and a batch above 4");
    DeviceGuard g(c->device);
    for (uint32_t i = 0; i < count; ++i) ms[i] = 0.f;
    ENX_CUDA(cudaStreamSynchronize(c->stream));
    return batch_profile(c, batch, ms, count);
}
