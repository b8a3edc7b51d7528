// Argument blocks and launchers of the decode kernels (k_decode.cu).
#pragma once

#include "k_matvec.cuh"

namespace enx {

constexpr uint32_t kAttnChunk = 64;  // positions per attention-score split
constexpr uint32_t kAttnSplit = 128; // positions per scores split (many-token attention)
constexpr uint32_t kApplySplit = 512; // positions per weighted-V split: attn_part holds at most
                                      // score_stride / kAttnSplit splits, more than it needs

// Buffers and geometry of one decode step (shared by every layer of the step).
struct StepArgs {
    uint32_t hidden, heads, kv_heads, head_dim, intermediate;
    float eps;
    float* x;              // [MT][hidden] residual stream
    float* q;              // [MT][hidden] rotated queries
    float* gated;          // [MT][intermediate]
    float* logits;         // [MT][vocab]
    float* normed;         // [MT][hidden] final-norm output
    float* scores;         // [MT][heads][score_stride] attention scores (workspace)
    float* attn_out;       // [MT][hidden] attention output
    uint32_t score_stride; // >= positions attended (a multiple of kAttnChunk)
    double* attn_part;     // [MT][score_stride/kAttnSplit][heads][head_dim] split partial sums, or null
    const uint32_t* pos;   // [MT] position written this step (device), or null: pos_base + t
    uint32_t pos_base;
    uint32_t seq_fixed;    // sequence of every token, or 0xFFFFFFFF: token t is sequence t
    const double* rope_cos;  // [max_context][head_dim/2], f64 (the reference's rotation precision)
    const double* rope_sin;
    uint16_t* kcache;      // f16 bits, [seq][layer][max_context][kv_heads*head_dim]
    uint16_t* vcache;
    uint32_t layers, max_context;

    __host__ __device__ uint32_t pos_of(uint32_t t) const { return pos ? pos[t] : pos_base + t; }
    __host__ __device__ uint32_t seq_of(uint32_t t) const { return seq_fixed == 0xFFFFFFFFu ? t : seq_fixed; }
    __host__ __device__ size_t cache_offset(uint32_t seq, uint32_t layer, uint32_t p) const {
        return (((size_t)seq * layers + layer) * max_context + p) * (size_t)(kv_heads * head_dim);
    }
};

struct LayerArgs {
    uint32_t layer;
    const float* norm_in;
    const float* norm_post;
    QW wq, wk, wv, wo, wg, wu, wd;
    const float* bq;
    const float* bk;
    const float* bv;
};

struct HeadArgs {
    QW embed;
    int bits;
    const float* norm;
};

// RoPE of one pair in the reference's arithmetic (test/reference/ops.ts:103-109): f64 products
// rounded separately (no fused multiply-add), one rounding to float.
__device__ __forceinline__ void rope_pair(float& a, float& b, double c, double s) {
    const double da = a, db = b;
    const float ra = (float)__dsub_rn(__dmul_rn(da, c), __dmul_rn(db, s));
    const float rb = (float)__dadd_rn(__dmul_rn(db, c), __dmul_rn(da, s));
    a = ra;
    b = rb;
}

// SiLU(g) * u in double, rounded once (test/reference/ops.ts:207-216).
__device__ __forceinline__ float silu_mul_value(float g, float u) {
    const double gd = g;
    return (float)__dmul_rn(__ddiv_rn(gd, __dadd_rn(1.0, exp(-gd))), (double)u);
}

int num_sms();
cudaError_t launch_embed(const uint32_t* ids, const QW& table, int bits, float* out, uint32_t seq,
                         uint32_t row_begin, uint32_t row_count, uint32_t out_stride,
                         cudaStream_t st, bool pdl);
cudaError_t launch_matmul(int bits, const float* x, const QW& w, const float* bias, float* out,
                          uint32_t m, uint32_t out_stride, uint32_t out_offset, cudaStream_t st,
                          bool pdl);
cudaError_t launch_layer(uint32_t mt, const LayerArgs& L, const StepArgs& S, cudaStream_t st);
cudaError_t launch_head(uint32_t mt, int bits, const HeadArgs& Hd, const StepArgs& S, cudaStream_t st);
// Attention of `ntok` queries (S.q rows) over the cache: scores into S.scores, then softmax and
// V into `out` [ntok][hidden].  Used by the layer path, prefill and the raw entry points.
// `only` >= 0 launches one stage (0 scores, 1 softmax rows, 2 weighted V, 3 combine), for timing.
cudaError_t launch_attn(const StepArgs& S, uint32_t layer, uint32_t ntok, float* out, cudaStream_t st, bool pdl,
                        int only = -1);
bool attn_split_path(const StepArgs& S, uint32_t ntok);
// Batched decode: RoPE of q (in place) and k, and k/v into each token's own cache row (token t is
// sequence t at position S.pos_of(t)).
cudaError_t launch_rope_cache_batch(const StepArgs& S, uint32_t layer, float* q, const float* k, const float* v,
                                    uint32_t B, cudaStream_t st);

}  // namespace enx
