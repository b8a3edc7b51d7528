// Decode-shaped kernels: the int4 projections with their fused prologues/epilogues, the int8
// tied head, the embedding gather, and split-history decode attention over the f16 cache.
//
// One decoder layer of one step is five launches (the reference issues 19 dispatches,
// src/model/graph_decode.ts:268-358):
//   k_qkv     RMSNorm prologue + q|k|v projections + bias + RoPE + f16 cache append
//   k_attn    scores, softmax and V-apply for one (kv head, 64-position split) per CTA
//   k_oproj   merge of the split partials + o projection + residual add
//   k_gateup  RMSNorm prologue + gate|up projections + SiLU*up
//   k_down    down projection + residual add
// and the step ends with k_head (final RMSNorm + int8 tied head).  Every kernel starts with
// griddepcontrol.launch_dependents and waits (griddepcontrol.wait) only after it has issued the
// L2 prefetch of its own weights, so under programmatic dependent launch the weight stream of
// kernel N+1 overlaps kernel N.
//
// MT (1..4) tokens per launch: batch-1 decode is MT = 1; a batch of up to 4 sequences shares one
// pass over the weights.

#include "k_matvec.cuh"
#include "k_decode.cuh"

namespace enx {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    // cp.async.bulk.prefetch wants a 16-byte aligned address and a multiple of 16 bytes.
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    uintptr_t b = a & ~uintptr_t(15);
    uint32_t n = (uint32_t)(((a + bytes + 15) & ~uintptr_t(15)) - b);
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
}

template <int BITS>
__device__ __forceinline__ void prefetch_row(const QW& w, uint32_t row) {
    uint32_t bytes = w.cols * BITS / 8;
    prefetch_l2(reinterpret_cast<const char*>(w.packed) + (size_t)row * bytes, bytes);
}

// ---------------------------------------------------------------------------------------------
// embedding gather (embed_gather_q8 / _q4, src/kernels/embedding_variants.ts:291-317)

template <int BITS>
__global__ void k_embed(const uint32_t* __restrict__ ids, QW table, float* __restrict__ out,
                        uint32_t row_begin, uint32_t row_count, uint32_t out_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t s = blockIdx.y;
    const uint32_t id = ids[s];
    if (id < row_begin || id >= row_begin + row_count) return;
    const uint32_t row = id - row_begin;
    const uint32_t K = table.cols, bpr = K / kBlock;
    for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < K; c += gridDim.x * blockDim.x) {
        size_t flat = (size_t)row * K + c;
        uint32_t q = BITS == 4 ? (table.packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu
                               : (table.packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
        uint32_t blk = row * bpr + c / kBlock;
        float z = (float)zero_code<BITS>(table.zeros, blk);
        out[(size_t)s * out_stride + c] = ((float)q - z) * table.scales[blk];
    }
}

// ---------------------------------------------------------------------------------------------
// generic projection (raw enx_matmul_q4 / enx_lm_head_q8 entry points)

template <int BITS, int MT>
__global__ void __launch_bounds__(kThreads) k_matmul(const float* __restrict__ x, QW w,
                                                     const float* __restrict__ bias,
                                                     float* __restrict__ out, uint32_t m,
                                                     uint32_t out_stride, uint32_t out_offset) {
    extern __shared__ float4 X4[];
    const uint32_t K = w.cols, N = w.rows, nchunk = K / Geom<BITS>::E;
    const uint32_t t0 = blockIdx.y * MT;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    // rows t0.. beyond m read a clamped row: results for them are not written
    {
        constexpr int E = Geom<BITS>::E, F4 = Geom<BITS>::F4;
        const uint32_t n4 = K / 4;
        for (uint32_t i = threadIdx.x; i < MT * n4; i += blockDim.x) {
            uint32_t t = i / n4, e4 = i % n4;
            uint32_t src = min(t0 + t, m - 1);
            float4 v = reinterpret_cast<const float4*>(x + (size_t)src * K)[e4];
            X4[(t * F4 + e4 % F4) * nchunk + (e4 * 4) / E] = v;
        }
        __syncthreads();
    }
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < N; r0 += gridDim.x * kWarps * 2) {
        uint32_t rows[2] = {r0, min(r0 + 1, N - 1)};
        float acc[2][MT] = {};
        dot_rows<BITS, MT, 2>(w, rows, X4, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
        if (lane < MT && t0 + lane < m) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && r0 + 1 >= N) break;
                float v = 0.f;
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t == lane) v = acc[r][t];
                if (bias) v += bias[rows[r]];
                out[(size_t)(t0 + lane) * out_stride + out_offset + rows[r]] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// fused decode stages

// Concatenated q|k|v row space: head slot hs in [0, heads + 2*kv_heads).  A work item is a RoPE
// pair (i, i + hd/2) of one head slot, so the rotation is done in registers.
template <int MT>
__global__ void __launch_bounds__(kThreads) k_qkv(LayerArgs L, StepArgs S) {
    extern __shared__ float4 X4[];
    __shared__ float rs[MT], red[kWarps];
    const uint32_t H = S.hidden, hd = S.head_dim, half = hd / 2;
    const uint32_t slots = S.heads + 2 * S.kv_heads;
    const uint32_t items = slots * half;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    // weights first: they do not depend on the previous kernel
    for (uint32_t it = blockIdx.x * kWarps + warp; it < items; it += gridDim.x * kWarps) {
        if (lane < 2) {
            uint32_t hs = it / half, i = it % half;
            const QW& w = hs < S.heads ? L.wq : hs < S.heads + S.kv_heads ? L.wk : L.wv;
            uint32_t base = hs < S.heads ? hs * hd : hs < S.heads + S.kv_heads ? (hs - S.heads) * hd
                                                                                : (hs - S.heads - S.kv_heads) * hd;
            prefetch_row<4>(w, base + i + lane * half);
        }
    }
    pdl_wait();
    rms_scale<MT>(rs, red, S.x, H, S.eps);
    stage_x<4, MT>(X4, S.x, H, rs, L.norm_in);
    const uint32_t nchunk = H / 32;
    for (uint32_t it = blockIdx.x * kWarps + warp; it < items; it += gridDim.x * kWarps) {
        const uint32_t hs = it / half, i = it % half;
        int kind;  // 0 q, 1 k, 2 v
        uint32_t head;
        if (hs < S.heads) { kind = 0; head = hs; }
        else if (hs < S.heads + S.kv_heads) { kind = 1; head = hs - S.heads; }
        else { kind = 2; head = hs - S.heads - S.kv_heads; }
        const QW& w = kind == 0 ? L.wq : kind == 1 ? L.wk : L.wv;
        const float* bias = kind == 0 ? L.bq : kind == 1 ? L.bk : L.bv;
        uint32_t rows[2] = {head * hd + i, head * hd + i + half};
        float acc[2][MT] = {};
        dot_rows<4, MT, 2>(w, rows, X4, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
        if (lane < MT) {
            float a = 0.f, b = 0.f;
#pragma unroll
            for (int t = 0; t < MT; ++t)
                if (t == lane) { a = acc[0][t]; b = acc[1][t]; }
            if (bias) { a += bias[rows[0]]; b += bias[rows[1]]; }
            const uint32_t pos = S.pos_of(lane);
            if (kind != 2) {  // RoPE, half rotation (src/kernels/rope.wgsl:42-52)
                float c = S.rope_cos[(size_t)pos * half + i], sn = S.rope_sin[(size_t)pos * half + i];
                float ra = a * c - b * sn, rb = b * c + a * sn;
                a = ra; b = rb;
            }
            if (kind == 0) {
                S.q[(size_t)lane * H + rows[0]] = a;
                S.q[(size_t)lane * H + rows[1]] = b;
            } else {
                uint16_t* cache = (kind == 1 ? S.kcache : S.vcache) + S.cache_offset(S.seq_of(lane), L.layer, pos);
                cache[head * hd + i] = __half_as_ushort(__float2half_rn(a));
                cache[head * hd + i + half] = __half_as_ushort(__float2half_rn(b));
            }
        }
    }
}

// Split-history decode attention.  grid = (kv_heads, splits, MT).  The CTA covers positions
// [split*64, split*64+64) of its token, all `group` query heads of its kv head, and writes an
// unnormalised partial (acc[hd], max, sum) per head.
template <int MT>
__global__ void __launch_bounds__(kThreads) k_attn(StepArgs S, uint32_t layer) {
    const uint32_t kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const uint32_t hd = S.head_dim, group = S.heads / S.kv_heads;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t pos = S.pos_of(t);
    const uint32_t j0 = split * kAttnChunk;
    if (j0 > pos) return;
    const uint32_t n = min(kAttnChunk, pos + 1 - j0);
    extern __shared__ float sm[];
    float* qs = sm;                          // [group][hd]
    float* sc = qs + group * hd;             // [group][kAttnChunk]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t i = threadIdx.x; i < group * hd; i += blockDim.x)
        qs[i] = S.q[(size_t)t * S.hidden + kvh * group * hd + i];
    __syncthreads();
    const uint16_t* K = S.kcache + S.cache_offset(S.seq_of(t), layer, 0) + kvh * hd;
    const uint16_t* V = S.vcache + S.cache_offset(S.seq_of(t), layer, 0) + kvh * hd;
    const uint32_t stride = S.kv_heads * hd;
    const float scale = rsqrtf((float)hd);
    // scores: a warp per position, each lane two dims (hd == 64)
    const bool live = 2u * lane < hd;  // hd <= 64, even
    for (uint32_t j = warp; j < n; j += kWarps) {
        float2 kf = make_float2(0.f, 0.f);
        if (live) kf = __half22float2(reinterpret_cast<const __half2*>(K + (size_t)(j0 + j) * stride)[lane]);
        for (uint32_t h = 0; h < group; ++h) {
            float p = live ? qs[h * hd + 2 * lane] * kf.x + qs[h * hd + 2 * lane + 1] * kf.y : 0.f;
            p = warp_sum(p);
            if (lane == 0) sc[h * kAttnChunk + j] = p * scale;
        }
    }
    __syncthreads();
    // per-head max and exp (one warp per head)
    float* mx = sc + group * kAttnChunk;     // [group]
    float* sum = mx + group;                 // [group]
    for (uint32_t h = warp; h < group; h += kWarps) {
        float m = -INFINITY;
        for (uint32_t j = lane; j < n; j += 32) m = fmaxf(m, sc[h * kAttnChunk + j]);
        m = warp_max(m);
        float s = 0.f;
        for (uint32_t j = lane; j < n; j += 32) {
            float e = __expf(sc[h * kAttnChunk + j] - m);
            sc[h * kAttnChunk + j] = e;
            s += e;
        }
        s = warp_sum(s);
        if (lane == 0) { mx[h] = m; sum[h] = s; }
    }
    __syncthreads();
    float* part = S.attn_part + (((size_t)t * S.splits + split) * S.heads + kvh * group) * (hd + 2);
    for (uint32_t o = threadIdx.x; o < group * hd; o += blockDim.x) {
        uint32_t h = o / hd, d = o % hd;
        float acc = 0.f;
        const float* e = sc + h * kAttnChunk;
        for (uint32_t j = 0; j < n; ++j)
            acc = fmaf(e[j], __half2float(__ushort_as_half(V[(size_t)(j0 + j) * stride + d])), acc);
        part[h * (hd + 2) + d] = acc;
        if (d == 0) {
            part[h * (hd + 2) + hd] = mx[h];
            part[h * (hd + 2) + hd + 1] = sum[h];
        }
    }
}

// Merge the split partials of MT tokens into X4 (q4 chunk layout over `hidden`).
template <int MT>
__device__ __forceinline__ void merge_attention(float4* X4, const StepArgs& S) {
    const uint32_t hd = S.head_dim, H = S.hidden, nchunk = H / 32;
    float* Xf = reinterpret_cast<float*>(X4);
    for (uint32_t i = threadIdx.x; i < MT * H; i += blockDim.x) {
        uint32_t t = i / H, o = i % H, h = o / hd, d = o % hd;
        uint32_t splits = S.pos_of(t) / kAttnChunk + 1;
        const float* base = S.attn_part + ((size_t)t * S.splits * S.heads + h) * (hd + 2);
        const size_t sstride = (size_t)S.heads * (hd + 2);
        float M = -INFINITY;
        for (uint32_t s = 0; s < splits; ++s) M = fmaxf(M, base[s * sstride + hd]);
        float L = 0.f, acc = 0.f;
        for (uint32_t s = 0; s < splits; ++s) {
            float f = __expf(base[s * sstride + hd] - M);
            L = fmaf(base[s * sstride + hd + 1], f, L);
            acc = fmaf(base[s * sstride + d], f, acc);
        }
        float v = acc / L;
        uint32_t c = o / 32, e = o % 32;
        Xf[((t * 8 + e / 4) * nchunk + c) * 4 + (e % 4)] = v;
    }
    __syncthreads();
}

// o projection + residual: x[t][r] += Wo[r] . attn[t]
template <int MT>
__global__ void __launch_bounds__(kThreads) k_oproj(LayerArgs L, StepArgs S) {
    extern __shared__ float4 X4[];
    const uint32_t H = S.hidden, nchunk = H / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2)
        if (lane < 2 && r0 + lane < H) prefetch_row<4>(L.wo, r0 + lane);
    pdl_wait();
    merge_attention<MT>(X4, S);
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2) {
        uint32_t rows[2] = {r0, min(r0 + 1, H - 1)};
        float acc[2][MT] = {};
        dot_rows<4, MT, 2>(L.wo, rows, X4, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= H) break;
                float v = 0.f;
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t == lane) v = acc[r][t];
                float* xp = S.x + (size_t)lane * H + rows[r];
                *xp = *xp + v;
            }
        }
    }
}

// RMSNorm + gate|up + SiLU(gate)*up: gated[t][r]
template <int MT>
__global__ void __launch_bounds__(kThreads) k_gateup(LayerArgs L, StepArgs S) {
    extern __shared__ float4 X4[];
    __shared__ float rs[MT], red[kWarps];
    const uint32_t H = S.hidden, I = S.intermediate, nchunk = H / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r = blockIdx.x * kWarps + warp; r < I; r += gridDim.x * kWarps) {
        if (lane == 0) prefetch_row<4>(L.wg, r);
        if (lane == 1) prefetch_row<4>(L.wu, r);
    }
    pdl_wait();
    rms_scale<MT>(rs, red, S.x, H, S.eps);
    stage_x<4, MT>(X4, S.x, H, rs, L.norm_post);
    for (uint32_t r = blockIdx.x * kWarps + warp; r < I; r += gridDim.x * kWarps) {
        float ag[1][MT] = {}, au[1][MT] = {};
        uint32_t rows[1] = {r};
        dot_rows<4, MT, 1>(L.wg, rows, X4, nchunk, lane, ag);
        dot_rows<4, MT, 1>(L.wu, rows, X4, nchunk, lane, au);
#pragma unroll
        for (int t = 0; t < MT; ++t) { ag[0][t] = warp_sum(ag[0][t]); au[0][t] = warp_sum(au[0][t]); }
        if (lane < MT) {
            float g = 0.f, u = 0.f;
#pragma unroll
            for (int t = 0; t < MT; ++t)
                if (t == lane) { g = ag[0][t]; u = au[0][t]; }
            // silu(g) * u = g / (1 + exp(-g)) * u (src/kernels/silu_mul.wgsl:19-26)
            S.gated[(size_t)lane * I + r] = g / (1.0f + expf(-g)) * u;
        }
    }
}

// down projection + residual: x[t][r] += Wd[r] . gated[t]
template <int MT>
__global__ void __launch_bounds__(kThreads) k_down(LayerArgs L, StepArgs S) {
    extern __shared__ float4 X4[];
    const uint32_t H = S.hidden, I = S.intermediate, nchunk = I / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2)
        if (lane < 2 && r0 + lane < H) prefetch_row<4>(L.wd, r0 + lane);
    pdl_wait();
    stage_x<4, MT>(X4, S.gated, I, nullptr, nullptr);
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2) {
        uint32_t rows[2] = {r0, min(r0 + 1, H - 1)};
        float acc[2][MT] = {};
        dot_rows<4, MT, 2>(L.wd, rows, X4, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= H) break;
                float v = 0.f;
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t == lane) v = acc[r][t];
                float* xp = S.x + (size_t)lane * H + rows[r];
                *xp = *xp + v;
            }
        }
    }
}

// final RMSNorm + tied int8 (or int4) head: logits[t][r] = E[r] . normed[t]
template <int BITS, int MT>
__global__ void __launch_bounds__(kThreads) k_head(HeadArgs Hd, StepArgs S) {
    extern __shared__ float4 X4[];
    __shared__ float rs[MT], red[kWarps];
    const uint32_t H = S.hidden, V = Hd.embed.rows, nchunk = H / Geom<BITS>::E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    rms_scale<MT>(rs, red, S.x, H, S.eps);
    stage_x<BITS, MT>(X4, S.x, H, rs, Hd.norm);
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < MT * H; i += blockDim.x)
            S.normed[i] = S.x[i] * rs[i / H] * Hd.norm[i % H];
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < V; r0 += gridDim.x * kWarps * 2) {
        uint32_t rows[2] = {r0, min(r0 + 1, V - 1)};
        float acc[2][MT] = {};
        dot_rows<BITS, MT, 2>(Hd.embed, rows, X4, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= V) break;
                float v = 0.f;
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t == lane) v = acc[r][t];
                S.logits[(size_t)lane * V + rows[r]] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// launchers

static int g_sms = 0;
int num_sms() {
    if (!g_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

template <typename Kern, typename... Args>
static cudaError_t launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, k, args...);
}

static uint32_t grid_for(uint32_t items, uint32_t per_cta, uint32_t cap) {
    uint32_t g = (items + per_cta - 1) / per_cta;
    return g < 1 ? 1 : (g > cap ? cap : g);
}

cudaError_t launch_embed(const uint32_t* ids, const QW& table, int bits, float* out, uint32_t seq,
                         uint32_t row_begin, uint32_t row_count, uint32_t out_stride,
                         cudaStream_t st, bool pdl) {
    dim3 grid((table.cols + 255) / 256, seq);
    if (bits == 8) return launch(k_embed<8>, grid, dim3(256), 0, st, pdl, ids, table, out, row_begin, row_count, out_stride);
    return launch(k_embed<4>, grid, dim3(256), 0, st, pdl, ids, table, out, row_begin, row_count, out_stride);
}

template <int BITS>
static cudaError_t launch_matmul_bits(const float* x, const QW& w, const float* bias, float* out,
                                      uint32_t m, uint32_t out_stride, uint32_t out_offset,
                                      cudaStream_t st, bool pdl) {
    const uint32_t cap = num_sms() * 4;
    uint32_t gx = grid_for(w.rows, kWarps * 2, cap);
    if (m == 1) {
        return launch(k_matmul<BITS, 1>, dim3(gx, 1), dim3(kThreads), (size_t)1 * w.cols * 4, st, pdl, x, w, bias,
                      out, m, out_stride, out_offset);
    }
    if (m == 2) {
        return launch(k_matmul<BITS, 2>, dim3(gx, 1), dim3(kThreads), (size_t)2 * w.cols * 4, st, pdl, x, w, bias,
                      out, m, out_stride, out_offset);
    }
    return launch(k_matmul<BITS, 4>, dim3(gx, (m + 3) / 4), dim3(kThreads), (size_t)4 * w.cols * 4, st, pdl, x,
                  w, bias, out, m, out_stride, out_offset);
}

cudaError_t launch_matmul(int bits, const float* x, const QW& w, const float* bias, float* out,
                          uint32_t m, uint32_t out_stride, uint32_t out_offset, cudaStream_t st,
                          bool pdl) {
    return bits == 8 ? launch_matmul_bits<8>(x, w, bias, out, m, out_stride, out_offset, st, pdl)
                     : launch_matmul_bits<4>(x, w, bias, out, m, out_stride, out_offset, st, pdl);
}

template <int MT>
static cudaError_t launch_layer_mt(const LayerArgs& L, const StepArgs& S, cudaStream_t st) {
    const uint32_t cap = num_sms() * 4;
    cudaError_t e;
    const uint32_t qkv_items = (S.heads + 2 * S.kv_heads) * (S.head_dim / 2);
    e = launch(k_qkv<MT>, dim3(grid_for(qkv_items, kWarps, cap)), dim3(kThreads),
               (size_t)MT * S.hidden * 4, st, true, L, S);
    if (e != cudaSuccess) return e;
    const uint32_t group = S.heads / S.kv_heads;
    size_t attn_smem = ((size_t)group * S.head_dim + (size_t)group * kAttnChunk + 2 * group) * 4;
    e = launch(k_attn<MT>, dim3(S.kv_heads, S.splits, MT), dim3(kThreads), attn_smem, st, true, S, L.layer);
    if (e != cudaSuccess) return e;
    e = launch(k_oproj<MT>, dim3(grid_for(S.hidden, kWarps * 2, cap)), dim3(kThreads),
               (size_t)MT * S.hidden * 4, st, true, L, S);
    if (e != cudaSuccess) return e;
    e = launch(k_gateup<MT>, dim3(grid_for(S.intermediate, kWarps, cap)), dim3(kThreads),
               (size_t)MT * S.hidden * 4, st, true, L, S);
    if (e != cudaSuccess) return e;
    return launch(k_down<MT>, dim3(grid_for(S.hidden, kWarps * 2, cap)), dim3(kThreads),
                  (size_t)MT * S.intermediate * 4, st, true, L, S);
}

cudaError_t launch_layer(uint32_t mt, const LayerArgs& L, const StepArgs& S, cudaStream_t st) {
    switch (mt) {
        case 1: return launch_layer_mt<1>(L, S, st);
        case 2: return launch_layer_mt<2>(L, S, st);
        case 3: return launch_layer_mt<3>(L, S, st);
        default: return launch_layer_mt<4>(L, S, st);
    }
}

template <int BITS, int MT>
static cudaError_t launch_head_mt(const HeadArgs& Hd, const StepArgs& S, cudaStream_t st) {
    const uint32_t cap = num_sms() * 4;
    return launch(k_head<BITS, MT>, dim3(grid_for(Hd.embed.rows, kWarps * 2, cap)), dim3(kThreads),
                  (size_t)MT * S.hidden * 4, st, true, Hd, S);
}

cudaError_t launch_head(uint32_t mt, int bits, const HeadArgs& Hd, const StepArgs& S, cudaStream_t st) {
    if (bits == 8) {
        switch (mt) {
            case 1: return launch_head_mt<8, 1>(Hd, S, st);
            case 2: return launch_head_mt<8, 2>(Hd, S, st);
            case 3: return launch_head_mt<8, 3>(Hd, S, st);
            default: return launch_head_mt<8, 4>(Hd, S, st);
        }
    }
    switch (mt) {
        case 1: return launch_head_mt<4, 1>(Hd, S, st);
        case 2: return launch_head_mt<4, 2>(Hd, S, st);
        case 3: return launch_head_mt<4, 3>(Hd, S, st);
        default: return launch_head_mt<4, 4>(Hd, S, st);
    }
}

cudaError_t launch_attn(const StepArgs& S, uint32_t layer, uint32_t ntok, cudaStream_t st) {
    const uint32_t group = S.heads / S.kv_heads;
    size_t attn_smem = ((size_t)group * S.head_dim + (size_t)group * kAttnChunk + 2 * group) * 4;
    return launch(k_attn<1>, dim3(S.kv_heads, S.splits, ntok), dim3(kThreads), attn_smem, st, false, S, layer);
}

// Merge of the split partials for the prefill / raw paths: out[t][o], grid.y = token.
__global__ void k_attn_merge(StepArgs S, float* out) {
    const uint32_t hd = S.head_dim, H = S.hidden, t = blockIdx.y;
    for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < H; o += gridDim.x * blockDim.x) {
        uint32_t h = o / hd, d = o % hd;
        uint32_t splits = S.pos_of(t) / kAttnChunk + 1;
        const float* base = S.attn_part + ((size_t)t * S.splits * S.heads + h) * (hd + 2);
        const size_t sstride = (size_t)S.heads * (hd + 2);
        float M = -INFINITY;
        for (uint32_t s = 0; s < splits; ++s) M = fmaxf(M, base[s * sstride + hd]);
        float L = 0.f, acc = 0.f;
        for (uint32_t s = 0; s < splits; ++s) {
            float f = __expf(base[s * sstride + hd] - M);
            L = fmaf(base[s * sstride + hd + 1], f, L);
            acc = fmaf(base[s * sstride + d], f, acc);
        }
        out[(size_t)t * H + o] = acc / L;
    }
}

cudaError_t launch_attn_merge(const StepArgs& S, float* out, uint32_t ntok, cudaStream_t st) {
    k_attn_merge<<<dim3((S.hidden + 255) / 256, ntok), 256, 0, st>>>(S, out);
    return cudaGetLastError();
}

}  // namespace enx
