// Decode-shaped kernels: the int4 projections with their fused prologues/epilogues, the int8
// tied head, the embedding gather, and decode attention over the f16 cache.
//
// One decoder layer of one step is six launches on this path (the reference issues 19
// dispatches, src/model/graph_decode.ts:268-358):
//   k_qkv          RMSNorm prologue + q|k|v projections + bias + RoPE + f16 cache append
//   k_attn_scores  q.K scores of 64 cached positions per CTA (all query heads of one kv head)
//   k_attn_apply   softmax + weighted V for all query heads of one kv head
//   k_oproj        o projection + residual add
//   k_gateup       RMSNorm prologue + gate|up projections + SiLU*up
//   k_down         down projection + residual add
// and the step ends with k_head (final RMSNorm + tied int8 head).  Each kernel issues its
// launch_dependents at once and an L2 prefetch of its own weights before waiting for its
// predecessor (programmatic dependent launch).  The persistent kernel (k_mega.cu) replaces this
// path whenever it fits; this path covers the rest (long contexts, other batch sizes).
//
// All reductions are in double and every stored activation is rounded to float exactly where the
// reference's CPU path rounds it (see k_matvec.cuh).

#include "k_matvec.cuh"
#include "k_decode.cuh"

namespace enx {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    // cp.async.bulk.prefetch wants a 16-byte aligned address and a multiple of 16 bytes
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t b = a & ~uintptr_t(15);
    const uint32_t n = (uint32_t)(((a + bytes + 15) & ~uintptr_t(15)) - b);
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
}

template <int BITS>
__device__ __forceinline__ void prefetch_row(const QW& w, uint32_t row) {
    const uint32_t bytes = w.cols * BITS / 8;
    prefetch_l2(reinterpret_cast<const char*>(w.packed) + (size_t)row * bytes, bytes);
}

template <int MT>
__device__ __forceinline__ double pick_d(const double (&a)[MT], int t) {
    double v = 0.0;
#pragma unroll
    for (int i = 0; i < MT; ++i)
        if (i == t) v = a[i];
    return v;
}

// ---------------------------------------------------------------------------------------------
// embedding gather (embed_gather_q8 / _q4, src/kernels/embedding_variants.ts:100-130)

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
        const size_t flat = (size_t)row * K + c;
        const uint32_t q = BITS == 4 ? (table.packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu
                                     : (table.packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
        const uint32_t blk = row * bpr + c / kBlock;
        // (q - z) * s: an exact small integer times a float, one rounding, as the reference
        out[(size_t)s * out_stride + c] = ((float)q - (float)zero_code<BITS>(table.zeros, blk)) * table.scales[blk];
    }
}

// ---------------------------------------------------------------------------------------------
// generic projection (raw enx_matmul_q4 / enx_lm_head_q8 entry points and prefill)

template <int BITS, int MT>
__global__ void __launch_bounds__(kThreads) k_matmul(const float* __restrict__ x, QW w,
                                                     const float* __restrict__ bias,
                                                     float* __restrict__ out, uint32_t m,
                                                     uint32_t out_stride, uint32_t out_offset) {
    extern __shared__ double2 XD[];
    const uint32_t K = w.cols, N = w.rows, nchunk = K / Geom<BITS>::E;
    const uint32_t t0 = blockIdx.y * MT;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    double* Xs = reinterpret_cast<double*>(XD);
    for (uint32_t i = threadIdx.x; i < MT * K; i += blockDim.x) {
        const uint32_t t = i / K, k = i % K;
        const uint32_t src = min(t0 + t, m - 1);  // rows past m read a clamped row, not written
        Xs[xd_index<BITS>(t, k, nchunk)] = (double)x[(size_t)src * K + k];
    }
    __syncthreads();
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < N; r0 += gridDim.x * kWarps * 2) {
        const uint32_t rows[2] = {r0, min(r0 + 1, N - 1)};
        double acc[2][MT] = {};
        dot_rows_d<BITS, MT, 2>(w, rows, XD, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
        if (lane < MT && t0 + lane < m) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && r0 + 1 >= N) break;
                double v = pick_d<MT>(acc[r], lane);
                if (bias) v += (double)bias[rows[r]];
                out[(size_t)(t0 + lane) * out_stride + out_offset + rows[r]] = (float)v;
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
    extern __shared__ double2 XD[];
    __shared__ double rs[MT], red[MT * kWarps];
    const uint32_t H = S.hidden, hd = S.head_dim, half = hd / 2;
    const uint32_t items = (S.heads + 2 * S.kv_heads) * half;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t it = blockIdx.x * kWarps + warp; it < items; it += gridDim.x * kWarps) {
        if (lane < 2) {
            const uint32_t hs = it / half, i = it % half;
            const QW& w = hs < S.heads ? L.wq : hs < S.heads + S.kv_heads ? L.wk : L.wv;
            const uint32_t base = hs < S.heads ? hs * hd
                                : hs < S.heads + S.kv_heads ? (hs - S.heads) * hd
                                                            : (hs - S.heads - S.kv_heads) * hd;
            prefetch_row<4>(w, base + i + lane * half);
        }
    }
    pdl_wait();
    rms_scale_d<MT, true>(rs, red, S.x, H, S.eps);
    stage_x_d<4, MT, true>(reinterpret_cast<double*>(XD), S.x, H, rs, L.norm_in);
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
        const uint32_t rows[2] = {head * hd + i, head * hd + i + half};
        double acc[2][MT] = {};
        dot_rows_d<4, MT, 2>(w, rows, XD, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
        if (lane < MT) {
            float a = (float)(pick_d<MT>(acc[0], lane) + (double)bias[rows[0]]);
            float b = (float)(pick_d<MT>(acc[1], lane) + (double)bias[rows[1]]);
            const uint32_t pos = S.pos_of(lane);
            if (kind != 2) rope_pair(a, b, S.rope_cos[(size_t)pos * half + i], S.rope_sin[(size_t)pos * half + i]);
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

// Scores of up to 64 positions for the query heads of one kv head:
// scores[t][h][j] = float(sum_d q[h][d] * K[j][kv][d] / sqrt(hd)), the sum in double
// (test/reference/ops.ts:123-151).  grid = (kv_heads, score_stride / 64, ntok).
__global__ void __launch_bounds__(kThreads) k_attn_scores(StepArgs S, uint32_t layer) {
    const uint32_t g = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const uint32_t hd = S.head_dim, group = S.heads / S.kv_heads, kvd = S.kv_heads * hd;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t pos = S.pos_of(t), j0 = split * kAttnChunk;
    if (j0 > pos) return;
    const uint32_t n = min(kAttnChunk, pos + 1 - j0);
    __shared__ double qd[8 * 64];                            // group <= 8, hd <= 64
    __shared__ __align__(16) uint16_t ks[kAttnChunk * 64];  // n cached rows of this kv head
    for (uint32_t i = threadIdx.x; i < group * hd; i += blockDim.x)
        qd[i] = (double)__ldcg(S.q + (size_t)t * S.hidden + g * group * hd + i);
    const uint16_t* K = S.kcache + S.cache_offset(S.seq_of(t), layer, j0) + g * hd;
    const uint32_t row8 = hd / 8;
    for (uint32_t i = threadIdx.x; i < n * row8; i += blockDim.x)
        reinterpret_cast<uint4*>(ks)[i] = __ldcg(reinterpret_cast<const uint4*>(K + (size_t)(i / row8) * kvd) + i % row8);
    __syncthreads();
    const double scale = 1.0 / sqrt((double)hd);
    for (uint32_t w = threadIdx.x; w < n * group; w += blockDim.x) {
        const uint32_t j = w / group, h = w % group;
        const double* qh = qd + h * hd;
        const uint16_t* kr = ks + j * hd;
        double acc = 0.0;
        for (uint32_t d = 0; d < hd; ++d) acc = fma(qh[d], (double)__half2float(__ushort_as_half(kr[d])), acc);
        S.scores[((size_t)t * S.heads + g * group + h) * S.score_stride + j0 + j] = (float)(acc * scale);
    }
}

// Softmax over the live positions and the weighted V sum for the query heads of one kv head,
// rounding as the reference does (test/reference/ops.ts:161-204): w = float(e) then
// float(w / sum) with e = exp(score - max) and the sum in double; out = float(sum_j w * v).
// grid = (kv_heads, ntok); dynamic shared memory holds group * score_stride weights.
__global__ void __launch_bounds__(kThreads) k_attn_apply(StepArgs S, uint32_t layer, float* out) {
    extern __shared__ float wts[];  // [group][score_stride]
    __shared__ __align__(16) uint16_t vs[kAttnChunk * 64];
    const uint32_t g = blockIdx.x, t = blockIdx.y;
    const uint32_t hd = S.head_dim, group = S.heads / S.kv_heads, kvd = S.kv_heads * hd;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t npos = S.pos_of(t) + 1;
    for (uint32_t h = warp; h < group; h += kWarps) {
        const float* sc = S.scores + ((size_t)t * S.heads + g * group + h) * S.score_stride;
        float* w = wts + (size_t)h * S.score_stride;
        float m = -INFINITY;
        for (uint32_t j = lane; j < npos; j += 32) m = fmaxf(m, __ldcg(sc + j));
        m = warp_max(m);
        double sum = 0.0;
        for (uint32_t j = lane; j < npos; j += 32) {
            const double e = exp((double)__ldcg(sc + j) - (double)m);
            w[j] = (float)e;
            sum += e;
        }
        sum = warp_sum_d(sum);
        for (uint32_t j = lane; j < npos; j += 32) w[j] = (float)((double)w[j] / sum);
    }
    const uint16_t* V = S.vcache + S.cache_offset(S.seq_of(t), layer, 0) + g * hd;
    const uint32_t outs = group * hd, row8 = hd / 8;
    double acc[2] = {0.0, 0.0};  // outputs threadIdx.x and threadIdx.x + blockDim.x (<= 512)
    for (uint32_t j0 = 0; j0 < npos; j0 += kAttnChunk) {
        const uint32_t n = min(kAttnChunk, npos - j0);
        __syncthreads();  // weights ready (first pass) / previous chunk consumed
        for (uint32_t i = threadIdx.x; i < n * row8; i += blockDim.x)
            reinterpret_cast<uint4*>(vs)[i] =
                __ldcg(reinterpret_cast<const uint4*>(V + (size_t)(j0 + i / row8) * kvd) + i % row8);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t o = threadIdx.x + k * blockDim.x;
            if (o >= outs) break;
            const uint32_t h = o / hd, d = o % hd;
            const float* w = wts + (size_t)h * S.score_stride + j0;
            double a = acc[k];
            for (uint32_t j = 0; j < n; ++j) a = fma((double)w[j], (double)__half2float(__ushort_as_half(vs[j * hd + d])), a);
            acc[k] = a;
        }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t o = threadIdx.x + k * blockDim.x;
        if (o < outs) out[(size_t)t * S.hidden + g * group * hd + o] = (float)acc[k];
    }
}

// o projection + residual: x[t][r] += float(Wo[r] . attn[t])
template <int MT>
__global__ void __launch_bounds__(kThreads) k_oproj(LayerArgs L, StepArgs S) {
    extern __shared__ double2 XD[];
    const uint32_t H = S.hidden, nchunk = H / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2)
        if (lane < 2 && r0 + lane < H) prefetch_row<4>(L.wo, r0 + lane);
    pdl_wait();
    stage_x_d<4, MT, true>(reinterpret_cast<double*>(XD), S.attn_out, H, nullptr, nullptr);
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2) {
        const uint32_t rows[2] = {r0, min(r0 + 1, H - 1)};
        double acc[2][MT] = {};
        dot_rows_d<4, MT, 2>(L.wo, rows, XD, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= H) break;
                float* xp = S.x + (size_t)lane * H + rows[r];
                *xp = *xp + (float)pick_d<MT>(acc[r], lane);
            }
        }
    }
}

// RMSNorm + gate|up + SiLU(gate)*up: gated[t][r]
template <int MT>
__global__ void __launch_bounds__(kThreads) k_gateup(LayerArgs L, StepArgs S) {
    extern __shared__ double2 XD[];
    __shared__ double rs[MT], red[MT * kWarps];
    const uint32_t H = S.hidden, I = S.intermediate, nchunk = H / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r = blockIdx.x * kWarps + warp; r < I; r += gridDim.x * kWarps) {
        if (lane == 0) prefetch_row<4>(L.wg, r);
        if (lane == 1) prefetch_row<4>(L.wu, r);
    }
    pdl_wait();
    rms_scale_d<MT, true>(rs, red, S.x, H, S.eps);
    stage_x_d<4, MT, true>(reinterpret_cast<double*>(XD), S.x, H, rs, L.norm_post);
    for (uint32_t r = blockIdx.x * kWarps + warp; r < I; r += gridDim.x * kWarps) {
        double ag[1][MT] = {}, au[1][MT] = {};
        const uint32_t rows[1] = {r};
        dot_rows_d<4, MT, 1>(L.wg, rows, XD, nchunk, lane, ag);
        dot_rows_d<4, MT, 1>(L.wu, rows, XD, nchunk, lane, au);
#pragma unroll
        for (int t = 0; t < MT; ++t) { ag[0][t] = warp_sum_d(ag[0][t]); au[0][t] = warp_sum_d(au[0][t]); }
        if (lane < MT)
            S.gated[(size_t)lane * I + r] = silu_mul_value((float)pick_d<MT>(ag[0], lane), (float)pick_d<MT>(au[0], lane));
    }
}

// down projection + residual: x[t][r] += float(Wd[r] . gated[t])
template <int MT>
__global__ void __launch_bounds__(kThreads) k_down(LayerArgs L, StepArgs S) {
    extern __shared__ double2 XD[];
    const uint32_t H = S.hidden, I = S.intermediate, nchunk = I / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2)
        if (lane < 2 && r0 + lane < H) prefetch_row<4>(L.wd, r0 + lane);
    pdl_wait();
    stage_x_d<4, MT, true>(reinterpret_cast<double*>(XD), S.gated, I, nullptr, nullptr);
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < H; r0 += gridDim.x * kWarps * 2) {
        const uint32_t rows[2] = {r0, min(r0 + 1, H - 1)};
        double acc[2][MT] = {};
        dot_rows_d<4, MT, 2>(L.wd, rows, XD, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= H) break;
                float* xp = S.x + (size_t)lane * H + rows[r];
                *xp = *xp + (float)pick_d<MT>(acc[r], lane);
            }
        }
    }
}

// final RMSNorm + tied head: logits[t][r] = float(E[r] . normed[t])
template <int BITS, int MT>
__global__ void __launch_bounds__(kThreads) k_head(HeadArgs Hd, StepArgs S) {
    extern __shared__ double2 XD[];
    __shared__ double rs[MT], red[MT * kWarps];
    const uint32_t H = S.hidden, V = Hd.embed.rows, nchunk = H / Geom<BITS>::E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    rms_scale_d<MT, true>(rs, red, S.x, H, S.eps);
    stage_x_d<BITS, MT, true>(reinterpret_cast<double*>(XD), S.x, H, rs, Hd.norm);
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < MT * H; i += blockDim.x)
            S.normed[i] = norm_value(__ldcg(S.x + i), rs[i / H], Hd.norm[i % H]);
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * 2; r0 < V; r0 += gridDim.x * kWarps * 2) {
        const uint32_t rows[2] = {r0, min(r0 + 1, V - 1)};
        double acc[2][MT] = {};
        dot_rows_d<BITS, MT, 2>(Hd.embed, rows, XD, nchunk, lane, acc);
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
        if (lane < MT) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r0 + r >= V) break;
                S.logits[(size_t)lane * V + rows[r]] = (float)pick_d<MT>(acc[r], lane);
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
static cudaError_t launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
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
        const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, k, args...);
}

static uint32_t grid_for(uint32_t items, uint32_t per_cta, uint32_t cap) {
    const uint32_t g = (items + per_cta - 1) / per_cta;
    return g < 1 ? 1 : (g > cap ? cap : g);
}

cudaError_t launch_embed(const uint32_t* ids, const QW& table, int bits, float* out, uint32_t seq, uint32_t row_begin,
                         uint32_t row_count, uint32_t out_stride, cudaStream_t st, bool pdl) {
    const dim3 grid((table.cols + 255) / 256, seq);
    if (bits == 8) return launch(k_embed<8>, grid, dim3(256), 0, st, pdl, ids, table, out, row_begin, row_count, out_stride);
    return launch(k_embed<4>, grid, dim3(256), 0, st, pdl, ids, table, out, row_begin, row_count, out_stride);
}

template <int BITS>
static cudaError_t launch_matmul_bits(const float* x, const QW& w, const float* bias, float* out, uint32_t m,
                                      uint32_t out_stride, uint32_t out_offset, cudaStream_t st, bool pdl) {
    const uint32_t gx = grid_for(w.rows, kWarps * 2, num_sms() * 4);
    if (m == 1)
        return launch(k_matmul<BITS, 1>, dim3(gx, 1), dim3(kThreads), (size_t)w.cols * 8, st, pdl, x, w, bias, out, m,
                      out_stride, out_offset);
    if (m == 2)
        return launch(k_matmul<BITS, 2>, dim3(gx, 1), dim3(kThreads), (size_t)2 * w.cols * 8, st, pdl, x, w, bias,
                      out, m, out_stride, out_offset);
    return launch(k_matmul<BITS, 4>, dim3(gx, (m + 3) / 4), dim3(kThreads), (size_t)4 * w.cols * 8, st, pdl, x, w,
                  bias, out, m, out_stride, out_offset);
}

cudaError_t launch_matmul(int bits, const float* x, const QW& w, const float* bias, float* out, uint32_t m,
                          uint32_t out_stride, uint32_t out_offset, cudaStream_t st, bool pdl) {
    return bits == 8 ? launch_matmul_bits<8>(x, w, bias, out, m, out_stride, out_offset, st, pdl)
                     : launch_matmul_bits<4>(x, w, bias, out, m, out_stride, out_offset, st, pdl);
}

// Many-token attention on the f64 tensor cores (mma.sync m8n8k4 .f64: D[8x8] += A[8x4] B[4x8]).
// Lane roles in a fragment: A row / D row = lane / 4, A column / B row (the k index) = lane % 4,
// B column = lane / 4, D columns = 2 (lane % 4) + {0, 1}.
constexpr uint32_t kMaxGroupSplit = 8;

__device__ __forceinline__ void dmma(double& d0, double& d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// Scores: one CTA per (kv head, split of kAttnSplit positions, token), a warp per 8 positions at a
// time: D[head][position] over the group's query heads (rows, 8 at most) and 8 positions
// (columns), k running over the head dimension.  Lane k-slot q (lane % 4) owns dimensions
// q*hd/4 .. q*hd/4 + hd/4 - 1, and MMA step s uses dimension q*hd/4 + s in both operands, so A
// (its head's query, widened once) stays in registers and B is one coalesced read of the lane's
// hd/4 K values per position.  scores[t][h][j] = float(sum_d q[h][d] * K[j][d] / sqrt(hd)), the
// products exact in double (test/reference/ops.ts:123-151).
__global__ void __launch_bounds__(kAttnSplit) k_attn_scores_split(StepArgs S, uint32_t layer) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t g = blockIdx.x, sp = blockIdx.y, t = blockIdx.z;
    const uint32_t hd = S.head_dim, group = S.heads / S.kv_heads, kvd = S.kv_heads * hd;
    const uint32_t npos = S.pos_of(t) + 1, j0 = sp * kAttnSplit;
    if (j0 >= npos) return;
    const uint32_t n = min(kAttnSplit, npos - j0);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = lane >> 2, quad = lane & 3;
    const uint32_t steps = hd / 4, base = quad * steps;  // hd in {32, 64}: 8 or 16 steps
    double qa[16];
    const float* qrow = S.q + (size_t)t * S.hidden + (size_t)(g * group + row) * hd + base;
#pragma unroll
    for (uint32_t s = 0; s < 16; ++s) qa[s] = (row < group && s < steps) ? (double)__ldcg(qrow + s) : 0.0;
    const double scale = 1.0 / sqrt((double)hd);
    const uint16_t* K = S.kcache + S.cache_offset(S.seq_of(t), layer, j0) + g * hd + base;
    float* out = S.scores + ((size_t)t * S.heads + g * group + row) * S.score_stride + j0;
    // the warp's positions p0 = 8 warp + 32 i, i < 4: all K reads issued before the first MMA
    uint4 kv[4][2];
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
        const uint32_t pos = warp * 8 + 32 * i + row;  // this lane's B column
        kv[i][0] = kv[i][1] = make_uint4(0, 0, 0, 0);
        if (pos < n) {
            const uint4* kp = reinterpret_cast<const uint4*>(K + (size_t)pos * kvd);
            kv[i][0] = __ldcg(kp);
            if (steps > 8) kv[i][1] = __ldcg(kp + 1);
        }
    }
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
        const uint32_t p0 = warp * 8 + 32 * i;
        if (p0 >= n) break;
        const __half* kh = reinterpret_cast<const __half*>(kv[i]);
        double d0 = 0.0, d1 = 0.0;
#pragma unroll
        for (uint32_t s = 0; s < 16; ++s)
            if (s < steps) dmma(d0, d1, qa[s], (double)__half2float(kh[s]));
        const uint32_t c0 = p0 + 2 * quad;  // D columns: positions c0, c0 + 1
        if (row < group) {
            if (c0 < n) out[c0] = (float)(d0 * scale);
            if (c0 + 1 < n) out[c0 + 1] = (float)(d1 * scale);
        }
    }
}

// Many-token attention, after k_attn_scores: the softmax of every (token, head) row in place --
// w = float(float(exp(score - max)) / sum), the exps and their sum in double
// (test/reference/ops.ts:161-178) -- by one CTA per row.
__global__ void __launch_bounds__(kThreads) k_attn_stats(StepArgs S) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t h = blockIdx.x, t = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t npos = S.pos_of(t) + 1;
    float* sc = S.scores + ((size_t)t * S.heads + h) * S.score_stride;
    __shared__ float fred[kWarps];
    __shared__ double dred[kWarps];
    float m = -INFINITY;
    for (uint32_t j = threadIdx.x; j < npos; j += blockDim.x) m = fmaxf(m, sc[j]);
    m = warp_max(m);
    if (lane == 0) fred[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, fred[w]);
    double sum = 0.0;
    for (uint32_t j = threadIdx.x; j < npos; j += blockDim.x) {
        const double e = exp((double)sc[j] - (double)m);
        sc[j] = (float)e;
        sum += e;
    }
    sum = warp_sum_d(sum);
    if (lane == 0) dred[warp] = sum;
    __syncthreads();
    sum = 0.0;
    for (int w = 0; w < kWarps; ++w) sum += dred[w];  // fixed order
    for (uint32_t j = threadIdx.x; j < npos; j += blockDim.x) sc[j] = (float)((double)sc[j] / sum);
}

// Weighted V on the f64 tensor cores: out[h][d] = sum_j w[h][j] V[j][d] over one split of
// kApplySplit positions for the query heads of one kv head (test/reference/ops.ts:181-204), into
// attn_part[t][split][h][d].  A warp per quarter of the split, 4 positions per MMA step: A = the
// weights (head x position), B = V (position x 8 dimensions).  D column c of tile n holds
// dimension c*hd/8 + n, so a lane (B column lane / 4) reads hd/8 contiguous f16 values of its
// position per step.  The quarters meet in fixed order; positions past the token's last are not
// read (the cache beyond it may hold stale bits).  grid = (kv_heads, splits, ntok), 4 warps.
__global__ void __launch_bounds__(128) k_attn_apply_split(StepArgs S, uint32_t layer) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t g = blockIdx.x, sp = blockIdx.y, t = blockIdx.z;
    const uint32_t hd = S.head_dim, group = S.heads / S.kv_heads, kvd = S.kv_heads * hd;
    const uint32_t npos = S.pos_of(t) + 1, j0 = sp * kApplySplit;
    if (j0 >= npos) return;
    const uint32_t n = min(kApplySplit, npos - j0);
    __shared__ double red[4][kMaxGroupSplit][64];  // per-quarter sums
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = lane >> 2, quad = lane & 3;
    const uint32_t tiles = hd / 8;  // 4 or 8
    const float* W = S.scores + ((size_t)t * S.heads + g * group + row) * S.score_stride + j0;
    const uint16_t* V = S.vcache + S.cache_offset(S.seq_of(t), layer, j0) + g * hd + row * tiles;
    double acc[8][2];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = 0.0;
    const uint32_t jb = warp * (kApplySplit / 4), je = min(jb + kApplySplit / 4, (n + 3) & ~3u);
    constexpr uint32_t kAhead = 8;  // MMA steps whose weights and V rows are read before their MMAs
    for (uint32_t k0 = jb; k0 < je; k0 += 4 * kAhead) {
        double w[kAhead];
        uint4 vv[kAhead];
#pragma unroll
        for (uint32_t i = 0; i < kAhead; ++i) {
            const uint32_t pos = k0 + 4 * i + quad;  // A column / B row
            const bool live = k0 + 4 * i < je && pos < n;
            w[i] = (row < group && live) ? (double)__ldcg(W + pos) : 0.0;
            vv[i] = make_uint4(0, 0, 0, 0);
            if (live) {
                if (tiles == 8) vv[i] = __ldcg(reinterpret_cast<const uint4*>(V + (size_t)pos * kvd));
                else {
                    const uint2 h = __ldcg(reinterpret_cast<const uint2*>(V + (size_t)pos * kvd));
                    vv[i].x = h.x;
                    vv[i].y = h.y;
                }
            }
        }
#pragma unroll
        for (uint32_t i = 0; i < kAhead; ++i) {
            if (k0 + 4 * i >= je) break;
            const __half* vh = reinterpret_cast<const __half*>(&vv[i]);
#pragma unroll
            for (uint32_t nn = 0; nn < 8; ++nn)
                if (nn < tiles) dmma(acc[nn][0], acc[nn][1], w[i], (double)__half2float(vh[nn]));
        }
    }
    if (row < group) {
#pragma unroll
        for (uint32_t nn = 0; nn < 8; ++nn) {
            if (nn < tiles) {
                red[warp][row][(2 * quad) * tiles + nn] = acc[nn][0];
                red[warp][row][(2 * quad + 1) * tiles + nn] = acc[nn][1];
            }
        }
    }
    __syncthreads();
    double* part = S.attn_part + (((size_t)t * (S.score_stride / kAttnSplit) + sp) * S.heads + g * group) * hd;
    for (uint32_t o = threadIdx.x; o < group * hd; o += blockDim.x) {
        const uint32_t h = o / hd, d = o % hd;
        double v = 0.0;
        for (uint32_t k = 0; k < 4; ++k) v += red[k][h][d];  // quarters in order (empty ones hold 0)
        part[o] = v;
    }
}

// out[t][h*hd + d] = float(sum over the token's splits of attn_part), splits in order.
__global__ void k_attn_combine(StepArgs S, float* out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t t = blockIdx.x, nsp = (S.pos_of(t) + kApplySplit) / kApplySplit, stride = S.score_stride / kAttnSplit;
    const double* part = S.attn_part + (size_t)t * stride * S.hidden;
    for (uint32_t o = threadIdx.x; o < S.hidden; o += blockDim.x) {
        double v = 0.0;
        for (uint32_t sp = 0; sp < nsp; ++sp) v += part[(size_t)sp * S.hidden + o];
        out[(size_t)t * S.hidden + o] = (float)v;
    }
}

cudaError_t launch_attn(const StepArgs& S, uint32_t layer, uint32_t ntok, float* out, cudaStream_t st, bool pdl,
                        int only) {
    const uint32_t group = S.heads / S.kv_heads;
    cudaError_t e = cudaSuccess;
    if (attn_split_path(S, ntok)) {
        // many tokens: scores over position splits, softmax rows, V over position splits, then
        // the fixed-order combine
        if (only < 0 || only == 0)
            e = launch(k_attn_scores_split, dim3(S.kv_heads, S.score_stride / kAttnSplit, ntok), dim3(kAttnSplit), 0,
                       st, pdl, S, layer);
        if (e == cudaSuccess && (only < 0 || only == 1))
            e = launch(k_attn_stats, dim3(S.heads, ntok), dim3(kThreads), 0, st, pdl, S);
        if (e == cudaSuccess && (only < 0 || only == 2))
            e = launch(k_attn_apply_split, dim3(S.kv_heads, (S.score_stride + kApplySplit - 1) / kApplySplit, ntok), dim3(128), 0, st,
                       pdl, S, layer);
        if (e == cudaSuccess && (only < 0 || only == 3)) e = launch(k_attn_combine, dim3(ntok), dim3(kThreads), 0, st, pdl, S, out);
        return e;
    }
    if (only < 0 || only == 0)
        e = launch(k_attn_scores, dim3(S.kv_heads, S.score_stride / kAttnChunk, ntok), dim3(kThreads), 0, st, pdl, S, layer);
    if (e == cudaSuccess && (only < 0 || only == 2))
        e = launch(k_attn_apply, dim3(S.kv_heads, ntok), dim3(kThreads), (size_t)group * S.score_stride * 4, st, pdl,
                   S, layer, out);
    return e;
}

bool attn_split_path(const StepArgs& S, uint32_t ntok) {
    return S.attn_part && ntok >= 8 && S.score_stride % kAttnSplit == 0 && S.heads / S.kv_heads <= kMaxGroupSplit &&
           (S.head_dim == 32 || S.head_dim == 64);
}

template <int MT>
static cudaError_t launch_layer_mt(const LayerArgs& L, const StepArgs& S, cudaStream_t st) {
    const uint32_t cap = num_sms() * 4;
    cudaError_t e;
    const uint32_t qkv_items = (S.heads + 2 * S.kv_heads) * (S.head_dim / 2);
    e = launch(k_qkv<MT>, dim3(grid_for(qkv_items, kWarps, cap)), dim3(kThreads), (size_t)MT * S.hidden * 8, st,
               true, L, S);
    if (e != cudaSuccess) return e;
    e = launch_attn(S, L.layer, MT, S.attn_out, st, true);
    if (e != cudaSuccess) return e;
    e = launch(k_oproj<MT>, dim3(grid_for(S.hidden, kWarps * 2, cap)), dim3(kThreads), (size_t)MT * S.hidden * 8, st,
               true, L, S);
    if (e != cudaSuccess) return e;
    e = launch(k_gateup<MT>, dim3(grid_for(S.intermediate, kWarps, cap)), dim3(kThreads), (size_t)MT * S.hidden * 8,
               st, true, L, S);
    if (e != cudaSuccess) return e;
    return launch(k_down<MT>, dim3(grid_for(S.hidden, kWarps * 2, cap)), dim3(kThreads),
                  (size_t)MT * S.intermediate * 8, st, true, L, S);
}

// Batched decode, after the q|k|v projections of B tokens (token t is sequence t, at position
// S.pos_of(t)): RoPE of q in place and of k, then k and v rounded to f16 into the token's own cache
// row (test/reference/ops.ts:103-109, src/kernels/cache_variants.ts:269-301).
__global__ void k_rope_cache_batch(StepArgs S, uint32_t layer, float* __restrict__ q, const float* __restrict__ k,
                                   const float* __restrict__ v, uint32_t B) {
    const uint32_t hd = S.head_dim, half = hd / 2, kvd = S.kv_heads * hd;
    const uint32_t qp = S.heads * half, kp = S.kv_heads * half, per = qp + kp + kvd;
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < B * per; g += gridDim.x * blockDim.x) {
        const uint32_t t = g / per, r = g % per, pos = S.pos_of(t);
        if (r < qp + kp) {
            const bool isq = r < qp;
            const uint32_t r2 = isq ? r : r - qp, h = r2 / half, i = r2 % half;
            const size_t base = isq ? (size_t)t * S.hidden + h * hd : (size_t)t * kvd + h * hd;
            float a = isq ? q[base + i] : k[base + i], b = isq ? q[base + i + half] : k[base + i + half];
            rope_pair(a, b, S.rope_cos[(size_t)pos * half + i], S.rope_sin[(size_t)pos * half + i]);
            if (isq) {
                q[base + i] = a;
                q[base + i + half] = b;
            } else {
                uint16_t* row = S.kcache + S.cache_offset(S.seq_of(t), layer, pos) + h * hd;
                row[i] = __half_as_ushort(__float2half_rn(a));
                row[i + half] = __half_as_ushort(__float2half_rn(b));
            }
        } else {
            const uint32_t e = r - qp - kp;
            S.vcache[S.cache_offset(S.seq_of(t), layer, pos) + e] = __half_as_ushort(__float2half_rn(v[(size_t)t * kvd + e]));
        }
    }
}

cudaError_t launch_rope_cache_batch(const StepArgs& S, uint32_t layer, float* q, const float* k, const float* v,
                                    uint32_t B, cudaStream_t st) {
    const uint32_t per = S.heads * (S.head_dim / 2) + S.kv_heads * (S.head_dim / 2) + S.kv_heads * S.head_dim;
    const uint32_t n = B * per;
    if (n == 0) return cudaSuccess;
    k_rope_cache_batch<<<(n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096, 256, 0, st>>>(S, layer, q, k, v, B);
    return cudaGetLastError();
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
    return launch(k_head<BITS, MT>, dim3(grid_for(Hd.embed.rows, kWarps * 2, num_sms() * 4)), dim3(kThreads),
                  (size_t)MT * S.hidden * 8, st, true, Hd, S);
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

}  // namespace enx
