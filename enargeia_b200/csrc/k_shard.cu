// Vocab-sharded tied-head sampling: the sampler of src/kernels/sample.wgsl:143-332 with the
// vocabulary split by contiguous id ranges across GPUs (rank r owns [row_begin_r, row_begin_r+n_r),
// ranks in ascending id order).  Inside a rank, `split` CTAs per row own contiguous sub-ranges,
// so the "units" (rank, cta) in rank-major order cover the vocabulary in ascending id order,
// which the draw depends on.
//
// Every phase writes one small record per (row, unit) to a send buffer; the caller allgathers
// the send buffers of all ranks into [world][rows][split] (NCCL between GPUs) and hands the
// gathered buffer to the next phase, which combines the units in order.  All ranks combine the
// same gathered values in the same order, so their decisions agree bit for bit.
//
//   prepare   repetition penalty in place (first occurrence of each history id in this shard),
//             the unit's greedy candidate (max logit, lowest id) and scaled candidate
//             (max logit/T, lowest id)                                             -> cand
//   probs     m = best scaled candidate; e = exp(logit/T - m) in double; the unit's sum -> sum
//   buckets   round k of the top-p bisection (8 steps per round, 4 rounds, k_topp.cuh): walk
//             round k-1's gathered bucket masses to the new interval (round 0: normalise p by
//             the total), then the unit's fixed-point masses of p in the 256 intervals cut by the
//             next 255 midpoints
//                                                                                    -> bucket
//   kept      walk the last round to the threshold; the unit's mass of p >= threshold -> kept
//   pick      offset of the unit = kept mass of the units before it; target = random *
//             max(total kept, 1e-20); the first id of the unit whose running mass reaches it
//                                                                                    -> pick
//   finish    greedy rows: best greedy candidate; others: the lowest picked id, else the best
//             scaled candidate's id.
//
// The arithmetic is the single-GPU sampler's (k_sample.cu): f32 penalty and scaling, double
// probabilities, kept masses and running totals, f32 bisection midpoints, exact 62-bit
// fixed-point bisection masses.

#include "enx_internal.cuh"
#include "k_small.cuh"
#include "k_topp.cuh"

namespace enx {

namespace {

constexpr int kShThreads = 1024, kShWarps = kShThreads / 32;
constexpr uint32_t kNone = 0xFFFFFFFFu;

// Per-row state each rank keeps between phases (identical on all ranks).
struct ShardState {
    float lohi[5][2];  // bisection interval after k rounds
    float gmax;        // max logit/T over the vocabulary
    uint32_t garg;     // its lowest id (the draw's fallback)
    double thr;        // top-p threshold (0 without top-p)
};
static_assert(sizeof(ShardState) == 56, "state layout");

struct ShRed {
    float f[kShWarps];
    uint32_t i[kShWarps];
    double d[kShWarps];
};

__device__ __forceinline__ bool better_sh(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// Block-wide (max, lowest id); the result in every thread.
__device__ void block_best(ShRed& r, float& v, uint32_t& i) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better_sh(ov, oi, v, i)) { v = ov; i = oi; }
    }
    if (lane == 0) { r.f[warp] = v; r.i[warp] = i; }
    __syncthreads();
    v = -1.0e30f;
    i = kNone;
    for (int w = 0; w < kShWarps; ++w)
        if (better_sh(r.f[w], r.i[w], v, i)) { v = r.f[w]; i = r.i[w]; }
    __syncthreads();
}

// Block-wide exclusive scan of one double per thread in thread order; the block total in
// *total (every thread).
__device__ double block_scan(ShRed& r, double v, double* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    if (lane == 31) r.d[warp] = inc;
    __syncthreads();
    double before = 0.0, all = 0.0;
    for (int w = 0; w < kShWarps; ++w) {
        if (w < warp) before += r.d[w];
        all += r.d[w];
    }
    __syncthreads();
    *total = all;
    return before + (inc - v);
}

// This CTA's id range inside the shard and this thread's sub-range.
struct Span {
    uint32_t cbeg, cend, tbeg, tend;
};
__device__ __forceinline__ Span my_span(uint32_t n, uint32_t split) {
    const uint32_t per = (n + split - 1) / split;
    Span s;
    s.cbeg = min(blockIdx.x * per, n);
    s.cend = min(s.cbeg + per, n);
    const uint32_t E = (per + kShThreads - 1) / kShThreads;
    s.tbeg = min(s.cbeg + threadIdx.x * E, s.cend);
    s.tend = min(s.tbeg + E, s.cend);
    return s;
}

// Unit u = rank * split + cta of row `row` in a gathered [world][rows][split] buffer.
__device__ __forceinline__ size_t gidx(uint32_t u, uint32_t row, uint32_t rows, uint32_t split) {
    return ((size_t)(u / split) * rows + row) * split + u % split;
}

// Tree of the current 8 bisection steps, suffix masses and the walked interval.
struct Walk {
    ToppTree t;
    fx62_t suffix[256];
    fx62_t wsum[8];
    float lo, hi;
};

// Replays 8 bisection steps from (lo, hi) on the gathered fixed-point bucket masses of the
// round that used that interval (k_topp.cuh).  Whole block; the new interval in w.lo / w.hi.
__device__ void walk(Walk& w, const fx62_t* bucket_all, uint32_t row, uint32_t rows, uint32_t units,
                     uint32_t split, float lo, float hi, float top_p) {
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) topp_build_tree_warp(w.t, lo, hi);
    if (threadIdx.x < 256) {
        fx62_t s = 0;
        for (uint32_t u = 0; u < units; ++u) s += bucket_all[gidx(u, row, rows, split) * 256 + threadIdx.x];
        const fx62_t v = topp_warp_suffix(s);
        w.suffix[threadIdx.x] = v;
        if (lane == 0) w.wsum[threadIdx.x >> 5] = v;
    }
    __syncthreads();
    if (threadIdx.x < 256) {
        fx62_t add = 0;
        for (int k = (threadIdx.x >> 5) + 1; k < 8; ++k) add += w.wsum[k];
        w.suffix[threadIdx.x] += add;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float l = lo, h = hi;
        topp_decide(w.t, w.suffix, top_p, l, h);
        w.lo = l;
        w.hi = h;
    }
    __syncthreads();
}

// Total of the gathered per-unit doubles of a row, units in order.
__device__ __forceinline__ double unit_total(const double* all, uint32_t row, uint32_t rows, uint32_t units,
                                             uint32_t split) {
    double t = 0.0;
    for (uint32_t u = 0; u < units; ++u) t += all[gidx(u, row, rows, split)];
    return t;
}

__global__ void __launch_bounds__(kShThreads) k_shard_prepare(float* logits_all, uint32_t n, uint32_t row_begin,
                                                              uint32_t split, const uint32_t* history,
                                                              uint32_t hstride, const uint32_t* hist_len,
                                                              const SampleRow* rows, uint32_t* cand) {
    const uint32_t row = blockIdx.y;
    const SampleRow P = rows[row];
    float* logits = logits_all + (size_t)row * n;
    extern __shared__ uint32_t bitmap[];  // one bit per id of this CTA's range
    __shared__ ShRed red;
    const Span S = my_span(n, split);
    if (P.repetition_penalty != 1.0f && history) {
        for (uint32_t w = threadIdx.x; w < (S.cend - S.cbeg + 31) / 32; w += kShThreads) bitmap[w] = 0u;
        __syncthreads();
        const uint32_t hl = hist_len ? hist_len[row] : hstride;
        const uint32_t* hist = history + (size_t)row * hstride;
        for (uint32_t h = threadIdx.x; h < hl; h += kShThreads) {
            const uint32_t id = hist[h];
            // another shard's or another CTA's id, or outside the vocabulary
            if (id < row_begin + S.cbeg || id >= row_begin + S.cend) continue;
            const uint32_t b = id - row_begin - S.cbeg, bit = 1u << (b & 31);
            if (atomicOr(&bitmap[b >> 5], bit) & bit) continue;  // already penalised
            const float v = logits[id - row_begin];
            logits[id - row_begin] = v > 0.0f ? v / P.repetition_penalty : v * P.repetition_penalty;
        }
        __syncthreads();
    }
    float gv = -1.0e30f, sv = -1.0e30f;
    uint32_t gi = kNone, si = kNone;
    for (uint32_t i = S.tbeg; i < S.tend; ++i) {
        const float v = logits[i];
        if (v > gv) { gv = v; gi = row_begin + i; }
        if (P.temperature > 0.0f) {
            const float s = v / P.temperature;
            if (s > sv) { sv = s; si = row_begin + i; }
        }
    }
    block_best(red, gv, gi);
    block_best(red, sv, si);
    if (threadIdx.x == 0) {
        uint32_t* c = cand + ((size_t)row * split + blockIdx.x) * 4;
        c[0] = __float_as_uint(gv);
        c[1] = gi;
        c[2] = __float_as_uint(sv);
        c[3] = si;
    }
}

__global__ void __launch_bounds__(kShThreads) k_shard_probs(const float* logits_all, uint32_t n, uint32_t split,
                                                            uint32_t world, const SampleRow* rows,
                                                            const uint32_t* cand_all, ShardState* state,
                                                            double* pbuf, double* sum) {
    const uint32_t row = blockIdx.y, nrows = gridDim.y;
    const float T = rows[row].temperature;
    __shared__ ShRed red;
    __shared__ float s_m;
    if (T <= 0.0f) {
        if (threadIdx.x == 0) sum[(size_t)row * split + blockIdx.x] = 0.0;
        return;
    }
    if (threadIdx.x == 0) {
        float bv = -1.0e30f;
        uint32_t bi = kNone;
        for (uint32_t u = 0; u < world * split; ++u) {
            const uint32_t* c = cand_all + gidx(u, row, nrows, split) * 4;
            const float v = __uint_as_float(c[2]);
            if (better_sh(v, c[3], bv, bi)) { bv = v; bi = c[3]; }
        }
        s_m = bv;
        if (blockIdx.x == 0) {
            state[row].gmax = bv;
            state[row].garg = bi == kNone ? 0u : bi;
            state[row].lohi[0][0] = 0.0f;
            state[row].lohi[0][1] = 1.0f;
        }
    }
    __syncthreads();
    const float* logits = logits_all + (size_t)row * n;
    double* p = pbuf + (size_t)row * n;
    const double m = (double)s_m;
    const Span S = my_span(n, split);
    double ls = 0.0;
    for (uint32_t i = S.tbeg; i < S.tend; ++i) {
        const double e = exp((double)(logits[i] / T) - m);
        p[i] = e;
        ls += e;
    }
    double total;
    block_scan(red, ls, &total);
    if (threadIdx.x == 0) sum[(size_t)row * split + blockIdx.x] = total;
}

__global__ void __launch_bounds__(kShThreads) k_shard_buckets(uint32_t n, uint32_t split, uint32_t world,
                                                              uint32_t round, const SampleRow* rows,
                                                              const double* sum_all, const fx62_t* bucket_prev,
                                                              ShardState* state, double* pbuf, fx62_t* bucket) {
    const uint32_t row = blockIdx.y, nrows = gridDim.y, units = world * split;
    const SampleRow P = rows[row];
    fx62_t* out = bucket + ((size_t)row * split + blockIdx.x) * 256;
    __shared__ Walk w;
    __shared__ fx62_t bk[kToppSubs * 256];
    __shared__ double s_sum;
    const Span S = my_span(n, split);
    double* p = pbuf + (size_t)row * n;
    if (P.temperature <= 0.0f) {
        for (int b = threadIdx.x; b < 256; b += kShThreads) out[b] = 0;
        return;
    }
    if (round == 0) {  // normalise by the vocabulary total, units in order
        if (threadIdx.x == 0) s_sum = unit_total(sum_all, row, nrows, units, split);
        __syncthreads();
        const double gs = s_sum;
        for (uint32_t i = S.tbeg; i < S.tend; ++i) p[i] = p[i] / gs;
    }
    if (P.top_p >= 1.0f) {
        for (int b = threadIdx.x; b < 256; b += kShThreads) out[b] = 0;
        return;
    }
    float lo = 0.0f, hi = 1.0f;
    if (round > 0) {
        walk(w, bucket_prev, row, nrows, units, split, state[row].lohi[round - 1][0], state[row].lohi[round - 1][1],
             P.top_p);
        lo = w.lo;
        hi = w.hi;
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            state[row].lohi[round][0] = lo;
            state[row].lohi[round][1] = hi;
        }
    }
    if (threadIdx.x < 32) topp_build_tree_warp(w.t, lo, hi);
    for (int b = threadIdx.x; b < kToppSubs * 256; b += kShThreads) bk[b] = 0;
    __syncthreads();
    topp_bucket_range(w.t, p, S.tbeg, S.tend, bk);
    __syncthreads();
    for (int b = threadIdx.x; b < 256; b += kShThreads) out[b] = topp_sub_total(bk, b);
}

__global__ void __launch_bounds__(kShThreads) k_shard_kept(uint32_t n, uint32_t split, uint32_t world,
                                                           uint32_t rounds, const SampleRow* rows,
                                                           const double* sum_all, const fx62_t* bucket_last,
                                                           ShardState* state, double* pbuf, double* kept) {
    const uint32_t row = blockIdx.y, nrows = gridDim.y, units = world * split;
    const SampleRow P = rows[row];
    __shared__ Walk w;
    __shared__ ShRed red;
    __shared__ double s_sum;
    double* p = pbuf + (size_t)row * n;
    const Span S = my_span(n, split);
    if (P.temperature <= 0.0f) {
        if (threadIdx.x == 0) kept[(size_t)row * split + blockIdx.x] = 0.0;
        return;
    }
    if (rounds == 0) {  // no bucket pass ran: normalise here
        if (threadIdx.x == 0) s_sum = unit_total(sum_all, row, nrows, units, split);
        __syncthreads();
        const double gs = s_sum;
        for (uint32_t i = S.tbeg; i < S.tend; ++i) p[i] = p[i] / gs;
    }
    double thr = 0.0;
    if (P.top_p < 1.0f && rounds > 0) {
        walk(w, bucket_last, row, nrows, units, split, state[row].lohi[rounds - 1][0],
             state[row].lohi[rounds - 1][1], P.top_p);
        thr = (double)w.lo;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) state[row].thr = thr;
    double mine = 0.0;
    for (uint32_t i = S.tbeg; i < S.tend; ++i)
        if (p[i] >= thr) mine += p[i];
    double total;
    block_scan(red, mine, &total);
    if (threadIdx.x == 0) kept[(size_t)row * split + blockIdx.x] = total;
}

__global__ void __launch_bounds__(kShThreads) k_shard_pick(uint32_t n, uint32_t row_begin, uint32_t split,
                                                           uint32_t world, uint32_t rank, const SampleRow* rows,
                                                           const double* kept_all, const ShardState* state,
                                                           const double* pbuf, uint32_t* pick) {
    const uint32_t row = blockIdx.y, nrows = gridDim.y, units = world * split;
    const SampleRow P = rows[row];
    __shared__ ShRed red;
    __shared__ double s_off, s_target;
    __shared__ uint32_t best;
    uint32_t* out = pick + (size_t)row * split + blockIdx.x;
    if (P.temperature <= 0.0f) {
        if (threadIdx.x == 0) *out = kNone;
        return;
    }
    if (threadIdx.x == 0) {
        const uint32_t me = rank * split + blockIdx.x;
        double before = 0.0, all = 0.0;
        for (uint32_t u = 0; u < units; ++u) {
            const double v = kept_all[gidx(u, row, nrows, split)];
            if (u < me) before += v;
            all += v;
        }
        s_off = before;
        s_target = (double)P.random * fmax(all, 1.0e-20);
        best = kNone;
    }
    __syncthreads();
    const double* p = pbuf + (size_t)row * n;
    const double thr = state[row].thr, target = s_target;
    const Span S = my_span(n, split);
    double mine = 0.0;
    for (uint32_t i = S.tbeg; i < S.tend; ++i)
        if (p[i] >= thr) mine += p[i];
    double total;
    double running = s_off + block_scan(red, mine, &total);
    for (uint32_t i = S.tbeg; i < S.tend; ++i) {
        if (p[i] >= thr) {
            running += p[i];
            if (running >= target) {
                atomicMin(&best, row_begin + i);
                break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *out = best;
}

__global__ void k_shard_finish(uint32_t nrows, uint32_t split, uint32_t world, const SampleRow* rows,
                               const uint32_t* cand_all, const uint32_t* pick_all, const ShardState* state,
                               uint32_t* out) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= nrows) return;
    const uint32_t units = world * split;
    if (rows[row].temperature <= 0.0f) {
        float bv = -1.0e30f;
        uint32_t bi = kNone;
        for (uint32_t u = 0; u < units; ++u) {
            const uint32_t* c = cand_all + gidx(u, row, nrows, split) * 4;
            const float v = __uint_as_float(c[0]);
            if (better_sh(v, c[1], bv, bi)) { bv = v; bi = c[1]; }
        }
        out[row] = bi == kNone ? 0u : bi;
        return;
    }
    uint32_t best = kNone;
    for (uint32_t u = 0; u < units; ++u) best = min(best, pick_all[gidx(u, row, nrows, split)]);
    out[row] = best == kNone ? state[row].garg : best;
}

}  // namespace

}  // namespace enx

using namespace enx;

namespace {

enx_status sh_launched(const char* who) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ENX_OK : cuda_fail(e, who);
}

bool sh_dims_ok(uint32_t n, uint32_t rows, uint32_t split, uint32_t world) {
    return n > 0 && rows > 0 && rows <= 65535 && split > 0 && split <= 64 && world > 0 && world <= 64;
}

}  // namespace

extern "C" size_t enx_shard_state_bytes(uint32_t rows) { return (size_t)rows * sizeof(ShardState); }

extern "C" enx_status enx_shard_prepare(float* logits, uint32_t n, uint32_t row_begin, uint32_t rows, uint32_t split,
                                        const uint32_t* history, uint32_t history_stride,
                                        const uint32_t* history_length, const enx_sampling_row* params,
                                        uint32_t* cand, void* stream) {
    if (!logits || !params || !cand) return fail(ENX_ERR_INVALID, "enx_shard_prepare: null pointer");
    if (!sh_dims_ok(n, rows, split, 1)) return fail(ENX_ERR_RANGE, "enx_shard_prepare: bad dimensions");
    const uint32_t per = (n + split - 1) / split;
    const size_t smem = ((size_t)per + 31) / 32 * 4;
    if (smem > 160 * 1024) return fail(ENX_ERR_RANGE, "enx_shard_prepare: shard too large for one split");
    cudaError_t e = cudaFuncSetAttribute(k_shard_prepare, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "enx_shard_prepare");
    k_shard_prepare<<<dim3(split, rows), kShThreads, smem, as_stream(stream)>>>(
        logits, n, row_begin, split, history, history_stride, history_length,
        reinterpret_cast<const SampleRow*>(params), cand);
    return sh_launched("enx_shard_prepare");
}

extern "C" enx_status enx_shard_probs(const float* logits, uint32_t n, uint32_t rows, uint32_t split,
                                      uint32_t world, const enx_sampling_row* params, const uint32_t* cand_all,
                                      void* state, double* probs, double* sum, void* stream) {
    if (!logits || !params || !cand_all || !state || !probs || !sum)
        return fail(ENX_ERR_INVALID, "enx_shard_probs: null pointer");
    if (!sh_dims_ok(n, rows, split, world)) return fail(ENX_ERR_RANGE, "enx_shard_probs: bad dimensions");
    k_shard_probs<<<dim3(split, rows), kShThreads, 0, as_stream(stream)>>>(
        logits, n, split, world, reinterpret_cast<const SampleRow*>(params), cand_all,
        static_cast<ShardState*>(state), probs, sum);
    return sh_launched("enx_shard_probs");
}

extern "C" enx_status enx_shard_buckets(uint32_t n, uint32_t rows, uint32_t split, uint32_t world, uint32_t round,
                                        const enx_sampling_row* params, const double* sum_all,
                                        const uint64_t* bucket_prev, void* state, double* probs, uint64_t* bucket,
                                        void* stream) {
    if (!params || !state || !probs || !bucket || (round == 0 && !sum_all) || (round > 0 && !bucket_prev))
        return fail(ENX_ERR_INVALID, "enx_shard_buckets: null pointer");
    if (!sh_dims_ok(n, rows, split, world) || round > 3)
        return fail(ENX_ERR_RANGE, "enx_shard_buckets: bad dimensions");
    k_shard_buckets<<<dim3(split, rows), kShThreads, 0, as_stream(stream)>>>(
        n, split, world, round, reinterpret_cast<const SampleRow*>(params), sum_all,
        reinterpret_cast<const fx62_t*>(bucket_prev), static_cast<ShardState*>(state), probs,
        reinterpret_cast<fx62_t*>(bucket));
    return sh_launched("enx_shard_buckets");
}

extern "C" enx_status enx_shard_kept(uint32_t n, uint32_t rows, uint32_t split, uint32_t world, uint32_t rounds,
                                     const enx_sampling_row* params, const double* sum_all,
                                     const uint64_t* bucket_last, void* state, double* probs, double* kept,
                                     void* stream) {
    if (!params || !state || !probs || !kept || (rounds == 0 && !sum_all) || (rounds > 0 && !bucket_last))
        return fail(ENX_ERR_INVALID, "enx_shard_kept: null pointer");
    if (!sh_dims_ok(n, rows, split, world) || (rounds != 0 && rounds != 4))
        return fail(ENX_ERR_RANGE, "enx_shard_kept: rounds must be 0 or 4");
    k_shard_kept<<<dim3(split, rows), kShThreads, 0, as_stream(stream)>>>(
        n, split, world, rounds, reinterpret_cast<const SampleRow*>(params), sum_all,
        reinterpret_cast<const fx62_t*>(bucket_last), static_cast<ShardState*>(state), probs, kept);
    return sh_launched("enx_shard_kept");
}

extern "C" enx_status enx_shard_pick(uint32_t n, uint32_t row_begin, uint32_t rows, uint32_t split, uint32_t world,
                                     uint32_t rank, const enx_sampling_row* params, const double* kept_all,
                                     const void* state, const double* probs, uint32_t* pick, void* stream) {
    if (!params || !kept_all || !state || !probs || !pick)
        return fail(ENX_ERR_INVALID, "enx_shard_pick: null pointer");
    if (!sh_dims_ok(n, rows, split, world) || rank >= world)
        return fail(ENX_ERR_RANGE, "enx_shard_pick: bad dimensions");
    k_shard_pick<<<dim3(split, rows), kShThreads, 0, as_stream(stream)>>>(
        n, row_begin, split, world, rank, reinterpret_cast<const SampleRow*>(params), kept_all,
        static_cast<const ShardState*>(state), probs, pick);
    return sh_launched("enx_shard_pick");
}

extern "C" enx_status enx_shard_finish(uint32_t rows, uint32_t split, uint32_t world, const enx_sampling_row* params,
                                       const uint32_t* cand_all, const uint32_t* pick_all, const void* state,
                                       uint32_t* out, void* stream) {
    if (!params || !cand_all || !pick_all || !state || !out)
        return fail(ENX_ERR_INVALID, "enx_shard_finish: null pointer");
    if (!sh_dims_ok(1, rows, split, world)) return fail(ENX_ERR_RANGE, "enx_shard_finish: bad dimensions");
    k_shard_finish<<<(rows + 127) / 128, 128, 0, as_stream(stream)>>>(
        rows, split, world, reinterpret_cast<const SampleRow*>(params), cand_all, pick_all,
        static_cast<const ShardState*>(state), out);
    return sh_launched("enx_shard_finish");
}
