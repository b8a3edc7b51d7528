// GPU sampler: the semantics of src/kernels/sample.wgsl:91-331, rebuilt for a thread-block
// cluster.
//
// One cluster of kCluster CTAs x 1024 threads samples one row.  CTA c owns the contiguous id
// range [c*per, (c+1)*per) and thread t of it a contiguous sub-range, so "concatenate the
// ranges in rank order" is ascending token id, which the draw depends on.  All cross-CTA
// exchange is distributed shared memory behind cluster barriers (hardware barriers, no spin).
//
// Steps, in the reference's order:
//  1. repetition penalty, in place, once per DISTINCT history id (first occurrence wins a
//     test-and-set bit in a per-CTA bitmap): logit > 0 ? logit / rp : logit * rp  (f32)
//  2. temperature <= 0: argmax of the penalised logits, ties to the lowest id, from -1e30
//  3. s = logit / T (f32); m = max s, its argmax (ties lowest) is the fallback
//  4. p = exp(s - m) / sum exp(s - m), in double, kept in shared memory
//  5. top_p < 1: the reference's 32 bisection steps on f32 midpoints, deciding
//     mass(p >= mid) < top_p, as four passes of 8 steps each (k_topp.cuh: a tree of midpoints,
//     fixed-point bucket masses, suffix sums, the 8 decisions replayed).
//  6. kept = sum of p >= threshold; target = random * max(kept, 1e-20); the first id in
//     ascending order whose running kept-mass reaches the target wins (argmax if none).
// Probabilities, kept masses and running totals are doubles (the oracle's exact-arithmetic
// rule); bisection masses are exact 62-bit fixed point.

#include <cooperative_groups.h>

#include "enx_internal.cuh"
#include "k_small.cuh"
#include "k_topp.cuh"

namespace cg = cooperative_groups;

namespace enx {

constexpr int kCluster = 8;
constexpr int kSThreads = 1024;
constexpr int kSWarps = kSThreads / 32;
constexpr uint32_t kMaxPer = 25344;  // ids per CTA kept on chip: 8 bytes each (+ 26 KB static, within 227 KB)

uint32_t sample_max_vocab() { return kMaxPer * kCluster; }

struct SampleSmem {
    fx62_t bucket[kToppSubs * 256];  // fixed-point bucket masses of this CTA (sub-histograms)
    fx62_t ctab[256];                // their totals, read by the cluster
    fx62_t suffix[256];     // cluster suffix masses mass(p >= thr[j])
    fx62_t wsum[8];
    ToppTree tree;          // midpoints of the current 8 bisection steps
    double wred[kSWarps];
    float fred[kSWarps];
    uint32_t ired[kSWarps];
    double cta_d[4];        // published per-CTA doubles (sum / kept)
    float cta_f;            // published per-CTA max
    uint32_t cta_i;         // published per-CTA argmax / crossing id
    float lo, hi;
};

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// Block-wide (max, lowest index) over 1024 threads.  Result valid in thread 0.
__device__ void block_argmax(SampleSmem& sm, float& v, uint32_t& i) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, v, o);
        uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    if (lane == 0) { sm.fred[warp] = v; sm.ired[warp] = i; }
    __syncthreads();
    if (warp == 0) {
        v = sm.fred[lane];
        i = sm.ired[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, v, o);
            uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (better(ov, oi, v, i)) { v = ov; i = oi; }
        }
    }
    __syncthreads();
}

__device__ double block_sum_d(SampleSmem& sm, double v) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_d(v);
    if (lane == 0) sm.wred[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < kSWarps; ++w) t += sm.wred[w];
    __syncthreads();
    return t;  // valid in thread 0
}

// Exclusive scan of one double per thread in thread order; returns this thread's offset and the
// block total in *total (all threads).
__device__ double block_exclusive_scan_d(SampleSmem& sm, double v, double* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    if (lane == 31) sm.wred[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        double w = sm.wred[lane];
        double winc = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double n = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += n;
        }
        sm.wred[lane] = winc - w;  // exclusive warp offsets
        if (lane == 31) sm.cta_d[3] = winc;
    }
    __syncthreads();
    double off = sm.wred[warp] + (inc - v);
    *total = sm.cta_d[3];
    __syncthreads();
    return off;
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kSThreads, 1)
    k_sample(float* __restrict__ logits_all, uint32_t vocab, const uint32_t* __restrict__ history,
             uint32_t history_stride, const uint32_t* __restrict__ hist_len, const SampleRow* rows,
             int rows_shared, SampleRow row0, uint32_t* __restrict__ out) {
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint32_t row = blockIdx.x / kCluster;
    __shared__ SampleSmem sm;
    extern __shared__ double pbuf[];  // [per] probabilities, then the penalty bitmap after it
    pdl_launch_dependents();
    pdl_wait();

    const SampleRow P = rows ? rows[rows_shared ? 0 : row] : row0;
    float* logits = logits_all + (size_t)row * vocab;
    const uint32_t per = (vocab + kCluster - 1) / kCluster;
    const uint32_t cbeg = min(rank * per, vocab), cend = min(cbeg + per, vocab);
    const uint32_t E = (per + kSThreads - 1) / kSThreads;
    const uint32_t tbeg = min(cbeg + threadIdx.x * E, cend), tend = min(tbeg + E, cend);
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(pbuf + per);
    const uint32_t nwords = (per + 31) / 32;

    // ---- 1. repetition penalty (in place, first occurrence only) -------------------------
    if (P.repetition_penalty != 1.0f) {
        for (uint32_t w = threadIdx.x; w < nwords; w += kSThreads) bitmap[w] = 0u;
        __syncthreads();
        const uint32_t hl = hist_len ? hist_len[row] : history_stride;
        const uint32_t* hist = history + (size_t)row * history_stride;
        for (uint32_t h = threadIdx.x; h < hl; h += kSThreads) {
            uint32_t id = hist[h];
            if (id < cbeg || id >= cend) continue;  // another CTA's range, or out of vocab
            uint32_t b = id - cbeg, bit = 1u << (b & 31);
            if (atomicOr(&bitmap[b >> 5], bit) & bit) continue;  // already penalised
            float v = logits[id];
            logits[id] = v > 0.0f ? v / P.repetition_penalty : v * P.repetition_penalty;
        }
        __syncthreads();
    }

    // ---- 2. greedy --------------------------------------------------------------------------
    if (P.temperature <= 0.0f) {
        float bv = -1.0e30f;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t i = tbeg; i < tend; ++i) {
            float v = logits[i];
            if (v > bv) { bv = v; bi = i; }
        }
        block_argmax(sm, bv, bi);
        if (threadIdx.x == 0) { sm.cta_f = bv; sm.cta_i = bi; }
        cluster.sync();
        if (rank == 0 && threadIdx.x == 0) {
            float gv = -1.0e30f;
            uint32_t gi = 0xFFFFFFFFu;
            for (int r = 0; r < kCluster; ++r) {
                SampleSmem* o = cluster.map_shared_rank(&sm, r);
                if (better(o->cta_f, o->cta_i, gv, gi)) { gv = o->cta_f; gi = o->cta_i; }
            }
            out[row] = gi == 0xFFFFFFFFu ? 0u : gi;
        }
        cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
        return;
    }

    // ---- 3. scaled logits, max and argmax -------------------------------------------------
    const float T = P.temperature;
    float bv = -1.0e30f;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = tbeg; i < tend; ++i) {
        float s = logits[i] / T;
        if (s > bv) { bv = s; bi = i; }
    }
    block_argmax(sm, bv, bi);
    if (threadIdx.x == 0) { sm.cta_f = bv; sm.cta_i = bi; }
    cluster.sync();
    __shared__ float gmax;
    __shared__ uint32_t garg;
    if (threadIdx.x == 0) {
        float gv = -1.0e30f;
        uint32_t gi = 0xFFFFFFFFu;
        for (int r = 0; r < kCluster; ++r) {
            SampleSmem* o = cluster.map_shared_rank(&sm, r);
            if (better(o->cta_f, o->cta_i, gv, gi)) { gv = o->cta_f; gi = o->cta_i; }
        }
        gmax = gv;
        garg = gi == 0xFFFFFFFFu ? 0u : gi;
    }
    __syncthreads();
    const double m = (double)gmax;

    // ---- 4. probabilities ----------------------------------------------------------------
    double ls = 0.0;
    for (uint32_t i = tbeg; i < tend; ++i) {
        double e = exp((double)(logits[i] / T) - m);
        pbuf[i - cbeg] = e;
        ls += e;
    }
    double cs = block_sum_d(sm, ls);
    cluster.sync();  // everyone finished reading the previous cta_* values
    if (threadIdx.x == 0) sm.cta_d[0] = cs;
    cluster.sync();
    __shared__ double gsum;
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int r = 0; r < kCluster; ++r) t += cluster.map_shared_rank(&sm, r)->cta_d[0];
        gsum = t;
    }
    __syncthreads();
    for (uint32_t i = tbeg; i < tend; ++i) pbuf[i - cbeg] = pbuf[i - cbeg] / gsum;

    // ---- 5. top-p threshold: 4 passes x 8 bisection steps (k_topp.cuh) --------------------
    float lo = 0.0f, hi = 1.0f;
    if (P.top_p < 1.0f) {
        const int lane = threadIdx.x & 31;
        for (int round = 0; round < 4; ++round) {
            if (threadIdx.x < 32) topp_build_tree_warp(sm.tree, lo, hi);
            for (int b = threadIdx.x; b < kToppSubs * 256; b += kSThreads) sm.bucket[b] = 0;
            __syncthreads();
            topp_bucket_range(sm.tree, pbuf, tbeg - cbeg, tend - cbeg, sm.bucket);
            __syncthreads();
            if (threadIdx.x < 256) sm.ctab[threadIdx.x] = topp_sub_total(sm.bucket, threadIdx.x);
            cluster.sync();
            // cluster bucket totals (a thread per bucket), then suffix masses: within each warp of
            // 32 buckets, then the warps above added on (integers: exact in any order)
            if (threadIdx.x < 256) {
                fx62_t t = 0;
                for (int r = 0; r < kCluster; ++r) t += cluster.map_shared_rank(&sm, r)->ctab[threadIdx.x];
                const fx62_t v = topp_warp_suffix(t);
                sm.suffix[threadIdx.x] = v;
                if (lane == 0) sm.wsum[threadIdx.x >> 5] = v;
            }
            __syncthreads();
            if (threadIdx.x < 256) {
                fx62_t add = 0;
                for (int w = (threadIdx.x >> 5) + 1; w < 8; ++w) add += sm.wsum[w];
                sm.suffix[threadIdx.x] += add;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float l = lo, h = hi;
                topp_decide(sm.tree, sm.suffix, P.top_p, l, h);
                sm.lo = l;
                sm.hi = h;
            }
            cluster.sync();  // all CTAs done reading ctab[] before the next round rewrites it
            lo = sm.lo;
            hi = sm.hi;
        }
    }
    const double thr = P.top_p < 1.0f ? (double)lo : 0.0;

    // ---- 6. kept mass and the draw -------------------------------------------------------
    double mine = 0.0;
    for (uint32_t i = tbeg; i < tend; ++i) {
        double p = pbuf[i - cbeg];
        if (p >= thr) mine += p;
    }
    double cta_total;
    double off = block_exclusive_scan_d(sm, mine, &cta_total);
    if (threadIdx.x == 0) { sm.cta_d[1] = cta_total; sm.cta_i = 0xFFFFFFFFu; }
    cluster.sync();
    __shared__ double cta_off, target;
    if (threadIdx.x == 0) {
        double before = 0.0, kept = 0.0;
        for (int r = 0; r < kCluster; ++r) {
            double v = cluster.map_shared_rank(&sm, r)->cta_d[1];
            if ((uint32_t)r < rank) before += v;
            kept += v;
        }
        cta_off = before;
        target = (double)P.random * fmax(kept, 1.0e-20);
    }
    __syncthreads();
    double running = cta_off + off;
    for (uint32_t i = tbeg; i < tend; ++i) {
        double p = pbuf[i - cbeg];
        if (p >= thr) {
            running += p;
            if (running >= target) {
                atomicMin(&sm.cta_i, i);
                break;
            }
        }
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        uint32_t pick = 0xFFFFFFFFu;
        for (int r = 0; r < kCluster; ++r) pick = min(pick, cluster.map_shared_rank(&sm, r)->cta_i);
        out[row] = pick == 0xFFFFFFFFu ? garg : pick;
    }
    cluster.sync();
}

cudaError_t launch_sample(float* logits, uint32_t vocab, uint32_t batch, const uint32_t* history,
                          uint32_t history_stride, const uint32_t* hist_len, const SampleRow* rows,
                          bool rows_shared, SampleRow row0, uint32_t* out, cudaStream_t st,
                          bool pdl) {
    const uint32_t per = (vocab + kCluster - 1) / kCluster;
    const size_t smem = (size_t)per * 8 + ((per + 31) / 32) * 4;
    cudaError_t e = cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster * batch);
    cfg.blockDim = dim3(kSThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_sample, logits, vocab, history, history_stride, hist_len, rows,
                              (int)rows_shared, row0, out);
}

}  // namespace enx
