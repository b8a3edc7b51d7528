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
//     mass(p >= mid) < top_p.  The next 8 midpoints form a binary tree fixed by (lo, hi); one
//     pass buckets every p by the tree's 255 sorted thresholds, suffix sums of the bucket masses
//     give mass(p >= t) at every node, and walking the tree replays the 8 decisions exactly.
//     Four passes replace 32 reductions.
//  6. kept = sum of p >= threshold; target = random * max(kept, 1e-20); the first id in
//     ascending order whose running kept-mass reaches the target wins (argmax if none).
// Probabilities, masses and running totals are doubles (the oracle's exact-arithmetic rule).

#include <cooperative_groups.h>

#include "enx_internal.cuh"
#include "k_small.cuh"

namespace cg = cooperative_groups;

namespace enx {

constexpr int kCluster = 8;
constexpr int kSThreads = 1024;
constexpr int kSWarps = kSThreads / 32;
constexpr uint32_t kMaxPer = 26624;  // ids per CTA kept on chip: 8 bytes each

uint32_t sample_max_vocab() { return kMaxPer * kCluster; }

struct SampleSmem {
    double bucket[256];     // bucket masses of this CTA (then of the cluster)
    double thr[256];        // sorted tree thresholds, thr[1..255]
    float mids[256];        // tree midpoints by heap index 1..255
    double wred[kSWarps];
    float fred[kSWarps];
    uint32_t ired[kSWarps];
    double cta_d[4];        // published per-CTA doubles (sum / kept)
    float cta_f;            // published per-CTA max
    uint32_t cta_i;         // published per-CTA argmax / crossing id
    float lo, hi;
    double suffix[257];
    float tl[256], th[256];  // tree interval bounds by heap index
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

    // ---- 5. top-p threshold: 4 passes x 8 bisection steps --------------------------------
    float lo = 0.0f, hi = 1.0f;
    if (P.top_p < 1.0f) {
        for (int round = 0; round < 4; ++round) {
            if (threadIdx.x == 0) {
                // heap-indexed tree of the next 8 midpoints, and its in-order (sorted) listing
                float* L = sm.tl;
                float* Hh = sm.th;
                L[1] = lo; Hh[1] = hi;
                for (int n = 1; n < 256; ++n) {
                    float mid = (L[n] + Hh[n]) * 0.5f;
                    sm.mids[n] = mid;
                    if (n < 128) {
                        L[2 * n] = L[n]; Hh[2 * n] = mid;
                        L[2 * n + 1] = mid; Hh[2 * n + 1] = Hh[n];
                    }
                }
                // in-order rank of heap node n at depth d (0-based): (2*(n - 2^d) + 1) * 2^(7-d)
                for (int n = 1; n < 256; ++n) {
                    int d = 31 - __clz(n);
                    int rnk = (2 * (n - (1 << d)) + 1) << (7 - d);
                    sm.thr[rnk] = (double)sm.mids[n];
                }
            }
            for (int b = threadIdx.x; b < 256; b += kSThreads) sm.bucket[b] = 0.0;
            __syncthreads();
            const double tlo = sm.thr[1], thi = sm.thr[255];
            double below = 0.0, above = 0.0;
            const int lane = threadIdx.x & 31;
            for (uint32_t k = 0; k < E; ++k) {
                uint32_t i = tbeg + k;
                bool valid = i < tend;
                double p = valid ? pbuf[i - cbeg] : 0.0;
                int b = -1;  // -1: no shared-memory update needed
                if (valid) {
                    if (p < tlo) below += p;
                    else if (p >= thi) above += p;
                    else {
                        int bb = 0;
#pragma unroll
                        for (int step = 128; step >= 1; step >>= 1)
                            if (sm.thr[bb + step] <= p) bb += step;
                        b = bb;
                    }
                }
                // aggregate equal buckets across the warp before touching shared memory
                unsigned pending = __ballot_sync(0xffffffffu, b >= 0);
                while (pending) {
                    int leader = __ffs(pending) - 1;
                    int lb = __shfl_sync(0xffffffffu, b, leader);
                    bool mine = (b == lb) && ((pending >> lane) & 1u);
                    double contrib = warp_sum_d(mine ? p : 0.0);
                    if (lane == leader) atomicAdd(&sm.bucket[lb], contrib);
                    pending &= ~__ballot_sync(0xffffffffu, mine);
                }
            }
            double tb = block_sum_d(sm, below);
            double ta = block_sum_d(sm, above);
            if (threadIdx.x == 0) { sm.bucket[0] += tb; sm.bucket[255] += ta; }
            cluster.sync();
            // cluster bucket totals (a thread per bucket, ranks in order), then suffix sums
            // mass(p >= thr[j]): within each warp of 32 buckets, then the warps above added on
            if (threadIdx.x < 256) {
                double t = 0.0;
                for (int r = 0; r < kCluster; ++r) t += cluster.map_shared_rank(&sm, r)->bucket[threadIdx.x];
                double v = t;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double n = __shfl_down_sync(0xffffffffu, v, o);
                    if (lane + o < 32) v += n;
                }
                sm.suffix[threadIdx.x] = v;
                if (lane == 0) sm.wred[threadIdx.x >> 5] = v;
            }
            __syncthreads();
            if (threadIdx.x < 256) {
                double add = 0.0;
                for (int w = (threadIdx.x >> 5) + 1; w < 8; ++w) add += sm.wred[w];
                sm.suffix[threadIdx.x] += add;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float l = lo, h = hi;
                int n = 1;
                for (int step = 0; step < 8; ++step) {
                    int d = 31 - __clz(n);
                    int rnk = (2 * (n - (1 << d)) + 1) << (7 - d);
                    // p >= mid  <=>  bucket >= rank  (thresholds sorted, bucket = #thr <= p)
                    double mass = sm.suffix[rnk];
                    if (mass < (double)P.top_p) { h = sm.mids[n]; n = 2 * n; }
                    else { l = sm.mids[n]; n = 2 * n + 1; }
                }
                sm.lo = l;
                sm.hi = h;
            }
            cluster.sync();  // all CTAs done reading bucket[] before the next round clears it
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
