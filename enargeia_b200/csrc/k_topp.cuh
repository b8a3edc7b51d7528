// Top-p bisection helpers shared by the single-GPU sampler (k_sample.cu) and the vocab-sharded
// sampler (k_shard.cu).
//
// The reference bisects the threshold 32 times on f32 midpoints, each step deciding
// mass(p >= mid) < top_p (src/kernels/sample.wgsl:241-262).  Eight steps at a time form a binary
// tree of 255 midpoints fixed by the current (lo, hi); one pass over the probabilities buckets
// every p by the tree's sorted thresholds (bucket = number of thresholds <= p), suffix sums of the
// bucket masses give mass(p >= t) at every node, and walking the tree replays the 8 decisions.
//
// Bucket masses are 62-bit fixed point, round(p * 2^62) (p <= 1): integer adds are exact and
// order-free, so one shared-memory atomic per element replaces any warp aggregation and the
// totals are the same on every run, every CTA split and every rank split.  mass < top_p is
// decided as fixed-point mass < round(top_p * 2^62).
#pragma once

#include <cstdint>

namespace enx {

typedef unsigned long long fx62_t;

__device__ __forceinline__ fx62_t fx62(double p) { return __double2ull_rn(p * 4611686018427387904.0); }

__device__ __forceinline__ int topp_inorder_rank(int n) {
    const int d = 31 - __clz(n);
    return (2 * (n - (1 << d)) + 1) << (7 - d);
}

struct ToppTree {
    float tl[256], th[256], mids[256];  // heap-indexed node intervals and midpoints, 1..255
    double thr[256];                    // sorted thresholds thr[1..255]
};

// One warp (all 32 lanes): the tree of the next 8 midpoints from (lo, hi), level by level, and
// its sorted listing.
__device__ inline void topp_build_tree_warp(ToppTree& t, float lo, float hi) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
        t.tl[1] = lo;
        t.th[1] = hi;
    }
    __syncwarp();
    for (int d = 0; d < 8; ++d) {
        for (int n = (1 << d) + lane; n < (2 << d); n += 32) {
            const float mid = (t.tl[n] + t.th[n]) * 0.5f;
            t.mids[n] = mid;
            t.thr[topp_inorder_rank(n)] = (double)mid;
            if (n < 128) {
                t.tl[2 * n] = t.tl[n]; t.th[2 * n] = mid;
                t.tl[2 * n + 1] = mid; t.th[2 * n + 1] = t.th[n];
            }
        }
        __syncwarp();
    }
}

// Sub-histograms a CTA spreads its bucket atomics over (warp % kToppSubs): with flat
// distributions most elements of a round fall into a few buckets, and one shared copy
// serialises them.
constexpr int kToppSubs = 8;

// Adds the fixed-point masses of p[i], i in [beg, end), to bk[bucket] of this warp's
// sub-histogram (shared, kToppSubs x 256 entries; sum them with topp_sub_total).  Whole warps:
// masses below the first threshold and from the last one up are summed per warp and added once.
__device__ __forceinline__ void topp_bucket_range(const ToppTree& t, const double* p, uint32_t beg, uint32_t end,
                                                  fx62_t* bk_subs) {
    fx62_t* bk = bk_subs + ((threadIdx.x >> 5) % kToppSubs) * 256;
    const double tlo = t.thr[1], thi = t.thr[255];
    fx62_t below = 0, above = 0;
    for (uint32_t i = beg; i < end; ++i) {
        const double v = p[i];
        const fx62_t f = fx62(v);
        if (v < tlo) below += f;
        else if (v >= thi) above += f;
        else {
            int bb = 0;
#pragma unroll
            for (int step = 128; step >= 1; step >>= 1)
                if (t.thr[bb + step] <= v) bb += step;
            atomicAdd(&bk[bb], f);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        below += __shfl_xor_sync(0xffffffffu, below, o);
        above += __shfl_xor_sync(0xffffffffu, above, o);
    }
    if ((threadIdx.x & 31) == 0) {
        if (below) atomicAdd(&bk[0], below);
        if (above) atomicAdd(&bk[255], above);
    }
}

// Bucket b's total over the sub-histograms (integers: exact in any order).
__device__ __forceinline__ fx62_t topp_sub_total(const fx62_t* bk_subs, int b) {
    fx62_t s = 0;
#pragma unroll
    for (int k = 0; k < kToppSubs; ++k) s += bk_subs[k * 256 + b];
    return s;
}

// Suffix sum within a warp of 32 consecutive buckets (lane l gets the sum of lanes l..31).
__device__ __forceinline__ fx62_t topp_warp_suffix(fx62_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const fx62_t n = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += n;
    }
    return v;
}

// One thread: the 8 decisions from (lo, hi) given suffix[r] = mass(p >= thr[r]); the new
// interval in lo, hi.
__device__ inline void topp_decide(const ToppTree& t, const fx62_t* suffix, float top_p, float& lo, float& hi) {
    const fx62_t goal = fx62((double)top_p);
    float l = lo, h = hi;
    int n = 1;
    for (int step = 0; step < 8; ++step) {
        if (suffix[topp_inorder_rank(n)] < goal) { h = t.mids[n]; n = 2 * n; }
        else { l = t.mids[n]; n = 2 * n + 1; }
    }
    lo = l;
    hi = h;
}

}  // namespace enx
