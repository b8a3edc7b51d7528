// Dequantise-in-registers matvec core for the int4 projections and the int8 tied head.
//
// Weight layout is the .enargeia layout, unchanged (verbatim upload): row r of an N x K tensor
// is K/8 (int4) or K/4 (int8) u32 words, reduction axis contiguous, low bits first; one f32
// scale per 64-element block; zero-points packed 8 (int4) or 4 (int8) per u32 word, block index
// r*(K/64) + k/64.
//
// Arithmetic is faithful to the reference's CPU path (test/reference/quant.ts:95-112): products
// and sums in double, the result rounded to float once.  This is not a luxury: K and V are
// rounded to f16 in the cache, and a float-accumulated projection that differs from the f64
// reference in the last bit lands on the other side of an f16 rounding boundary often enough to
// move logits by ~1e-4 after a few layers.  Done this way the device results match the CPU
// reference except where an f64 sum taken in a different order rounds differently (about one
// value in 10^8).
//
// Work split: a "chunk" is 16 bytes of packed codes (32 int4 or 16 int8 elements).  Lane l of a
// warp handles chunks l, l+32, ... of the row it is on, so a row is read with coalesced 16-byte
// loads.  Activations sit in shared memory as doubles transposed by chunk
// (XD[(t*F2 + j)*nchunk + c] = x[t][c*E + 2j .. 2j+1]) so the lanes' 16-byte reads are
// conflict-free.  A code becomes an exact double with the 2^52 exponent trick, (q - z) is exact,
// and each chunk contributes s * sum_j (q_j - z) * x_j (four interleaved partial sums).
#pragma once

#include "enx_internal.cuh"

namespace enx {

struct QW {
    const uint32_t* packed;
    const float* scales;
    const uint32_t* zeros;
    uint32_t rows, cols;
};

template <int BITS>
struct Geom {
    static constexpr int E = BITS == 4 ? 32 : 16;   // elements per 16-byte chunk
    static constexpr int F2 = E / 2;                // double2 of x per chunk
    static constexpr int CPB = kBlock / E;          // chunks per quantisation block
};

template <int BITS>
__device__ __forceinline__ uint32_t zero_code(const uint32_t* zeros, uint32_t blk) {
    if (BITS == 4) return (__ldg(zeros + (blk >> 3)) >> ((blk & 7u) * 4u)) & 0xFu;
    return (__ldg(zeros + (blk >> 2)) >> ((blk & 3u) * 8u)) & 0xFFu;
}

// Block barrier of the helpers below: NT == 0 is __syncthreads(); otherwise named barrier 1 over
// the first NT threads (the persistent kernel's consumer warps, excluding its producer warp).
template <int NT>
__device__ __forceinline__ void csync() {
    if (NT == 0) __syncthreads();
    else asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// 2^52 + v as a double (0 <= v < 2^32): (2^52 + q) - (2^52 + z) is exactly q - z.
__device__ __forceinline__ double magic_d(uint32_t v) { return __hiloint2double(0x43300000, (int)v); }

// Chunk-transposed index of element k of token t.
template <int BITS>
__device__ __forceinline__ uint32_t xd_index(uint32_t t, uint32_t k, uint32_t nchunk) {
    constexpr int E = Geom<BITS>::E, F2 = Geom<BITS>::F2;
    return ((t * F2 + (k % E) / 2) * nchunk + k / E) * 2 + (k & 1);
}

// Per-token RMS scale 1/sqrt(mean(x^2) + eps) in double (test/reference/ops.ts:38-45), of MT
// rows of length K, into rs[MT] (shared).  `red` needs MT * warps doubles.  Whole block; ends
// with __syncthreads().
template <int MT, bool CG, int NT = 0>
__device__ __forceinline__ void rms_scale_d(double* rs, double* red, const float* x, uint32_t K, float eps) {
    const uint32_t nthreads = NT ? NT : blockDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = nthreads >> 5;
    for (int t = 0; t < MT; ++t) {
        double s = 0.0;
        for (uint32_t k = threadIdx.x; k < K; k += nthreads) {
            const double v = CG ? __ldcg(x + (size_t)t * K + k) : x[(size_t)t * K + k];
            s = fma(v, v, s);
        }
        s = warp_sum_d(s);
        if (lane == 0) red[t * nw + warp] = s;
    }
    csync<NT>();
    if ((int)threadIdx.x < MT) {
        double tot = 0.0;
        for (int w = 0; w < nw; ++w) tot += red[threadIdx.x * nw + w];
        rs[threadIdx.x] = 1.0 / sqrt(tot / (double)K + (double)eps);
    }
    csync<NT>();
}

// The stored (float) RMSNorm output x * scale * w, exactly as the reference rounds it.
__device__ __forceinline__ float norm_value(float x, double scale, float w) {
    return (float)__dmul_rn(__dmul_rn((double)x, scale), (double)w);
}

// Stage MT activation rows into the chunk-transposed double layout: rs == nullptr stages x as
// is, otherwise the RMSNorm output (float-rounded, then widened).  Ends with __syncthreads().
template <int BITS, int MT, bool CG, int NT = 0>
__device__ __forceinline__ void stage_x_d(double* XD, const float* x, uint32_t K, const double* rs,
                                          const float* gain) {
    const uint32_t nchunk = K / Geom<BITS>::E;
    const uint32_t nthreads = NT ? NT : blockDim.x;
    for (uint32_t i = threadIdx.x; i < MT * K; i += nthreads) {
        const uint32_t t = i / K, k = i % K;
        float v = CG ? __ldcg(x + i) : x[i];
        if (rs) v = norm_value(v, rs[t], gain[k]);
        XD[xd_index<BITS>(t, k, nchunk)] = (double)v;
    }
    csync<NT>();
}

// Shared inner step: one chunk of R rows (codes q[r], scale s[r], zero zc[r]) against MT tokens.
template <int BITS, int MT, int R>
__device__ __forceinline__ void chunk_dot(const uint4 (&q)[R], const float (&s)[R], const uint32_t (&zc)[R],
                                          const double2* __restrict__ XD, uint32_t nchunk, uint32_t c,
                                          double (&acc)[R][MT]) {
    constexpr int F2 = Geom<BITS>::F2;
    constexpr int NP = 4;  // independent partial sums per row: short dependency chains
    double zd[R];
#pragma unroll
    for (int r = 0; r < R; ++r) zd[r] = magic_d(zc[r]);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        double part[R][NP];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int p = 0; p < NP; ++p) part[r][p] = 0.0;
#pragma unroll
        for (int j = 0; j < F2; ++j) {
            const double2 xv = XD[(t * F2 + j) * nchunk + c];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int el = j * 2 + e;
                const int word = BITS == 4 ? el >> 3 : el >> 2;
                const int sh = BITS == 4 ? (el & 7) * 4 : (el & 3) * 8;
                const uint32_t mask = BITS == 4 ? 0xFu : 0xFFu;
                const double xe = e == 0 ? xv.x : xv.y;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint32_t wd = word == 0 ? q[r].x : word == 1 ? q[r].y : word == 2 ? q[r].z : q[r].w;
                    part[r][el % NP] = fma(magic_d((wd >> sh) & mask) - zd[r], xe, part[r][el % NP]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
            acc[r][t] = fma((part[r][0] + part[r][1]) + (part[r][2] + part[r][3]), (double)s[r], acc[r][t]);
    }
}

// acc[r][t] += lane's share of row rows[r] . x[t], weights read from global memory.
template <int BITS, int MT, int R>
__device__ __forceinline__ void dot_rows_d(const QW& w, const uint32_t (&rows)[R], const double2* __restrict__ XD,
                                           uint32_t nchunk, int lane, double (&acc)[R][MT]) {
    constexpr int CPB = Geom<BITS>::CPB;
    const uint4* P = reinterpret_cast<const uint4*>(w.packed);
    const uint32_t bpr = w.cols / kBlock;
    for (uint32_t c = lane; c < nchunk; c += 32) {
        uint4 q[R];
        float s[R];
        uint32_t zc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) q[r] = ld_stream(P + (size_t)rows[r] * nchunk + c);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t blk = rows[r] * bpr + c / CPB;
            s[r] = __ldg(w.scales + blk);
            zc[r] = zero_code<BITS>(w.zeros, blk);
        }
        chunk_dot<BITS, MT, R>(q, s, zc, XD, nchunk, c, acc);
    }
}

}  // namespace enx
