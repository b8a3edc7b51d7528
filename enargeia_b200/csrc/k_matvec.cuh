// Dequantise-in-registers matvec core for the int4 projections and the int8 tied head.
//
// Weight layout is the .enargeia layout, unchanged (verbatim upload): row r of an N x K tensor
// is K/8 (int4) or K/4 (int8) u32 words, reduction axis contiguous, low bits first; one f32
// scale per 64-element block; zero-points packed 8 (int4) or 4 (int8) per u32 word, block index
// r*(K/64) + k/64.
//
// Work split: a "chunk" is 16 bytes of packed codes (32 int4 or 16 int8 elements).  Lane l of a
// warp always handles chunks l, l+32, ... of whatever row the warp is on, so a row is read with
// fully coalesced 16-byte loads.  The activations sit in shared memory transposed by chunk
// (X4[(t*F4 + j)*nchunk + c] = x[t][c*E + 4j .. 4j+3]) so that the lanes' float4 reads are
// conflict-free.  Codes become floats with the 2^23 exponent trick and (q - z) is formed exactly,
// then scaled once per chunk: acc += s * sum_j (q_j - z) * x_j.
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
    static constexpr int F4 = E / 4;                // float4 of x per chunk
    static constexpr int CPB = kBlock / E;          // chunks per quantisation block
};

template <int BITS>
__device__ __forceinline__ uint32_t zero_code(const uint32_t* zeros, uint32_t blk) {
    if (BITS == 4) return (__ldg(zeros + (blk >> 3)) >> ((blk & 7u) * 4u)) & 0xFu;
    return (__ldg(zeros + (blk >> 2)) >> ((blk & 3u) * 8u)) & 0xFFu;
}

// Stage MT activation rows (x[t*K + k], optionally times `scale[t]` and `gain[k]`) into the
// chunk-transposed layout.  Call with the whole block; ends with __syncthreads().
template <int BITS, int MT>
__device__ __forceinline__ void stage_x(float4* X4, const float* x, uint32_t K, const float* rs,
                                        const float* gain) {
    constexpr int E = Geom<BITS>::E, F4 = Geom<BITS>::F4;
    const uint32_t nchunk = K / E;
    const uint32_t n4 = K / 4;
    for (uint32_t i = threadIdx.x; i < MT * n4; i += blockDim.x) {
        uint32_t t = i / n4, e4 = i % n4;
        float4 v = reinterpret_cast<const float4*>(x + (size_t)t * K)[e4];
        if (rs) {
            float s = rs[t];
            float4 g = gain ? reinterpret_cast<const float4*>(gain)[e4] : make_float4(1.f, 1.f, 1.f, 1.f);
            // x * scale * w, in that order (src/kernels/rmsnorm.wgsl:60)
            v.x = v.x * s * g.x; v.y = v.y * s * g.y; v.z = v.z * s * g.z; v.w = v.w * s * g.w;
        }
        uint32_t c = (e4 * 4) / E, j = e4 % F4;
        X4[(t * F4 + j) * nchunk + c] = v;
    }
    __syncthreads();
}

// Per-token RMS scale 1/sqrt(mean(x^2) + eps) of MT rows of length K, into rs[MT] (shared).
// Whole block; ends with __syncthreads().
template <int MT>
__device__ __forceinline__ void rms_scale(float* rs, float* red, const float* x, uint32_t K,
                                          float eps) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int t = 0; t < MT; ++t) {
        float s = 0.f;
        for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) {
            float v = x[(size_t)t * K + k];
            s = fmaf(v, v, s);
        }
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        if (threadIdx.x == 0) {
            float tot = 0.f;
            for (int w = 0; w < nw; ++w) tot += red[w];
            rs[t] = 1.0f / sqrtf(tot / (float)K + eps);
        }
        __syncthreads();
    }
}

// acc[r][t] += lane's share of row rows[r] . x[t].  Caller reduces across the warp.
template <int BITS, int MT, int R>
__device__ __forceinline__ void dot_rows(const QW& w, const uint32_t (&rows)[R],
                                         const float4* __restrict__ X4, uint32_t nchunk, int lane,
                                         float (&acc)[R][MT]) {
    constexpr int F4 = Geom<BITS>::F4, CPB = Geom<BITS>::CPB;
    const uint4* P = reinterpret_cast<const uint4*>(w.packed);
    const uint32_t bpr = w.cols / kBlock;
    for (uint32_t c = lane; c < nchunk; c += 32) {
        uint4 q[R];
#pragma unroll
        for (int r = 0; r < R; ++r) q[r] = ld_stream(P + (size_t)rows[r] * nchunk + c);
        float s[R], zf[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            uint32_t blk = rows[r] * bpr + c / CPB;
            s[r] = __ldg(w.scales + blk);
            zf[r] = magic_u(zero_code<BITS>(w.zeros, blk));
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            float part[R];
#pragma unroll
            for (int r = 0; r < R; ++r) part[r] = 0.f;
#pragma unroll
            for (int j = 0; j < F4; ++j) {
                float4 xv = X4[(t * F4 + j) * nchunk + c];
                float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int el = j * 4 + e;          // element within the chunk
                    const int word = BITS == 4 ? el >> 3 : el >> 2;
                    const int sh = BITS == 4 ? (el & 7) * 4 : (el & 3) * 8;
                    const uint32_t mask = BITS == 4 ? 0xFu : 0xFFu;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        uint32_t wd = word == 0 ? q[r].x : word == 1 ? q[r].y : word == 2 ? q[r].z : q[r].w;
                        float wv = magic_u((wd >> sh) & mask) - zf[r];  // exact q - z
                        part[r] = fmaf(wv, xs[e], part[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][t] = fmaf(part[r], s[r], acc[r][t]);
        }
    }
}

}  // namespace enx
