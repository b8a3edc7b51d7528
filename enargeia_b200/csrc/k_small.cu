// Row-wise and elementwise ops used by the prefill path and by the raw kernel entry points:
// RMSNorm (src/kernels/rmsnorm.wgsl:27-63), RoPE from a cos/sin table (src/kernels/rope.wgsl:
// 28-53), f16 cache pack (src/kernels/cache_variants.ts:269-301), SiLU*up
// (src/kernels/silu_mul.wgsl:19-26) and add (src/kernels/add.wgsl:15-21).

#include "enx_internal.cuh"
#include "k_decode.cuh"
#include "k_small.cuh"

namespace enx {

// RMSNorm in the reference's arithmetic: f64 sum of squares, f64 scale, one rounding per output.
__global__ void k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w,
                          float* __restrict__ out, uint32_t features, float eps) {
    __shared__ double red[32];
    __shared__ double scale;
    const float* xr = x + (size_t)blockIdx.x * features;
    double s = 0.0;
    for (uint32_t f = threadIdx.x; f < features; f += blockDim.x) s = fma((double)xr[f], (double)xr[f], s);
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (uint32_t i = 0; i < blockDim.x / 32; ++i) t += red[i];
        scale = 1.0 / sqrt(t / (double)features + (double)eps);
    }
    __syncthreads();
    float* o = out + (size_t)blockIdx.x * features;
    for (uint32_t f = threadIdx.x; f < features; f += blockDim.x) o[f] = norm_value(xr[f], scale, w[f]);
}

template <typename T>
__global__ void k_rope(const float* __restrict__ x, float* __restrict__ out, const T* __restrict__ ct,
                       const T* __restrict__ st, uint32_t seq, uint32_t heads, uint32_t hd, uint32_t pos0,
                       uint32_t out_offset) {
    const uint32_t half = hd / 2, per_row = heads * half;
    const uint32_t total = seq * per_row;
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < total; g += gridDim.x * blockDim.x) {
        const uint32_t s = g / per_row, rem = g % per_row, h = rem / half, i = rem % half;
        const uint32_t pos = pos0 + s;
        const size_t base = ((size_t)s * heads + h) * hd;
        float a = x[base + i], b = x[base + i + half];
        rope_pair(a, b, (double)ct[(size_t)pos * half + i], (double)st[(size_t)pos * half + i]);
        out[out_offset + base + i] = a;
        out[out_offset + base + i + half] = b;
    }
}

__global__ void k_cache_pack(const float* __restrict__ src, uint16_t* __restrict__ dst,
                             uint32_t count, uint32_t dst_offset) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        dst[(size_t)dst_offset + i] = __half_as_ushort(__float2half_rn(src[i]));
}

__global__ void k_silu_mul(const float* __restrict__ g, const float* __restrict__ u,
                           float* __restrict__ out, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        out[i] = silu_mul_value(g[i], u[i]);
    }
}

__global__ void k_add(const float* __restrict__ a, const float* __restrict__ b,
                      float* __restrict__ out, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

static uint32_t blocks_for(uint32_t n) {
    uint32_t b = (n + 255) / 256;
    return b < 1 ? 1 : (b > 4096 ? 4096 : b);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, uint32_t seq,
                           uint32_t features, float eps, cudaStream_t st) {
    if (seq == 0) return cudaSuccess;
    k_rmsnorm<<<seq, 256, 0, st>>>(x, w, out, features, eps);
    return cudaGetLastError();
}

cudaError_t launch_rope(const float* x, float* out, const float* ct, const float* sn, uint32_t seq,
                        uint32_t heads, uint32_t hd, uint32_t pos0, uint32_t out_offset,
                        cudaStream_t st) {
    uint32_t n = seq * heads * (hd / 2);
    if (n == 0) return cudaSuccess;
    k_rope<float><<<blocks_for(n), 256, 0, st>>>(x, out, ct, sn, seq, heads, hd, pos0, out_offset);
    return cudaGetLastError();
}

cudaError_t launch_rope_d(const float* x, float* out, const double* ct, const double* sn, uint32_t seq,
                          uint32_t heads, uint32_t hd, uint32_t pos0, uint32_t out_offset, cudaStream_t st) {
    uint32_t n = seq * heads * (hd / 2);
    if (n == 0) return cudaSuccess;
    k_rope<double><<<blocks_for(n), 256, 0, st>>>(x, out, ct, sn, seq, heads, hd, pos0, out_offset);
    return cudaGetLastError();
}

cudaError_t launch_cache_pack(const float* src, uint16_t* dst, uint32_t count, uint32_t dst_offset,
                              cudaStream_t st) {
    if (count == 0) return cudaSuccess;
    k_cache_pack<<<blocks_for(count), 256, 0, st>>>(src, dst, count, dst_offset);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* g, const float* u, float* out, uint32_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    k_silu_mul<<<blocks_for(n), 256, 0, st>>>(g, u, out, n);
    return cudaGetLastError();
}

cudaError_t launch_add(const float* a, const float* b, float* out, uint32_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    k_add<<<blocks_for(n), 256, 0, st>>>(a, b, out, n);
    return cudaGetLastError();
}

// Negative log-likelihood of `target` under the softmax of one logits row, in double, as the
// reference's perplexity harness computes it (test/parity/quality.test.ts:93-99): max over the
// float logits, sum of exp(logit - max) in double, -((logit[target] - max) - log(sum)).  One
// block; the partial sums are combined in a fixed order (deterministic).
__global__ void k_nll(const float* __restrict__ logits, uint32_t vocab, uint32_t target, double* __restrict__ out) {
    __shared__ float redf[32];
    __shared__ double redd[32];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, logits[i]);
    m = warp_max(m);
    if (lane == 0) redf[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (uint32_t w = 0; w < nw; ++w) m = fmaxf(m, redf[w]);
    const double md = (double)m;
    double s = 0.0;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) s += exp((double)logits[i] - md);
    s = warp_sum_d(s);
    if (lane == 0) redd[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (uint32_t w = 0; w < nw; ++w) t += redd[w];
        *out = -(((double)logits[target] - md) - log(t));
    }
}

cudaError_t launch_nll(const float* logits, uint32_t vocab, uint32_t target, double* out, cudaStream_t st) {
    k_nll<<<1, 1024, 0, st>>>(logits, vocab, target, out);
    return cudaGetLastError();
}

}  // namespace enx
