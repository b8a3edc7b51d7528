// Quantised projection GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators), for
// M >= 16 tokens: Y[m][n] = float(sum_k x[m][k] * (q[n][k] - z[n][b]) * s[n][b] (+ bias[n])).
//
// The reference sums these products in double (test/reference/quant.ts:95-112).  Tensor cores
// cannot multiply doubles, but they can sum integers exactly, so the activations go in as
// integers: for each token and 64-element quantisation block, x is scaled by a power of two 2^F
// (F from the block's largest exponent) to a 46-bit integer X = rint(x * 2^F) -- exact unless a
// value is 2^-22 below the block's largest -- split into six balanced int8 limbs (two more zero
// limbs pad each token to 8 columns).  One kind::i8 MMA pair per block gives, per (row, token,
// limb), the exact int32 sum over the block of q * limb.  The epilogue joins the limbs into the
// exact int64 sum of q * X, takes off z * sum(X), and adds s * 2^-F times that to a double
// accumulator: one rounding per block where the reference rounds per product.
//
// Layout: a CTA owns 128 weight rows (M = 128 of the MMA) and 32 tokens (N = 8 limbs x 32 = 256).
// Per 64-element block, all 256 threads unpack the rows' codes into a K-major shared-memory tile
// (int4: nibbles to bytes, even elements then odd ones -- the limb tile uses the same order), one
// thread streams the block's limb tile in with a bulk copy, one thread issues the MMAs into one of
// two TMEM accumulators, and both warpgroups read the other accumulator (tokens 0-15 and 16-31)
// while the tensor cores work.  Every wait is bounded; on timeout the kernel records an error and
// returns, having freed its tensor memory.

#include "enx_internal.cuh"
#include "k_decode.cuh"
#include "k_gemm_tc.cuh"

namespace enx {

namespace {

constexpr int kTcThreads = 256;
constexpr uint32_t kTcRows = 128;     // weight rows per CTA (MMA M)
constexpr uint32_t kTcTokens = 32;    // tokens per CTA (MMA N = 8 * 32)
constexpr uint32_t kTcN = 8 * kTcTokens;
constexpr uint32_t kTcTmemCols = 512;  // two accumulators of 256 columns
constexpr uint32_t kTcSpin = 1u << 24;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Byte offset of (row, k-byte) in a K-major, unswizzled canonical tile of 64 k-bytes per row:
// 8-row x 16-byte core matrices, the four k-chunks of a row group adjacent (128 B apart), row
// groups 512 B apart.
__host__ __device__ __forceinline__ uint32_t canon(uint32_t r, uint32_t kb) {
    return (r >> 3) * 512 + (kb >> 4) * 128 + (r & 7) * 16 + (kb & 15);
}

// Shared-memory matrix descriptor: start, leading-byte offset 128, stride-byte offset 512,
// version 1, no swizzle.
__device__ __forceinline__ uint64_t mdesc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor: s32 accumulate, A u8 (codes), B s8 (limbs), both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (2u << 4) | (0u << 7) | (1u << 10) | ((kTcN >> 3) << 17) | ((kTcRows >> 4) << 24);

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < kTcSpin; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok)
                     : "r"(su32(bar)), "r"(parity)
                     : "memory");
        if (ok) return true;
    }
    return false;
}

// Element order inside a 64-element block for int4 codes: slot j < 32 holds element 8(j/4)+2(j%4),
// slot 32 + j holds the next (odd) element -- the order in which nibbles unpack to bytes.
__host__ __device__ __forceinline__ uint32_t slot_element(int bits, uint32_t j) {
    if (bits == 8) return j;
    return j < 32 ? 8 * (j >> 2) + 2 * (j & 3) : 8 * ((j - 32) >> 2) + 2 * ((j - 32) & 3) + 1;
}

}  // namespace

// Per (token group, block): the 256 x 64 limb tile (canonical layout, rows token*8 + limb), then
// per token the exact block sum of X (int64) and 2^-F (double).
__global__ void __launch_bounds__(256) k_limbs(const float* __restrict__ x, uint32_t ld, uint32_t M, uint32_t K,
                                               int bits, uint8_t* __restrict__ out) {
    const uint32_t g = blockIdx.y, b = blockIdx.x, nb = K / kBlock;
    const uint32_t t = threadIdx.x >> 3, part = threadIdx.x & 7;  // token of the group, 8 elements each
    const uint32_t m = g * kTcTokens + t;
    uint8_t* tile = out + ((size_t)g * nb + b) * kTcLimbTileBytes;
    // my 8 slots: part*8 .. part*8+7 of the block's 64 slots
    float v[8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t e = slot_element(bits, part * 8 + i);
        v[i] = m < M ? x[(size_t)m * ld + (size_t)b * kBlock + e] : 0.f;
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // |x| < 2^e for the block's largest |x| (normal or zero); F = 46 - e keeps |X| < 2^46
    const int e = amax == 0.f ? 0 : (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    const int F = 46 - e;
    const double up = __hiloint2double((1023 + F) << 20, 0);
    long long X[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        X[i] = __double2ll_rn((double)v[i] * up);
        sum += X[i];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // balanced base-256 digits: digit l of X is byte l of X + 0x808080808080, minus 128
#pragma unroll
    for (uint32_t l = 0; l < 8; ++l) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t d = l < 6 ? (uint32_t)(((unsigned long long)(X[i] + 0x808080808080LL) >> (8 * l)) & 0xFF) - 128u : 0u;
            if (i < 4) w0 |= (d & 0xFFu) << (8 * i);
            else w1 |= (d & 0xFFu) << (8 * (i - 4));
        }
        uint2* dst = reinterpret_cast<uint2*>(tile + canon(t * 8 + l, part * 8));
        *dst = make_uint2(w0, w1);
    }
    if (part == 0) {
        long long* xs = reinterpret_cast<long long*>(tile + kTcN * 64);
        xs[2 * t] = sum;
        reinterpret_cast<double*>(xs)[2 * t + 1] = __hiloint2double((1023 - F) << 20, 0);
    }
}

template <int BITS>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const uint8_t* __restrict__ limbs, QW w, const float* __restrict__ bias, float* __restrict__ out,
              uint32_t M, uint32_t out_stride, uint32_t out_offset, uint32_t* err) {
    constexpr uint32_t kATile = kTcRows * 64;  // 8 KB of codes per block
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr uint32_t kSt = 3;                           // stages of codes and limb tiles
    uint8_t* sA = smem;                                   // [3][kATile]
    uint8_t* sB = smem + kSt * kATile;                    // [3][kTcLimbTileBytes]
    float* sS = reinterpret_cast<float*>(sB + kSt * kTcLimbTileBytes);  // [3][128] scales
    uint32_t* sZ = reinterpret_cast<uint32_t*>(sS + kSt * kTcRows);     // [3][128] zero codes
    __shared__ __align__(8) uint64_t bar_b[kSt], bar_d[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t K = w.cols, nb = K / kBlock, bpr = K / kBlock;
    const uint32_t r0 = blockIdx.x * kTcRows, g = blockIdx.y;
    const uint8_t* ltile = limbs + (size_t)g * nb * kTcLimbTileBytes;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < kSt; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bar_b[i])));
        for (int i = 0; i < 2; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bar_d[i])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    // epilogue role: warpgroup wg takes tokens wg*16 .. wg*16+15 of rows 32*(warp%4) + lane
    const uint32_t wg = warp >> 2, erow = 32 * (warp & 3) + lane, grow = r0 + erow;
    double acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0;

    auto issue_b = [&](uint32_t b) {  // one thread: the block's limb tile into stage b % 3
        const uint32_t s = b % kSt;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&bar_b[s])), "r"(kTcLimbTileBytes)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         su32(sB + s * kTcLimbTileBytes)),
                     "l"(ltile + (size_t)b * kTcLimbTileBytes), "r"(kTcLimbTileBytes), "r"(su32(&bar_b[s]))
                     : "memory");
    };
    if (tid == 0) issue_b(0);

    // Block b: codes and limbs in stage b % 3, accumulator b & 1.  Stage (b + 1) % 3 last held
    // block b - 2, whose MMA finished (waited in iteration b - 1) and whose epilogue ran in
    // iteration b - 1, so the limb copy for b + 1 may start right after the MMA of b.
    for (uint32_t b = 0; b <= nb; ++b) {
        const uint32_t s = b % kSt;
        if (b < nb) {
            // codes of block b into stage s: two threads per row, 32 elements each
            const uint32_t row = tid >> 1, half = tid & 1, gr = r0 + row;
            if (BITS == 4) {
                uint4 q = make_uint4(0, 0, 0, 0);
                if (gr < w.rows) q = __ldg(reinterpret_cast<const uint4*>(w.packed + (size_t)gr * (K / 8) + b * 8 + half * 4));
                const uint32_t ww[4] = {q.x, q.y, q.z, q.w};
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    lo[i] = ww[i] & 0x0F0F0F0Fu;
                    hi[i] = (ww[i] >> 4) & 0x0F0F0F0Fu;
                }
                // slots: lo of words 0..7 fill k-bytes 0..31, hi fill 32..63
                *reinterpret_cast<uint4*>(sA + s * kATile + canon(row, half * 16)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4*>(sA + s * kATile + canon(row, 32 + half * 16)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            } else {
                uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
                if (gr < w.rows) {
                    const uint4* p = reinterpret_cast<const uint4*>(w.packed + (size_t)gr * (K / 4) + b * 16 + half * 8);
                    q0 = __ldg(p);
                    q1 = __ldg(p + 1);
                }
                *reinterpret_cast<uint4*>(sA + s * kATile + canon(row, half * 32)) = q0;
                *reinterpret_cast<uint4*>(sA + s * kATile + canon(row, half * 32 + 16)) = q1;
            }
            if (half == 0) {
                const uint32_t blk = gr * bpr + b;
                sS[s * kTcRows + row] = gr < w.rows ? __ldg(w.scales + blk) : 0.f;
                sZ[s * kTcRows + row] = gr < w.rows ? zero_code<BITS>(w.zeros, blk) : 0u;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // codes written; the previous epilogue is done with its accumulator
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (tid == 0 && b < nb) {
            if (!mbar_wait(&bar_b[s], (b / kSt) & 1)) {
                atomicMax(err, 3u);
                s_fail = 1;
            } else {
                const uint32_t dcol = tmem + (b & 1) * kTcN;
#pragma unroll
                for (uint32_t kk = 0; kk < 2; ++kk) {
                    const uint64_t ad = mdesc(su32(sA + s * kATile) + kk * 256);
                    const uint64_t bd = mdesc(su32(sB + s * kTcLimbTileBytes) + kk * 256);
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                                     dcol),
                                 "l"(ad), "l"(bd), "r"(kIdesc), "r"(kk));
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&bar_d[b & 1]))
                             : "memory");
                if (b + 1 < nb) issue_b(b + 1);
            }
        }
        if (b == 0) continue;
        // epilogue of block b-1 from accumulator (b-1) & 1 (its scales and sums in stage (b-1) % 3)
        const uint32_t pb = b - 1, ps = pb & 1, pst = pb % kSt;
        if (tid == 0 && !s_fail && !mbar_wait(&bar_d[ps], (pb >> 1) & 1)) {
            atomicMax(err, 3u);
            s_fail = 1;
        }
        __syncthreads();
        if (s_fail) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        {
            const double sc = (double)sS[pst * kTcRows + erow];
            const long long zc = (long long)sZ[pst * kTcRows + erow];
            const long long* xs = reinterpret_cast<const long long*>(sB + pst * kTcLimbTileBytes + kTcN * 64);
#pragma unroll
            for (int tt = 0; tt < 16; ++tt) {
                const uint32_t t = wg * 16 + tt;
                uint32_t d[8];
                const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + ps * kTcN + t * 8;
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7])
                             : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                long long T = 0;
#pragma unroll
                for (int l = 5; l >= 0; --l) T = T * 256 + (long long)(int)d[l];
                T -= zc * xs[2 * t];
                const double down = reinterpret_cast<const double*>(xs)[2 * t + 1];
                acc[tt] = fma((double)T, sc * down, acc[tt]);
            }
        }
    }
    if (!s_fail && grow < w.rows) {
        const double bv = bias ? (double)__ldg(bias + grow) : 0.0;
#pragma unroll
        for (int tt = 0; tt < 16; ++tt) {
            const uint32_t m = g * kTcTokens + wg * 16 + tt;
            if (m < M) out[(size_t)m * out_stride + out_offset + grow] = (float)(acc[tt] + bv);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
}

size_t gemm_tc_workspace_bytes(uint32_t m, uint32_t k) {
    const size_t groups = (m + kTcTokens - 1) / kTcTokens;
    return groups * (k / kBlock) * (size_t)kTcLimbTileBytes;
}

cudaError_t launch_gemm_tc(int bits, const float* x, uint32_t ld, const QW& w, const float* bias, float* out,
                           uint32_t m, uint32_t out_stride, uint32_t out_offset, uint8_t* workspace, uint32_t* err,
                           cudaStream_t st) {
    const uint32_t groups = (m + kTcTokens - 1) / kTcTokens, nb = w.cols / kBlock;
    k_limbs<<<dim3(nb, groups), 256, 0, st>>>(x, ld, m, w.cols, bits, workspace);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = 3 * ((size_t)kTcRows * 64 + (size_t)kTcLimbTileBytes + kTcRows * 4 + kTcRows * 4);
    const dim3 grid((w.rows + kTcRows - 1) / kTcRows, groups);
    if (bits == 4) {
        e = cudaFuncSetAttribute(k_gemm_tc<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_gemm_tc<4><<<grid, kTcThreads, smem, st>>>(workspace, w, bias, out, m, out_stride, out_offset, err);
    } else {
        e = cudaFuncSetAttribute(k_gemm_tc<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_gemm_tc<8><<<grid, kTcThreads, smem, st>>>(workspace, w, bias, out, m, out_stride, out_offset, err);
    }
    return e == cudaSuccess ? cudaGetLastError() : e;
}

}  // namespace enx
