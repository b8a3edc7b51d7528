// Quantised projection GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators), for
// M >= 16 tokens: Y[m][n] = float(sum_k x[m][k] * (q[n][k] - z[n][b]) * s[n][b] (+ bias[n])).
//
// The reference sums these products in double (test/reference/quant.ts:95-112).  Tensor cores
// cannot multiply doubles, but they can sum integers exactly, so the activations go in as
// integers: each token's row of x is scaled by a power of two 2^F (F from the row's largest
// exponent) to 46-bit integers X = rint(x * 2^F) -- exact unless a value is 2^-22 below the row's
// largest -- split into six balanced int8 limbs (k_limbs).  The weights go in as a byte matrix:
// int8 codes q as stored, int4 codes as q - z (a signed byte; k_codes_i8).  One kind::i8 MMA
// pair per 64-element block gives, per (row, token, limb), the exact int32 sum over the block of
// a * limb.  The epilogue joins the limbs into the exact int64 sum of a * X, takes off z * sum(X)
// for int8, and adds s times that to a double accumulator (one rounding per block where the
// reference rounds per product); 2^-F is applied once at the end, exactly.
//
// Layout: a CTA owns 128 weight rows (M = 128 of the MMA), 32 tokens (N = 6 limbs x 32 = 192,
// limb-major) and a range of 64-element blocks (split-K when the row tiles x token groups do not
// fill the GPU; the splits' double partials are then summed in split order by a second kernel).
// Token groups of a row tile are adjacent in the grid, so they read the tile's codes from L2.
//
// Warp roles, synchronised by mbarriers only:
//   warps 0-15  epilogue: warpgroup wg drains tokens 8wg..8wg+7 of the accumulator the tensor
//               cores are not writing (thread = row, one 8-column TMEM load per limb), then
//               releases it;
//   warp 16     TMEM allocation; lane 0 issues the two MMAs of each block;
//   warp 17     producer: lane 0 loads each block's codes (one 64-byte-swizzled TMA box of 128
//               rows) and its limb tile (one bulk copy) into a stage.
// Eight stages of (codes, limbs), two accumulators 256 TMEM columns apart.  Every wait is
// bounded; on timeout the kernel records an error, every role stops, and the tensor memory is
// freed.

#include <cuda.h>

#include "enx_internal.cuh"
#include "k_decode.cuh"
#include "k_gemm_tc.cuh"

namespace enx {

namespace {

constexpr uint32_t kTcRows = 128;     // weight rows per CTA (MMA M)
constexpr uint32_t kTcTokens = 32;    // tokens per CTA
constexpr uint32_t kTcLimbs = 6;       // balanced int8 limbs of a 46-bit X
constexpr uint32_t kTcN = kTcLimbs * kTcTokens;  // MMA N = 192, limb-major: column 32 l + t
constexpr uint32_t kTcAccCols = 256;   // columns between the two accumulators
constexpr uint32_t kTcTmemCols = 512;  // TMEM allocation: the two accumulators
constexpr uint32_t kTcSpin = 1u << 24;  // default wait limit, and the limit of the drain waits

// Spins a wait may take before it gives up (enx_set_wait_limit; per device).  Drain waits (copies
// and MMAs still in flight when the CTA stops) always use kTcSpin.
__device__ uint32_t g_tc_spin = kTcSpin;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Byte offset of (row, k-byte) in a K-major, unswizzled canonical tile of 64 k-bytes per row (the
// limb tiles): 8-row x 16-byte core matrices, the four k-chunks of a row group adjacent (128 B
// apart), row groups 512 B apart.
__host__ __device__ __forceinline__ uint32_t canon(uint32_t r, uint32_t kb) {
    return (r >> 3) * 512 + (kb >> 4) * 128 + (r & 7) * 16 + (kb & 15);
}

// Shared-memory matrix descriptor of a limb tile: start, leading-byte offset 128, stride-byte
// offset 512, version 1, no swizzle.
__device__ __forceinline__ uint64_t mdesc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor: s32 accumulate, B s8 (limbs), both K-major, N = 192, M = 128; A is u8
// (int8 codes q) or s8 (int4: q - z, which fits a signed byte).
template <int BITS>
__host__ __device__ constexpr uint32_t idesc() {
    return (2u << 4) | ((BITS == 4 ? 1u : 0u) << 7) | (1u << 10) | ((kTcN >> 3) << 17) | ((kTcRows >> 4) << 24);
}

// Element order inside a 64-element block for int4 codes: slot j < 32 holds element 8(j/4)+2(j%4),
// slot 32 + j holds the next (odd) element -- the order in which nibbles unpack to bytes.
__host__ __device__ __forceinline__ uint32_t slot_element(int bits, uint32_t j) {
    if (bits == 8) return j;
    return j < 32 ? 8 * (j >> 2) + 2 * (j & 3) : 8 * ((j - 32) >> 2) + 2 * ((j - 32) & 3) + 1;
}

}  // namespace

// Limb tiles: per (token group, block) the 256 x 64 limb tile (canonical layout, rows token*8 +
// limb), then per token the exact block sum of X (int64) and 2^-F (double).  F is per token, from
// the largest |x| of the token's whole row, so the tensor-core epilogue applies 2^-F once at the
// end.  A warp per token and chunk of kLimbChunk blocks: the row maximum, then per block two slots
// per lane, limbs staged through shared memory so each lane stores one 16-byte chunk.
constexpr uint32_t kLimbChunk = 2;

__global__ void __launch_bounds__(256) k_limbs(const float* __restrict__ x, uint32_t ld, uint32_t M, uint32_t K,
                                               int bits, uint8_t* __restrict__ out) {
    pdl_launch_dependents();  // the GEMM may start its prologue; it waits for this grid's results
    __shared__ __align__(16) uint8_t stage[8][8 * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m = blockIdx.x * 8 + warp, g = m / kTcTokens, t = m % kTcTokens;
    const uint32_t nb = K / kBlock, b0 = blockIdx.y * kLimbChunk, b1 = min(b0 + kLimbChunk, nb);
    const bool live = m < M;  // tokens past M fill their tile rows with zero limbs
    const float* row = x + (size_t)(live ? m : 0) * ld;
    float amax = 0.f;
    if (live)
        for (uint32_t k = lane * 4; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // |x| < 2^e for the row's largest |x| (normal or zero); F = 46 - e keeps |X| < 2^46
    const int e = amax == 0.f ? 0 : (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    const int F = 46 - e;
    const double up = __hiloint2double((1023 + F) << 20, 0);
    const uint32_t s0 = slot_element(bits, 2 * lane), s1 = slot_element(bits, 2 * lane + 1);
    float v[kLimbChunk][2];
#pragma unroll
    for (uint32_t j = 0; j < kLimbChunk; ++j) {
        const uint32_t b = b0 + j;
        v[j][0] = live && b < b1 ? row[(size_t)b * kBlock + s0] : 0.f;
        v[j][1] = live && b < b1 ? row[(size_t)b * kBlock + s1] : 0.f;
    }
    uint8_t* st = stage[warp];
#pragma unroll
    for (uint32_t j = 0; j < kLimbChunk; ++j) {
        const uint32_t b = b0 + j;
        if (b >= b1) break;
        uint8_t* tile = out + ((size_t)g * nb + b) * kTcLimbTileBytes;
        const long long X0 = __double2ll_rn((double)v[j][0] * up), X1 = __double2ll_rn((double)v[j][1] * up);
        long long sum = X0 + X1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        // balanced base-256 digits: digit l of X is byte l of X + 0x808080808080, minus 128
        const unsigned long long u0 = (unsigned long long)(X0 + 0x808080808080LL);
        const unsigned long long u1 = (unsigned long long)(X1 + 0x808080808080LL);
#pragma unroll
        for (uint32_t l = 0; l < kTcLimbs; ++l) {
            const uint32_t d0 = (uint32_t)((u0 >> (8 * l)) & 0xFF) - 128u;
            const uint32_t d1 = (uint32_t)((u1 >> (8 * l)) & 0xFF) - 128u;
            *reinterpret_cast<uint16_t*>(st + l * 64 + 2 * lane) = (uint16_t)((d0 & 0xFFu) | ((d1 & 0xFFu) << 8));
        }
        __syncwarp();
        if (lane < 4 * kTcLimbs) {
            const uint32_t l = lane >> 2, c = lane & 3;  // lane stores chunk c of limb l's row
            *reinterpret_cast<uint4*>(tile + canon(l * kTcTokens + t, c * 16)) =
                *reinterpret_cast<const uint4*>(st + l * 64 + c * 16);
        }
        if (lane == 0) {
            long long* rec = reinterpret_cast<long long*>(tile + kTcN * 64);
            rec[2 * t] = sum;
            reinterpret_cast<double*>(rec)[2 * t + 1] = __hiloint2double((1023 - F) << 20, 0);
        }
        __syncwarp();
    }
}

constexpr uint32_t kTcStages = 8;  // loads take ~2 us to land: 8 blocks in flight
constexpr int kTcEpiGroups = 4;                          // epilogue warpgroups
constexpr int kTcEpiTok = kTcTokens / kTcEpiGroups;      // tokens per epilogue thread (8)
constexpr int kTcEpiWarps = 4 * kTcEpiGroups, kTcMmaWarp = kTcEpiWarps, kTcProdWarp = kTcEpiWarps + 1;
constexpr int kTcWsThreads = (kTcEpiWarps + 2) * 32;     // 576
constexpr uint32_t kTcATile = kTcRows * 64;               // 8 KB of codes per block
constexpr uint32_t kTcMaxSplit = 16;

// Bounded wait on an mbarrier phase that gives up early when another role has failed.
__device__ __forceinline__ bool mbar_wait_f(uint64_t* bar, uint32_t parity, volatile int* fail, uint32_t* err,
                                            uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok)
                     : "r"(su32(bar)), "r"(parity)
                     : "memory");
        if (ok) return true;
        if ((it & 31) == 31 && *fail) return false;
    }
    atomicMax(err, 3u);
    *fail = 1;
    return false;
}

// Waits (bounded by kTcSpin, ignoring other roles' failure) until a phase has completed: the drain
// of copies or MMAs this thread issued, before the CTA may release its shared memory and TMEM.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < kTcSpin; ++it) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok)
                     : "r"(su32(bar)), "r"(parity)
                     : "memory");
        if (ok) return;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}

// Code tiles arrive by TMA from a byte matrix [rows][K] (int8 codes as stored; int4 as the signed
// bytes q - z prepared by k_codes_i8): one 2D box of 64 bytes x 128 rows per block, written with
// the 64-byte swizzle, which is the K-major SWIZZLE_64B layout the MMA reads directly (rows of
// 64 bytes, 8-row groups 512 bytes apart; the second K = 32 half starts 32 bytes in).
__device__ __forceinline__ uint64_t mdesc_a(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46) | (4ull << 61);
}

__device__ __forceinline__ void tma_codes(uint8_t* dst, const CUtensorMap* map, uint32_t block, uint32_t row,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            su32(dst)),
        "l"(map), "r"(block * 64), "r"(row), "r"(su32(bar))  // x = 64 * block bytes: 16-byte aligned
        : "memory");
}

// int4 codes to the byte matrix the GEMM reads: per row and 64-element block, the signed bytes
// q - z in MMA slot order (the low nibbles of the block's 32 packed bytes, then the high ones).
// A thread per (row, block).
__global__ void k_codes_i8(QW w, uint8_t* __restrict__ out) {
    const uint32_t nb = w.cols / kBlock;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)w.rows * nb) return;
    const uint32_t row = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
    const uint4* q = reinterpret_cast<const uint4*>(w.packed + (size_t)row * (w.cols / 8) + b * 8);
    const uint32_t zz = zero_code<4>(w.zeros, row * nb + b) * 0x01010101u;
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)row * w.cols + (size_t)b * kBlock);
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // words 4h..4h+3: low nibbles to bytes 16h.., high to 32+16h..
        const uint4 v = __ldg(q + h);
        const uint32_t ww[4] = {v.x, v.y, v.z, v.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // per byte ((q | 0x80) - z) ^ 0x80: no borrow, 0x80 + q - z >= 0x71
            lo[k] = (((ww[k] & 0x0F0F0F0Fu) | 0x80808080u) - zz) ^ 0x80808080u;
            hi[k] = ((((ww[k] >> 4) & 0x0F0F0F0Fu) | 0x80808080u) - zz) ^ 0x80808080u;
        }
        dst[h] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        dst[2 + h] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

template <int BITS>
__global__ void __launch_bounds__(kTcWsThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap cmap, const uint8_t* __restrict__ limbs, QW w,
              const float* __restrict__ bias, float* out, double* __restrict__ partial, uint32_t M,
              uint32_t out_stride, uint32_t out_offset, uint32_t blocks_per_split, uint32_t* err, const float* residual,
              TcSeg seg) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sA = smem;                                // [stages][kTcATile]
    uint8_t* sB = smem + kTcStages * kTcATile;         // [stages][kTcLimbTileBytes]
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], accf[2], acce[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t K = w.cols, nb = K / kBlock, bpr = K / kBlock;
    const uint32_t g = blockIdx.x, r0 = blockIdx.y * kTcRows;
    const uint32_t kb0 = blockIdx.z * blocks_per_split, kb1 = min(kb0 + blocks_per_split, nb);
    const uint32_t nblk = kb1 > kb0 ? kb1 - kb0 : 0;
    const uint8_t* ltile = limbs + (size_t)g * nb * kTcLimbTileBytes;

    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < kTcStages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[i])));
        }
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&accf[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&acce[i])), "r"(kTcEpiWarps));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const uint32_t spin = g_tc_spin;

    if (warp == kTcProdWarp) {
        // ---- producer: one thread, a TMA box of codes and a bulk copy of limbs per block ------------
        if (lane == 0) {
            uint32_t issued = 0;
            for (uint32_t i = 0; i < nblk; ++i) {
                const uint32_t s = i % kTcStages;
                if (i >= kTcStages && !mbar_wait_f(&empty[s], ((i / kTcStages) - 1) & 1, &s_fail, err, spin)) break;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[s])),
                             "r"(kTcATile + kTcLimbTileBytes)
                             : "memory");
                tma_codes(sA + s * kTcATile, &cmap, kb0 + i, r0, &full[s]);  // weights: no wait needed
                if (i == 0) pdl_wait();  // the limb tiles (previous grid) are complete from here on
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                 su32(sB + s * kTcLimbTileBytes)),
                             "l"(ltile + (size_t)(kb0 + i) * kTcLimbTileBytes), "r"(kTcLimbTileBytes), "r"(su32(&full[s]))
                             : "memory");
                issued = i + 1;
            }
            // no copy may still be landing when the CTA releases its shared memory (error path)
            for (uint32_t i = issued > kTcStages ? issued - kTcStages : 0; i < issued; ++i)
                mbar_drain(&full[i % kTcStages], (i / kTcStages) & 1);
        }
        __syncwarp();
    } else if (warp == kTcMmaWarp) {
        // ---- MMA issue: one thread ----------------------------------------------------------------
        pdl_wait();
        if (lane == 0) {
            uint32_t mmas = 0;
            for (uint32_t i = 0; i < nblk; ++i) {
                const uint32_t s = i % kTcStages, a = i & 1;
                if (!mbar_wait_f(&full[s], (i / kTcStages) & 1, &s_fail, err, spin)) break;
                if (i >= 2 && !mbar_wait_f(&acce[a], ((i >> 1) - 1) & 1, &s_fail, err, spin)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dcol = tmem + a * kTcAccCols;
#pragma unroll
                for (uint32_t kk = 0; kk < 2; ++kk) {  // K = 32 per MMA: the two halves of A's 64-byte rows
                    const uint64_t ad = mdesc_a(su32(sA + s * kTcATile) + kk * 32);
                    const uint64_t bd = mdesc(su32(sB + s * kTcLimbTileBytes) + kk * 256);
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                                     dcol),
                                 "l"(ad), "l"(bd), "r"(idesc<BITS>()), "r"(kk));
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&empty[s]))
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&accf[a]))
                             : "memory");
                mmas = i + 1;
            }
            // every issued MMA complete before TMEM is freed (its last commit tracks all of them)
            if (mmas) mbar_drain(&accf[(mmas - 1) & 1], ((mmas - 1) >> 1) & 1);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warpgroup wg, tokens 8wg..8wg+7, thread = row 32*(warp%4) + lane -------------
        pdl_wait();  // limb records and the output may be touched from here on
        const uint32_t wg = warp >> 2, erow = 32 * (warp & 3) + lane, grow = r0 + erow;
        const bool rok = grow < w.rows;
        double acc[kTcEpiTok];
#pragma unroll
        for (int i = 0; i < kTcEpiTok; ++i) acc[i] = 0.0;
        float sc_next = (nblk && rok) ? __ldg(w.scales + (size_t)grow * bpr + kb0) : 0.f;
        uint32_t z_next = (BITS == 8 && nblk && rok) ? zero_code<BITS>(w.zeros, grow * bpr + kb0) : 0u;
        for (uint32_t i = 0; i < nblk; ++i) {
            const uint32_t a = i & 1, b = kb0 + i;
            const double sc = (double)sc_next;
            const long long zc = (long long)z_next;
            if (i + 1 < nblk && rok) {  // the next block's scale (and int8 zero code) while this one drains
                sc_next = __ldg(w.scales + (size_t)grow * bpr + b + 1);
                if (BITS == 8) z_next = zero_code<BITS>(w.zeros, grow * bpr + b + 1);
            }
            int ok = 1;
            if (lane == 0) ok = mbar_wait_f(&accf[a], (i >> 1) & 1, &s_fail, err, spin);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // per token of this block (int8 only): the X sum, from the limb tile in global memory
            const int* tok = reinterpret_cast<const int*>(ltile + (size_t)b * kTcLimbTileBytes + kTcN * 64) +
                             (wg * kTcEpiTok) * 4;
            // limb l of the warpgroup's 8 tokens: 8 accumulator columns 32 l + 8 wg .. + 7, one load each
            uint32_t d[kTcLimbs][8];
#pragma unroll
            for (uint32_t l = 0; l < kTcLimbs; ++l) {
                const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + a * kTcAccCols + l * kTcTokens + wg * kTcEpiTok;
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(d[l][0]), "=r"(d[l][1]), "=r"(d[l][2]), "=r"(d[l][3]), "=r"(d[l][4]), "=r"(d[l][5]),
                               "=r"(d[l][6]), "=r"(d[l][7])
                             : "r"(ta));
            }
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[a]);  // in registers: accumulator a may take block i + 2
#pragma unroll
            for (int tt = 0; tt < kTcEpiTok; ++tt) {
                // exact: each pair d_l + 256 d_(l+1) fits 32 bits
                const long long a0 = (long long)((int)d[0][tt] + (int)d[1][tt] * 256);
                const long long a1 = (long long)((int)d[2][tt] + (int)d[3][tt] * 256);
                const long long a2 = (long long)((int)d[4][tt] + (int)d[5][tt] * 256);
                long long T = a0 + a1 * 65536LL + a2 * 4294967296LL;
                if (BITS == 8) {
                    const int2 xs = __ldg(reinterpret_cast<const int2*>(tok + 4 * tt));
                    T -= zc * (((long long)xs.y << 32) | (unsigned)xs.x);
                }
                acc[tt] = fma((double)T, sc, acc[tt]);
            }
        }
        if (!s_fail && rok && nblk) {
            // each token's 2^-F (the same in every block's record), applied once: exact
            const double* rec = reinterpret_cast<const double*>(ltile + (size_t)kb0 * kTcLimbTileBytes + kTcN * 64);
#pragma unroll
            for (int tt = 0; tt < kTcEpiTok; ++tt) acc[tt] *= __ldg(rec + 2 * (wg * kTcEpiTok + tt) + 1);
            if (partial) {  // split-K: this split's double partial, [split][M][rows]
                double* pp = partial + (size_t)blockIdx.z * M * w.rows;
#pragma unroll
                for (int tt = 0; tt < kTcEpiTok; ++tt) {
                    const uint32_t m = g * kTcTokens + wg * kTcEpiTok + tt;
                    if (m < M) pp[(size_t)m * w.rows + grow] = acc[tt];
                }
            } else {
                // this row's output: the single one, or its segment of a stacked weight
                float* o_ptr = out;
                const float* b_ptr = bias;
                uint32_t o_stride = out_stride, o_col = out_offset + grow, b_row = grow;
                if (BITS == 4 && seg.n) {  // stacked weights are int4 projections
                    const bool s0 = grow < seg.end[0], s1 = !s0 && grow < seg.end[1];  // static picks: no local copy
                    const uint32_t sb = s0 ? 0 : (s1 ? seg.end[0] : seg.end[1]);
                    o_ptr = s0 ? seg.out[0] : (s1 ? seg.out[1] : seg.out[2]);
                    b_ptr = s0 ? seg.bias[0] : (s1 ? seg.bias[1] : seg.bias[2]);
                    o_stride = s0 ? seg.stride[0] : (s1 ? seg.stride[1] : seg.stride[2]);
                    o_col = b_row = grow - sb;
                }
                const double bv = b_ptr ? (double)__ldg(b_ptr + b_row) : 0.0;
#pragma unroll
                for (int tt = 0; tt < kTcEpiTok; ++tt) {
                    const uint32_t m = g * kTcTokens + wg * kTcEpiTok + tt;
                    if (m < M) {
                        // with a residual: the projection rounded to float, then the float add of the
                        // reference's separate add kernel (test/reference/ops.ts:219-225)
                        const size_t o = (size_t)m * o_stride + o_col;
                        const float v = (float)(acc[tt] + bv);
                        o_ptr[o] = residual ? residual[o] + v : v;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == kTcMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
}

cudaError_t tc_set_spin(uint32_t spins) {
    const uint32_t v = spins ? spins : kTcSpin;
    return cudaMemcpyToSymbol(g_tc_spin, &v, sizeof(v));
}

// Split-K: out = float(sum of the splits' partials in split order + bias).
__global__ void k_gemm_tc_combine(const double* __restrict__ partial, uint32_t splits, uint32_t M, uint32_t N,
                                  const float* __restrict__ bias, float* out, uint32_t out_stride,
                                  uint32_t out_offset, const float* residual, TcSeg seg) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * N) return;
    const uint32_t m = (uint32_t)(i / N), n = (uint32_t)(i % N);
    double acc = 0.0;
    for (uint32_t s = 0; s < splits; ++s) acc += partial[(size_t)s * M * N + i];
    float* o_ptr = out;
    const float* b_ptr = bias;
    uint32_t o_stride = out_stride, o_col = out_offset + n, b_row = n;
    if (seg.n) {  // the row's segment of a stacked weight
        const bool s0 = n < seg.end[0], s1 = !s0 && n < seg.end[1];
        const uint32_t sb = s0 ? 0 : (s1 ? seg.end[0] : seg.end[1]);
        o_ptr = s0 ? seg.out[0] : (s1 ? seg.out[1] : seg.out[2]);
        b_ptr = s0 ? seg.bias[0] : (s1 ? seg.bias[1] : seg.bias[2]);
        o_stride = s0 ? seg.stride[0] : (s1 ? seg.stride[1] : seg.stride[2]);
        o_col = b_row = n - sb;
    }
    if (b_ptr) acc += (double)__ldg(b_ptr + b_row);
    const size_t o = (size_t)m * o_stride + o_col;
    o_ptr[o] = residual ? residual[o] + (float)acc : (float)acc;
}

// Splits of the reduction axis: the count that minimises the modelled time waves(s) * (blocks
// per split + kTcFixed), waves(s) = ceil(groups * row tiles * s / SMs), at least 2 blocks each.
constexpr uint32_t kTcFixed = 3;  // per-CTA prologue and flush, in block times
static uint32_t tc_splits(uint32_t m, uint32_t n, uint32_t k) {
    const uint32_t groups = (m + kTcTokens - 1) / kTcTokens, tiles = (n + kTcRows - 1) / kTcRows;
    const uint32_t ctas = groups * tiles, nb = k / kBlock;
    const uint32_t sms = (uint32_t)num_sms();
    uint32_t best = 1;
    uint64_t best_cost = ~0ull;
    for (uint32_t s = 1; s <= min(kTcMaxSplit, max(1u, nb / 2)); ++s) {
        const uint32_t per = (nb + s - 1) / s, used = (nb + per - 1) / per;  // no empty splits
        const uint64_t waves = ((uint64_t)ctas * used + sms - 1) / sms;
        const uint64_t cost = waves * (per + kTcFixed);
        if (cost < best_cost) {
            best_cost = cost;
            best = used;
        }
    }
    return best;
}

static size_t limb_bytes(uint32_t m, uint32_t k) {
    const size_t groups = (m + kTcTokens - 1) / kTcTokens;
    return (groups * (k / kBlock) * (size_t)kTcLimbTileBytes + 255) / 256 * 256;
}

// Rows x splits the partial region of a workspace holds; launches that would need more run with
// fewer splits.
static size_t partial_rows(uint32_t m) {
    const size_t groups = (m + kTcTokens - 1) / kTcTokens;
    return 4 * 148 * (size_t)kTcRows / groups + kTcRows;
}

static size_t partial_bytes(uint32_t m) { return ((size_t)m * partial_rows(m) * sizeof(double) + 255) / 256 * 256; }

size_t gemm_tc_workspace_bytes(uint32_t m, uint32_t k) { return limb_bytes(m, k) + partial_bytes(m); }

size_t gemm_tc_codes_bytes(uint32_t rows, uint32_t k) { return ((size_t)rows * k + 255) / 256 * 256; }

cudaError_t launch_codes_i8(const QW& w, uint8_t* out, cudaStream_t st) {
    const size_t n = (size_t)w.rows * (w.cols / kBlock);
    k_codes_i8<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, out);
    return cudaGetLastError();
}

// cuTensorMapEncodeTiled, looked up through the runtime so the library needs no link-time driver
// dependency (it loads on hosts without a GPU driver, where only its exports are inspected).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

cudaError_t launch_gemm_tc(int bits, const float* x, uint32_t ld, const QW& w, const uint8_t* codes8, const float* bias,
                           float* out, uint32_t m, uint32_t out_stride, uint32_t out_offset, uint8_t* workspace,
                           uint32_t* err, cudaStream_t st, bool limbs_ready, const float* residual, const TcSeg* segp) {
    const uint32_t groups = (m + kTcTokens - 1) / kTcTokens, nb = w.cols / kBlock;
    TcSeg seg{};
    if (segp) {
        // segments: int4 stacks only (the int8 kernel writes the single output), no residual
        if (bits != 4 || residual || segp->n == 0 || segp->n > 3 || segp->end[segp->n - 1] != w.rows)
            return cudaErrorInvalidValue;
        seg = *segp;
        for (uint32_t s2 = seg.n; s2 < 3; ++s2) seg.end[s2] = w.rows;
    }
    cudaError_t e;
    if (bits == 8) {
        codes8 = reinterpret_cast<const uint8_t*>(w.packed);  // int8 codes are the byte matrix already
    } else if (!codes8) {  // no prepared copy: convert into the workspace's code region
        uint8_t* conv = workspace + limb_bytes(m, w.cols) + partial_bytes(m);
        e = launch_codes_i8(w, conv, st);
        if (e != cudaSuccess) return e;
        codes8 = conv;
    }
    if (!limbs_ready) {  // else: the workspace holds the limbs of this x from the previous call
        k_limbs<<<dim3(groups * (kTcTokens / 8), (nb + kLimbChunk - 1) / kLimbChunk), 256, 0, st>>>(x, ld, m, w.cols,
                                                                                              bits, workspace);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // the code bytes as a 2D tensor (K bytes x rows); a box is one 64-element block of 128 rows
    CUtensorMap cmap;
    {
        const cuuint64_t dims[2] = {w.cols, w.rows};
        const cuuint64_t strides[1] = {w.cols};
        const cuuint32_t box[2] = {64, kTcRows};
        const cuuint32_t estr[2] = {1, 1};
        const EncodeTiledFn encode = encode_tiled();
        if (!encode) return cudaErrorNotSupported;
        const CUresult r = encode(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)codes8, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    uint32_t splits = tc_splits(m, w.rows, w.cols);
    while (splits > 1 && (size_t)splits * w.rows > partial_rows(m)) --splits;  // workspace bound
    const uint32_t per = (nb + splits - 1) / splits;
    double* partial = splits > 1 ? reinterpret_cast<double*>(workspace + limb_bytes(m, w.cols)) : nullptr;
    const size_t smem = (size_t)kTcStages * (kTcATile + kTcLimbTileBytes);
    const dim3 grid(groups, (w.rows + kTcRows - 1) / kTcRows, splits);
    // programmatic dependent launch: the prologue and the code loads overlap k_limbs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kTcWsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (bits == 4) {
        e = cudaFuncSetAttribute(k_gemm_tc<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaLaunchKernelEx(&cfg, k_gemm_tc<4>, cmap, (const uint8_t*)workspace, w, bias, out, partial, m,
                                   out_stride, out_offset, per, err, residual, seg);
    } else {
        e = cudaFuncSetAttribute(k_gemm_tc<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaLaunchKernelEx(&cfg, k_gemm_tc<8>, cmap, (const uint8_t*)workspace, w, bias, out, partial, m,
                                   out_stride, out_offset, per, err, residual, seg);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess || splits == 1) return e;
    const size_t total = (size_t)m * w.rows;
    k_gemm_tc_combine<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(partial, splits, m, w.rows, bias, out, out_stride,
                                                                       out_offset, residual, seg);
    return cudaGetLastError();
}

// A tile of 128 rows x 128 code bytes (two 64-element blocks) written by TMA with the 128-byte
// swizzle: the K-major SWIZZLE_128B layout (rows of 128 bytes, 8-row groups 1024 bytes apart);
// the K = 32 steps inside a row start 32 bytes apart.
__device__ __forceinline__ uint64_t mdesc_a128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// ---------------------------------------------------------------------------------------------
// The tied int8 head for a few tokens (decode): logits[t][row] = x_t . W[row] over every row.
//
// Same exact-limb arithmetic as k_gemm_tc, shaped for 1-4 tokens: the weight rows are the MMA's
// M (128 per tile) and the activation limbs its N (6 limbs x NT tokens, padded to 16 or 32), so
// the tensor pipe does 16 (or 32) columns of work per weight byte and the kernel streams the
// table instead of spending a DFMA per weight.  Code boxes are 128 bytes wide (two blocks, 128-byte
// swizzle): with 64-byte boxes the same kernel streamed at 3.2 TB/s whatever its ring depth,
// epilogue or L2 promotion (measured), so the box rows are what the table stream costs.  Each 64-column block of a tile accumulates into
// its own TMEM columns (the per-block scale is applied in the epilogue), so a tile of 128 rows x
// 14 blocks holds 14 x N columns; tiles alternate between two accumulators.
//
// Persistent: one CTA per SM walks row tiles blockIdx.x, + gridDim.x, ...  Warp 0 streams the
// codes with TMA (they do not depend on the previous kernel, so with programmatic dependent launch
// the weight stream starts while that kernel drains); warps 1-9 then build the limb tile of the
// activations in shared memory (optionally normalised here with the final-norm gain); warp 1
// issues the MMAs; warps 2-9 (two per TMEM lane quadrant, a thread per row and half of the blocks)
// join limbs, take off z * sum(X), scale per block in double, and add the two halves in order.
constexpr uint32_t kHtStages = 10;      // 16 KB code boxes in flight (160 KB)
constexpr uint32_t kHtBox = kTcRows * 128;  // a box: 128 rows x two 64-byte blocks
constexpr uint32_t kHtEpiWarps = 8;     // two per TMEM lane quadrant (block halves)
constexpr uint32_t kHtThreads = 32 * (2 + kHtEpiWarps);
constexpr uint32_t kHtMaxBlocks = 16;   // K <= 1024

template <int NT>  // token capacity: 2 (N = 16) or 4 (N = 32)
__global__ void __launch_bounds__(kHtThreads, 1) k_head_tc(const __grid_constant__ CUtensorMap cmap, const HeadTcArgs a) {
    constexpr uint32_t N = NT <= 2 ? 16 : 32;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sA = smem;                                 // [stages][16 KB] code boxes
    uint8_t* sB = smem + kHtStages * kHtBox;            // [blocks][N x 64] limb tiles (canonical)
    __shared__ __align__(8) uint64_t full[kHtStages], empty[kHtStages], accf[2], acce[2];
    __shared__ long long xsumb[kHtMaxBlocks][NT];      // per block and token: sum of X
    __shared__ double scal[NT];                         // per token: 2^-F
    __shared__ float xs[NT][1024];
    __shared__ double red[NT][kHtThreads / 32];
    __shared__ float amaxs[NT][kHtThreads / 32];
    __shared__ double hsum[2 * 2 * kTcRows * NT];       // [tile parity][half][row][token] partial sums
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t K = a.w.cols, nb = K / kBlock, rows = a.w.rows;
    const uint32_t ntiles = (rows + kTcRows - 1) / kTcRows;
    const uint32_t cols_per_tile = nb * N;
    const uint32_t nacc = 2 * cols_per_tile <= 512 ? 2 : 1;
    const uint32_t spin = g_tc_spin;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < kHtStages; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[i])));
        }
        for (int i = 0; i < 2; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&accf[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&acce[i])), "r"(kHtEpiWarps));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        // ---- producer: a TMA box of 128 rows x 64 code bytes per (tile, block) -------------------
        if (lane == 0) {
            uint32_t issued = 0;
            for (uint32_t tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x)
                for (uint32_t bx = 0; bx < nb / 2; ++bx, ++issued) {
                    const uint32_t s = issued % kHtStages;
                    if (issued >= kHtStages && !mbar_wait_f(&empty[s], ((issued / kHtStages) - 1) & 1, &s_fail, a.err, spin))
                        goto produced;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[s])), "r"(kHtBox)
                                 : "memory");
                    tma_codes(sA + s * kHtBox, &cmap, 2 * bx, tile * kTcRows, &full[s]);  // x = 128 bx bytes
                }
        produced:
            // no copy may still be landing when the CTA releases its shared memory (error path)
            for (uint32_t i = issued > kHtStages ? issued - kHtStages : 0; i < issued; ++i)
                mbar_drain(&full[i % kHtStages], (i / kHtStages) & 1);
        }
        __syncwarp();
    } else {
        // ---- warps 1-9: the activation limbs (after the previous kernel's results are visible) ---
        pdl_wait();
        const uint32_t t5 = tid - 32, n5 = kHtThreads - 32, w5 = t5 >> 5;
        auto bar5 = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(kHtThreads - 32) : "memory"); };
        for (uint32_t i = t5; i < NT * K; i += n5) {
            const uint32_t t = i / K, k = i % K;
            xs[t][k] = t < a.ntok ? a.x[(size_t)t * K + k] : 0.f;
        }
        bar5();
        if (a.gain) {  // the final RMSNorm (test/reference/ops.ts:30-51), one rounding per value
            double ss[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) ss[t] = 0.0;
            for (uint32_t k = t5; k < K; k += n5)
#pragma unroll
                for (int t = 0; t < NT; ++t) ss[t] = fma((double)xs[t][k], (double)xs[t][k], ss[t]);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const double v = warp_sum_d(ss[t]);
                if (lane == 0) red[t][w5] = v;
            }
            bar5();
            double rs[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                double tot = 0.0;
                for (uint32_t w = 0; w < n5 / 32; ++w) tot += red[t][w];
                rs[t] = 1.0 / sqrt(tot / (double)K + (double)a.eps);
            }
            bar5();
            for (uint32_t i = t5; i < NT * K; i += n5) {
                const uint32_t t = i / K, k = i % K;
                const float v = norm_value(xs[t][k], rs[t], a.gain[k]);
                xs[t][k] = v;
                if (blockIdx.x == 0 && a.normed_out && t < a.ntok) a.normed_out[(size_t)t * K + k] = v;
            }
            bar5();
        }
        // F per token from its largest |x|: X = rint(x 2^F) has |X| < 2^46 (exact unless an element
        // is 2^-22 below the largest, as in k_limbs)
        {
            float m[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) m[t] = 0.f;
            for (uint32_t k = t5; k < K; k += n5)
#pragma unroll
                for (int t = 0; t < NT; ++t) m[t] = fmaxf(m[t], fabsf(xs[t][k]));
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_max(m[t]);
                if (lane == 0) amaxs[t][w5] = v;
            }
        }
        for (uint32_t i = t5; i < N * K / 4; i += n5) reinterpret_cast<uint32_t*>(sB)[i] = 0u;  // padding rows stay 0
        bar5();
        auto up_of = [&](uint32_t t) {
            float am = 0.f;
            for (uint32_t w = 0; w < n5 / 32; ++w) am = fmaxf(am, amaxs[t][w]);
            const int e = am == 0.f ? 0 : (int)((__float_as_uint(am) >> 23) & 0xFF) - 126;
            return 46 - e;  // F
        };
        // limb bytes: a thread per (token, element); balanced base-256 digits as in k_limbs
        for (uint32_t i = t5; i < NT * K; i += n5) {
            const uint32_t t = i / K, k = i % K, b = k / kBlock, j = k % kBlock;
            const int F = up_of(t);
            const long long X = __double2ll_rn((double)xs[t][k] * __hiloint2double((1023 + F) << 20, 0));
            const unsigned long long u = (unsigned long long)(X + 0x808080808080LL);
            uint8_t* tb = sB + b * (N * 64);
#pragma unroll
            for (uint32_t l = 0; l < kTcLimbs; ++l) tb[canon(l * NT + t, j)] = (uint8_t)(((u >> (8 * l)) & 0xFF) - 128u);
            if (k == 0) scal[t] = __hiloint2double((1023 - F) << 20, 0);
        }
        // block sums of X: a warp per (block, token), fixed shuffle order
        for (uint32_t bt = w5; bt < nb * NT; bt += n5 / 32) {
            const uint32_t b = bt / NT, t = bt % NT;
            const double up = __hiloint2double((1023 + up_of(t)) << 20, 0);
            long long sx = __double2ll_rn((double)xs[t][b * kBlock + lane] * up) +
                           __double2ll_rn((double)xs[t][b * kBlock + 32 + lane] * up);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
            if (lane == 0) xsumb[b][t] = sx;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // limb bytes visible to the MMA
        bar5();

        if (warp == 1) {
            // ---- MMA issue: one thread --------------------------------------------------------
            if (lane == 0) {
                uint32_t consumed = 0, t_i = 0, last = 0xFFFFFFFFu;
                const uint32_t id = (2u << 4) | (1u << 10) | ((N >> 3) << 17) | ((kTcRows >> 4) << 24);
                for (uint32_t tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x, ++t_i) {
                    const uint32_t acc = t_i % nacc;
                    if (t_i >= nacc && !mbar_wait_f(&acce[acc], ((t_i / nacc) - 1) & 1, &s_fail, a.err, spin)) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    bool ok = true;
                    for (uint32_t bx = 0; bx < nb / 2; ++bx, ++consumed) {
                        const uint32_t s = consumed % kHtStages;
                        if (!mbar_wait_f(&full[s], (consumed / kHtStages) & 1, &s_fail, a.err, spin)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; ++kk) {  // K = 32 steps: blocks 2 bx (kk < 2), 2 bx + 1
                            const uint32_t b = 2 * bx + kk / 2;
                            const uint32_t dcol = tmem + acc * cols_per_tile + b * N;
                            const uint64_t ad = mdesc_a128(su32(sA + s * kHtBox) + kk * 32);
                            const uint64_t bd = mdesc(su32(sB + b * (N * 64)) + (kk & 1) * 256);
                            asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
                                             dcol),
                                         "l"(ad), "l"(bd), "r"(id), "r"(kk & 1));
                        }
                        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                         su32(&empty[s]))
                                     : "memory");
                    }
                    // (also after a failed wait: the drain below then covers the MMAs issued so far)
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     su32(&accf[acc]))
                                 : "memory");
                    last = t_i;
                    if (!ok) break;
                }
                // every issued MMA complete before TMEM is freed
                if (last != 0xFFFFFFFFu) mbar_drain(&accf[last % nacc], (last / nacc) & 1);
            }
            __syncwarp();
        } else {
            // ---- epilogue: warps 2-9, thread = row 32 (warp % 4) + lane of the tile; warps 2-5 take
            // the first half of the blocks, warps 6-9 the second; the halves meet in shared memory
            const uint32_t quad = warp & 3, erow = 32 * quad + lane, half = (warp - 2) >> 2;
            const uint32_t hb = (nb + 1) / 2, b0 = half * hb, b1 = min(nb, b0 + hb);
            uint32_t t_i = 0;
            for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t_i) {
                const uint32_t acc = t_i % nacc, row = tile * kTcRows + erow;
                const bool live = row < rows;
                // this row's scales and zero points of the half, in flight while the tile's MMAs run
                // (zero points are bytes of the packed words, little-endian: byte row * nb + b)
                float sreg[kHtMaxBlocks / 2];
                uint32_t zreg[kHtMaxBlocks / 2];
                const uint8_t* zb = reinterpret_cast<const uint8_t*>(a.w.zeros) + (size_t)row * nb;
#pragma unroll
                for (uint32_t bb = 0; bb < kHtMaxBlocks / 2; ++bb) {
                    const bool use = live && b0 + bb < b1;
                    sreg[bb] = use ? __ldg(a.w.scales + (size_t)row * nb + b0 + bb) : 0.f;
                    zreg[bb] = use ? (uint32_t)__ldg(zb + b0 + bb) : 0u;
                }
                // a warp whose wait gives up still meets the others at the half-sum barrier below
                // (a named barrier cannot time out), then every epilogue warp leaves together
                int ok = 1;
                if (lane == 0) ok = mbar_wait_f(&accf[acc], (t_i / nacc) & 1, &s_fail, a.err, spin);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                double sum[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) sum[t] = 0.0;
                // one block's limb columns -> sum[t] += s * (sum_l d_l 256^l - z * sum(X))
                auto fold = [&](const uint32_t* d, uint32_t bb) {
                    const double sc = (double)sreg[bb];
                    const long long zc = (long long)zreg[bb];
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        // exact: each pair d_l + 256 d_(l+1) fits 32 bits
                        const long long a0 = (long long)((int)d[0 * NT + t] + (int)d[1 * NT + t] * 256);
                        const long long a1 = (long long)((int)d[2 * NT + t] + (int)d[3 * NT + t] * 256);
                        const long long a2 = (long long)((int)d[4 * NT + t] + (int)d[5 * NT + t] * 256);
                        const long long T = a0 + a1 * 65536LL + a2 * 4294967296LL - zc * xsumb[b0 + bb][t];
                        sum[t] = fma((double)T, sc, sum[t]);
                    }
                };
                auto ld16 = [&](uint32_t* d, uint32_t ta) {
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]),
                                   "=r"(d[7]), "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]),
                                   "=r"(d[14]), "=r"(d[15])
                                 : "r"(ta));
                };
                const uint32_t tbase = tmem + (quad * 32u << 16) + acc * cols_per_tile;
                if (!ok) {
                } else if constexpr (N == 16) {  // two blocks per wait
#pragma unroll
                    for (uint32_t bb = 0; bb < kHtMaxBlocks / 2; bb += 2) {
                        if (b0 + bb >= b1) break;
                        uint32_t d0[16], d1[16];
                        ld16(d0, tbase + (b0 + bb) * N);
                        if (b0 + bb + 1 < b1) ld16(d1, tbase + (b0 + bb + 1) * N);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        fold(d0, bb);
                        if (b0 + bb + 1 < b1) fold(d1, bb + 1);
                    }
                } else {
#pragma unroll
                    for (uint32_t bb = 0; bb < kHtMaxBlocks / 2; ++bb) {
                        if (b0 + bb >= b1) break;
                        uint32_t d[32];
                        ld16(d, tbase + (b0 + bb) * N);
                        ld16(d + 16, tbase + (b0 + bb) * N + 16);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        fold(d, bb);
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&acce[acc])) : "memory");
                double* hs = hsum + (size_t)(t_i & 1) * 2 * kTcRows * NT;
#pragma unroll
                for (int t = 0; t < NT; ++t) hs[(half * kTcRows + erow) * NT + t] = sum[t];
                asm volatile("bar.sync 2, %0;" ::"n"(kHtEpiWarps * 32) : "memory");
                if (s_fail) break;  // set before the barrier by any warp that gave up
                if (half == 0 && live)
#pragma unroll
                    for (int t = 0; t < NT; ++t)
                        if ((uint32_t)t < a.ntok)
                            a.out[(size_t)t * a.out_stride + row] =
                                (float)((hs[erow * NT + t] + hs[(kTcRows + erow) * NT + t]) * scal[t]);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

cudaError_t launch_head_tc(const HeadTcArgs& args, cudaStream_t st, bool pdl) {
    const uint32_t nb = args.w.cols / kBlock, N = args.ntok <= 2 ? 16u : 32u;
    if (args.ntok == 0 || args.ntok > 4 || args.w.cols % (2 * kBlock) || nb > kHtMaxBlocks || nb * N > 512)
        return cudaErrorInvalidValue;
    CUtensorMap cmap;
    {
        const cuuint64_t dims[2] = {args.w.cols, args.w.rows};
        const cuuint64_t strides[1] = {args.w.cols};
        const cuuint32_t box[2] = {128, kTcRows};
        const cuuint32_t estr[2] = {1, 1};
        const EncodeTiledFn encode = encode_tiled();
        if (!encode) return cudaErrorNotSupported;
        const CUresult r = encode(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)args.w.packed, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
    const uint32_t ntiles = (args.w.rows + kTcRows - 1) / kTcRows;
    const uint32_t sms = (uint32_t)num_sms();
    const size_t smem = (size_t)kHtStages * kHtBox + (size_t)nb * N * 64;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntiles < sms ? ntiles : sms);
    cfg.blockDim = dim3(kHtThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e;
    if (args.ntok <= 2) {
        e = cudaFuncSetAttribute(k_head_tc<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, k_head_tc<2>, cmap, args);
    } else {
        e = cudaFuncSetAttribute(k_head_tc<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, k_head_tc<4>, cmap, args);
    }
    return e == cudaSuccess ? cudaGetLastError() : e;
}

}  // namespace enx
