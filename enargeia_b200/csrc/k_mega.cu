// Persistent decode step: the whole decoder + tied head for MT tokens in ONE cooperative launch.
//
// A batch-1 decode step of this model moves 351 MB (54 us at the measured HBM rate) but has
// ~100 dependent stages.  As separate kernels each stage pays a launch, a cold activation read
// and a cold weight read in sequence (7-15 us per kernel, measured with ncu).  Here one CTA per
// SM runs every stage.  A producer warp streams the CTA's weight slices for the coming stages
// into a shared-memory ring with TMA bulk copies (cp.async.bulk, full/empty mbarriers), running
// ahead of the grid barriers; 16 consumer warps compute.  What each CTA copies and computes in
// every slice is a table built on the host (mega_build_table), so no thread plans on the device.
//
// Stages per layer (a grid barrier after each):
//   S1  RMSNorm(x) -> q|k|v rows (RoPE pairs) + bias + RoPE; q to global, k/v into the f16 cache
//   S2  attention, one CTA per (token, query head) -> attn_out (no weights)
//   S3  o-projection rows + residual into x
//   S4  RMSNorm(x) -> gate|up rows -> SiLU(gate)*up into `gated`
//   S5  down-projection rows + residual into x
// then the final RMSNorm and this CTA's slice of the tied head rows, streamed in chunks.
// Arithmetic is the faithful double-sum, float-store scheme of k_matvec.cuh.
//
// Grid barriers are a monotonic 64-bit arrival counter (zeroed by a memset node before each
// launch).  Every wait is bounded and reports through `err` instead of hanging; the producer
// waits for its copies in flight before it leaves.  Activations written by other CTAs are read
// with ld.global.cg (L2), never through L1.

#include "k_decode.cuh"
#include "k_mega.cuh"

namespace enx {

constexpr int kMWarps = 16;                  // consumer warps
constexpr int kMConsumers = kMWarps * 32;    // consumer threads (named barrier 1)
constexpr int kMThreads = kMConsumers + 32;  // + one producer warp
constexpr uint32_t kSpinLimit = 1u << 24;    // bounded waits (well under a minute), then an error
constexpr uint32_t kMaxGroup = 8;            // query heads per kv head
constexpr uint32_t kKvStage = 64;            // cached positions staged in shared memory at a time
constexpr int kMaxRes = 96;                  // rows of results exchanged in shared memory per stage

// ---------------------------------------------------------------------------------------------
// PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < kSpinLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Plain (non-multicast) bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_copy(uint32_t dst_smem, unsigned long long src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kMConsumers) : "memory"); }

// Stage trace: consumer thread 0 of CTA 0 stamps %globaltimer at the start of a stage (after its
// barrier), when its weights have landed, and when its compute is done: trace[3*stage + k].
__device__ __forceinline__ void stamp(const MegaArgs& A, uint32_t idx) {
    if (A.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        A.trace[idx] = t;
    }
}

// ---------------------------------------------------------------------------------------------
// grid barrier (consumer threads only; bounded)

__device__ bool grid_sync(const MegaArgs& A, uint32_t& index, volatile int* s_fail) {
    cbar();
    if (threadIdx.x == 0) {
        const unsigned long long target = (unsigned long long)(index + 1) * gridDim.x;
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(A.bar) : "memory");
        for (uint32_t it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(A.bar) : "memory");
            if (v >= target) break;
            if (it > kSpinLimit) {
                atomicMax(A.err, 1u);
                *s_fail = 1;
                break;
            }
            if ((it & 255u) == 255u && *reinterpret_cast<volatile uint32_t*>(A.err)) {
                *s_fail = 1;
                break;
            }
        }
    }
    ++index;
    cbar();
    return !*s_fail;
}

// ---------------------------------------------------------------------------------------------
// dot product of one staged row over chunks [c0, c1): lane l takes chunks c0+l, c0+l+32, ...

template <int BITS, int MT>
__device__ __forceinline__ void row_dot(const uint8_t* slot, const MegaRange& R, uint32_t row, uint32_t cols,
                                        const double2* __restrict__ XD, uint32_t nchunk, uint32_t c0, uint32_t c1,
                                        int lane, double (&acc)[MT]) {
    constexpr int CPB = Geom<BITS>::CPB;
    const uint32_t bpr = cols / kBlock;
    const uint4* P = reinterpret_cast<const uint4*>(slot + R.off_p) + (size_t)(row - R.r0) * nchunk;
    const float* sc = reinterpret_cast<const float*>(slot + R.off_s);
    const uint32_t* zw = reinterpret_cast<const uint32_t*>(slot + R.off_z);
    double a[1][MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) a[0][t] = 0.0;
    for (uint32_t c = c0 + lane; c < c1; c += 32) {
        const uint4 q[1] = {P[c]};
        const uint32_t blk = row * bpr + c / CPB;
        const float s[1] = {sc[blk - R.s_base]};
        const uint32_t zc[1] = {BITS == 4 ? (zw[(blk >> 3) - R.z_base] >> ((blk & 7u) * 4u)) & 0xFu
                                          : (zw[(blk >> 2) - R.z_base] >> ((blk & 3u) * 8u)) & 0xFFu};
        chunk_dot<BITS, MT, 1>(q, s, zc, XD, nchunk, c, a);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = warp_sum_d(a[0][t]);
}

// Two staged rows at once (each x chunk read from shared memory serves both): acc[r][t].
template <int BITS, int MT>
__device__ __forceinline__ void row_dot2(const uint8_t* slot, const MegaRange& Ra, uint32_t ra, const MegaRange& Rb,
                                         uint32_t rb, uint32_t cols, const double2* __restrict__ XD, uint32_t nchunk,
                                         int lane, double (&acc)[2][MT]) {
    if constexpr (MT > 2) {  // register budget: one row at a time
        row_dot<BITS, MT>(slot, Ra, ra, cols, XD, nchunk, 0, nchunk, lane, acc[0]);
        row_dot<BITS, MT>(slot, Rb, rb, cols, XD, nchunk, 0, nchunk, lane, acc[1]);
        return;
    }
    constexpr int CPB = Geom<BITS>::CPB;
    const uint32_t bpr = cols / kBlock;
    const MegaRange* Rs[2] = {&Ra, &Rb};
    const uint32_t rows[2] = {ra, rb};
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = 0.0;
    for (uint32_t c = lane; c < nchunk; c += 32) {
        uint4 q[2];
        float s[2];
        uint32_t zc[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const MegaRange& R = *Rs[r];
            q[r] = (reinterpret_cast<const uint4*>(slot + R.off_p) + (size_t)(rows[r] - R.r0) * nchunk)[c];
            const uint32_t blk = rows[r] * bpr + c / CPB;
            s[r] = reinterpret_cast<const float*>(slot + R.off_s)[blk - R.s_base];
            const uint32_t* zw = reinterpret_cast<const uint32_t*>(slot + R.off_z);
            zc[r] = BITS == 4 ? (zw[(blk >> 3) - R.z_base] >> ((blk & 7u) * 4u)) & 0xFu
                              : (zw[(blk >> 2) - R.z_base] >> ((blk & 3u) * 8u)) & 0xFFu;
        }
        chunk_dot<BITS, MT, 2>(q, s, zc, XD, nchunk, c, acc);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
}

// One pass: read MT rows of x (L2 or shared), RMSNorm them in double, stage the float-rounded
// outputs as doubles.  K * MT must be at most 8 * kMConsumers.
template <int BITS, int MT>
__device__ void load_norm(double* Xd, const float* x, bool from_smem, uint32_t K, const float* gain, float eps,
                          double* rs, double* red) {
    constexpr int PER = 8;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float v[PER];
    double ss[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) ss[t] = 0.0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const uint32_t i = tid + k * kMConsumers;
        v[k] = 0.f;
        if (i < MT * K) v[k] = from_smem ? x[i] : __ldcg(x + i);
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const uint32_t i = tid + k * kMConsumers;
        const uint32_t t = i / K;
#pragma unroll
        for (int u = 0; u < MT; ++u)
            if (i < MT * K && t == (uint32_t)u) ss[u] = fma((double)v[k], (double)v[k], ss[u]);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        const double s = warp_sum_d(ss[t]);
        if (lane == 0) red[t * kMWarps + warp] = s;
    }
    cbar();
    if (tid < MT) {
        double tot = 0.0;
        for (int w = 0; w < kMWarps; ++w) tot += red[tid * kMWarps + w];
        rs[tid] = 1.0 / sqrt(tot / (double)K + (double)eps);
    }
    cbar();
    const uint32_t nchunk = K / Geom<BITS>::E;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const uint32_t i = tid + k * kMConsumers;
        if (i < MT * K) {
            const uint32_t t = i / K, kk = i % K;
            Xd[xd_index<BITS>(t, kk, nchunk)] = (double)norm_value(v[k], rs[t], __ldg(gain + kk));
        }
    }
    cbar();
}

template <int MT>
__device__ __forceinline__ double pick(const double (&a)[MT], int t) {
    double v = 0.0;
#pragma unroll
    for (int i = 0; i < MT; ++i)
        if (i == t) v = a[i];
    return v;
}

// Exact f16 -> double by bit manipulation (the conversion instructions are a slow path): the half
// exponent is rebiased into the double one and the 10 mantissa bits move to the top of the double
// mantissa; zero/subnormal halves are m * 2^-24.
__device__ __forceinline__ double half_bits_to_double(uint32_t b) {
    const uint32_t sgn = (b & 0x8000u) << 16, e = (b >> 10) & 0x1Fu, m = b & 0x3FFu;
    if (e == 0) {
        const double v = (magic_d(m) - 4503599627370496.0) * 0x1p-24;
        return sgn ? -v : v;
    }
    const uint32_t ed = e == 31 ? 0x7FFu : e + 1008u;
    return __hiloint2double((int)(sgn | (ed << 20) | (m << 10)), 0);
}

// Attention of token t, query head h (test/reference/ops.ts:123-204), by one CTA:
//   score_j = float(sum_d q[d] * K[j][d] / sqrt(hd))          (sum in double)
//   w_j     = float(float(exp(score_j - max)) / sum_j exp(.))  (exp and sum in double)
//   out[d]  = float(sum_j w_j * V[j][d])                       (sum in double)
// Cached rows of the kv head are staged in shared memory a chunk at a time.  pw holds the scores,
// then the weights, as doubles (npos <= the activation area's MT * x4 doubles).  `red` needs 32
// doubles.
__device__ void attend(const MegaArgs& A, uint32_t l, uint32_t t, uint32_t h, double* pw, double* qd,
                       uint16_t* kvs, double* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t hd = A.head_dim, kvd = A.kv_heads * hd, g = h / (A.heads / A.kv_heads);
    const uint32_t npos = A.S.pos_of(t) + 1, row8 = hd / 8;
    const uint32_t cap = kKvStage * A.kv_heads;  // positions of one kv head per staged chunk
    const size_t base = A.S.cache_offset(A.S.seq_of(t), l, 0) + g * hd;
    const uint16_t* Kc = A.S.kcache + base;
    const uint16_t* Vc = A.S.vcache + base;
    for (uint32_t d = tid; d < hd; d += kMConsumers) qd[d] = (double)__ldcg(A.S.q + (size_t)t * A.hidden + h * hd + d);
    const double scale = 1.0 / sqrt((double)hd);
    // scores: 8 threads per position, hd/8 dims each, combined over the 8 lanes
    const uint32_t sub = tid & 7;
    float mloc = -INFINITY;
    for (uint32_t j0 = 0; j0 < npos; j0 += cap) {
        const uint32_t n = min(cap, npos - j0);
        for (uint32_t i = tid; i < n * row8; i += kMConsumers)
            reinterpret_cast<uint4*>(kvs)[i] = __ldcg(reinterpret_cast<const uint4*>(Kc + (size_t)(j0 + i / row8) * kvd) + i % row8);
        cbar();
        for (uint32_t jb = 0; jb < n; jb += kMConsumers / 8) {
            const uint32_t j = jb + (tid >> 3);
            double acc = 0.0;
            if (j < n) {
                const uint16_t* kr = kvs + (size_t)j * hd + sub * row8;
                for (uint32_t d = 0; d < row8; ++d) acc = fma(qd[sub * row8 + d], half_bits_to_double(kr[d]), acc);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            if (j < n && sub == 0) {
                const float sc = (float)(acc * scale);
                pw[j0 + j] = (double)sc;
                mloc = fmaxf(mloc, sc);
            }
        }
        cbar();  // chunk consumed
    }
    stamp(A, 3 * (kMegaStages * l + 1) + 1);
    // softmax over npos
    mloc = warp_max(mloc);
    float* redf = reinterpret_cast<float*>(red + kMWarps);
    if (lane == 0) redf[warp] = mloc;
    cbar();
    float m = -INFINITY;
    for (int w = 0; w < kMWarps; ++w) m = fmaxf(m, redf[w]);
    double sloc = 0.0;
    for (uint32_t j = tid; j < npos; j += kMConsumers) {
        const double e = exp(pw[j] - (double)m);
        pw[j] = (double)(float)e;
        sloc += e;
    }
    sloc = warp_sum_d(sloc);
    if (lane == 0) red[warp] = sloc;
    cbar();
    double sum = 0.0;
    for (int w = 0; w < kMWarps; ++w) sum += red[w];
    for (uint32_t j = tid; j < npos; j += kMConsumers) pw[j] = (double)(float)(pw[j] / sum);
    // weighted V: thread (d, slice) sums positions j = slice, slice + S, ... of each chunk
    const uint32_t S = kMConsumers / hd, slice = tid / hd, d = tid % hd;
    double a0 = 0.0, a1 = 0.0;
    for (uint32_t j0 = 0; j0 < npos; j0 += cap) {
        const uint32_t n = min(cap, npos - j0);
        cbar();  // weights final / previous chunk consumed
        for (uint32_t i = tid; i < n * row8; i += kMConsumers)
            reinterpret_cast<uint4*>(kvs)[i] = __ldcg(reinterpret_cast<const uint4*>(Vc + (size_t)(j0 + i / row8) * kvd) + i % row8);
        cbar();
        if (slice < S) {
            uint32_t j = slice;
            for (; j + S < n; j += 2 * S) {
                a0 = fma(pw[j0 + j], half_bits_to_double(kvs[(size_t)j * hd + d]), a0);
                a1 = fma(pw[j0 + j + S], half_bits_to_double(kvs[(size_t)(j + S) * hd + d]), a1);
            }
            if (j < n) a0 = fma(pw[j0 + j], half_bits_to_double(kvs[(size_t)j * hd + d]), a0);
        }
    }
    cbar();
    double* part = reinterpret_cast<double*>(kvs);  // [S][hd]
    if (slice < S) part[slice * hd + d] = a0 + a1;
    cbar();
    if ((uint32_t)tid < hd) {
        double v = 0.0;
        for (uint32_t s2 = 0; s2 < S; ++s2) v += part[s2 * hd + tid];  // fixed order
        A.S.attn_out[(size_t)t * A.hidden + h * hd + tid] = (float)v;
    }
}

// ---------------------------------------------------------------------------------------------
// the kernel

template <int MT, int HB>
__global__ void __launch_bounds__(kMThreads, 1) k_mega(const __grid_constant__ MegaArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double rs[MT], red[MT * kMWarps];
    __shared__ double res[kMaxRes][MT];  // per-row results of a stage, exchanged between warps
    __shared__ volatile int s_fail;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t c = blockIdx.x;
    const uint32_t H = A.hidden, I = A.intermediate, hd = A.head_dim, half = hd / 2;
    const uint32_t NS = A.nslots, SB = A.slot_bytes;

    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMegaSlots;
    uint8_t* slots = smem + 256;
    double* Xd = reinterpret_cast<double*>(slots + (size_t)NS * SB);  // [MT][x4] activations (doubles)
    const double2* XD = reinterpret_cast<const double2*>(Xd);
    float* qs = reinterpret_cast<float*>(Xd + (size_t)MT * A.x4_floats);  // [MT][H] queries / temporary
    uint16_t* kvs = reinterpret_cast<uint16_t*>(qs + (size_t)MT * H);     // [kKvStage][kv*hd] f16 stage

    const MegaSlice* T = A.table + (size_t)c * A.table_stride;
    const uint32_t total = A.nslices[c];

    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // ---------------- producer warp: stream every slice through the ring ---------------------
    if (warp == kMWarps) {
        if (lane != 0) return;
        uint32_t issued = 0;
        for (uint32_t i = 0; i < total; ++i) {
            const uint32_t slot = i % NS;
            if (i >= NS && !mbar_wait_bounded(empty + slot, ((i / NS) - 1) & 1u)) {
                atomicMax(A.err, 2u);
                break;
            }
            if (*reinterpret_cast<volatile uint32_t*>(A.err)) break;
            const MegaSlice& D = T[i];
            const uint32_t base = smem_u32(slots + (size_t)slot * SB);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(full + slot, D.bytes);
            for (uint32_t k = 0; k < D.ncopy; ++k) bulk_copy(base + D.copy[k].dst, D.copy[k].src, D.copy[k].bytes, full + slot);
            issued = i + 1;
        }
        // no copy may still be writing into shared memory when the CTA retires
        for (uint32_t i = issued > NS ? issued - NS : 0; i < issued; ++i) mbar_wait_bounded(full + i % NS, (i / NS) & 1u);
        return;
    }

    // ---------------- consumers ---------------------------------------------------------------
    uint32_t bar_index = 0, slice = 0;
    // Thread 0 alone waits (bounded) so that every consumer takes the same branch; the others
    // then observe the completed phase themselves, which orders the copied bytes before their reads.
    auto wait_slice = [&]() -> bool {
        if (tid == 0 && !mbar_wait_bounded(full + slice % NS, (slice / NS) & 1u)) {
            atomicMax(A.err, 2u);
            s_fail = 1;
        }
        cbar();
        if (s_fail) return false;
        if (tid != 0) mbar_wait_bounded(full + slice % NS, (slice / NS) & 1u);
        return true;
    };
    auto release_slice = [&]() {
        cbar();  // every consumer is done with this slot
        if (tid == 0) mbar_arrive(empty + slice % NS);
        ++slice;
    };
    auto slot_ptr = [&]() { return slots + (size_t)(slice % NS) * SB; };

    for (uint32_t l = 0; l < A.layers; ++l) {
        const LayerArgs& La = A.layer[l];

        // ---------------- S1: RMSNorm + q|k|v + RoPE + cache ---------------------------------
        stamp(A, 3 * (kMegaStages * l + 0));
        if (l == 0) {
            // embedding rows of the tied table (for this CTA's norm); the rows this CTA owns in
            // S3 and S5 also initialise the residual stream
            const MegaSlice& Do = T[1];
            const uint32_t o0 = Do.nrange ? Do.range[0].r0 : 0, o1 = Do.nrange ? Do.range[0].r1 : 0;
            const uint32_t bpr = H / kBlock;
            for (uint32_t i = tid; i < MT * H; i += kMConsumers) {
                const uint32_t t = i / H, k = i % H, row = A.tokens[t];
                const size_t flat = (size_t)row * H + k;
                const uint32_t q = HB == 4 ? (A.head.packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu
                                           : (A.head.packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
                const uint32_t blk = row * bpr + k / kBlock;
                const float v = ((float)q - (float)zero_code<HB>(A.head.zeros, blk)) * A.head.scales[blk];
                qs[i] = v;
                if (k >= o0 && k < o1) A.S.x[i] = v;
            }
            cbar();
            load_norm<4, MT>(Xd, qs, true, H, La.norm_in, A.eps, rs, red);
        } else {
            load_norm<4, MT>(Xd, A.S.x, false, H, La.norm_in, A.eps, rs, red);
        }
        if (!wait_slice()) return;
        stamp(A, 3 * (kMegaStages * l + 0) + 1);
        {
            const MegaSlice& D = T[slice];
            const uint8_t* slot = slot_ptr();
            const uint32_t nrows = D.nrange * 4;  // ranges of 4 rows: (i0..i0+3) then (+half)
            for (uint32_t w = warp; w < nrows; w += kMWarps) {
                const MegaRange& R = D.range[w / 4];
                double acc[MT];
                row_dot<4, MT>(slot, R, R.r0 + w % 4, H, XD, H / 32, 0, H / 32, lane, acc);
                if (lane == 0)
#pragma unroll
                    for (int t = 0; t < MT; ++t) res[w][t] = acc[t];
            }
            cbar();
            // epilogue: a thread per (RoPE pair, token)
            for (uint32_t e = tid; e < (nrows / 2) * MT; e += kMConsumers) {
                const uint32_t p = e / MT, t = e % MT;
                const uint32_t u = p / 4, i4 = p % 4;
                const MegaRange& Ra = D.range[2 * u];
                const uint32_t kind = Ra.tag;
                const uint32_t ra = Ra.r0 + i4, rb = D.range[2 * u + 1].r0 + i4;
                const float* bias = kind == 0 ? La.bq : kind == 1 ? La.bk : La.bv;
                float a = (float)(res[(2 * u) * 4 + i4][t] + (double)bias[ra]);
                float b = (float)(res[(2 * u + 1) * 4 + i4][t] + (double)bias[rb]);
                const uint32_t head = ra / hd, i = ra % hd;
                const uint32_t pos = A.S.pos_of(t);
                if (kind != 2) rope_pair(a, b, A.S.rope_cos[(size_t)pos * half + i], A.S.rope_sin[(size_t)pos * half + i]);
                if (kind == 0) {
                    A.S.q[(size_t)t * H + ra] = a;
                    A.S.q[(size_t)t * H + rb] = b;
                } else {
                    uint16_t* cache = (kind == 1 ? A.S.kcache : A.S.vcache) + A.S.cache_offset(A.S.seq_of(t), l, pos);
                    cache[head * hd + i] = __half_as_ushort(__float2half_rn(a));
                    cache[head * hd + i + half] = __half_as_ushort(__float2half_rn(b));
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 0) + 2);
        if (!grid_sync(A, bar_index, &s_fail)) return;

        // ---------------- S2: attention, one CTA per (token, query head) ---------------------
        stamp(A, 3 * (kMegaStages * l + 1));
        if (c < MT * A.heads) attend(A, l, c / A.heads, c % A.heads, Xd, reinterpret_cast<double*>(qs), kvs, &res[0][0]);
        stamp(A, 3 * (kMegaStages * l + 1) + 2);
        if (!grid_sync(A, bar_index, &s_fail)) return;

        // ---------------- S3: o-projection + residual -----------------------------------------
        stamp(A, 3 * (kMegaStages * l + 2));
        for (uint32_t i = tid; i < MT * H; i += kMConsumers) Xd[xd_index<4>(i / H, i % H, H / 32)] = (double)__ldcg(A.S.attn_out + i);
        cbar();
        if (!wait_slice()) return;
        stamp(A, 3 * (kMegaStages * l + 2) + 1);
        {
            const MegaSlice& D = T[slice];
            if (D.nrange) {
                const MegaRange& R = D.range[0];
                const uint8_t* slot = slot_ptr();
                for (uint32_t r = R.r0 + warp; r < R.r1; r += kMWarps) {
                    double acc[MT];
                    row_dot<4, MT>(slot, R, r, H, XD, H / 32, 0, H / 32, lane, acc);
                    if (lane < MT) {
                        float* xp = A.S.x + (size_t)lane * H + r;
                        *xp = __ldcg(xp) + (float)pick<MT>(acc, lane);
                    }
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 2) + 2);
        if (!grid_sync(A, bar_index, &s_fail)) return;

        // ---------------- S4: RMSNorm + gate|up + SiLU --------------------------------------
        stamp(A, 3 * (kMegaStages * l + 3));
        load_norm<4, MT>(Xd, A.S.x, false, H, La.norm_post, A.eps, rs, red);
        if (!wait_slice()) return;
        stamp(A, 3 * (kMegaStages * l + 3) + 1);
        {
            const MegaSlice& D = T[slice];
            if (D.nrange) {
                const uint8_t* slot = slot_ptr();
                const MegaRange& Rg = D.range[0];
                const MegaRange& Ru = D.range[1];
                const uint32_t nr = Rg.r1 - Rg.r0;
                for (uint32_t i = warp; i < nr; i += kMWarps) {  // gate row i with up row i
                    double acc[2][MT];
                    row_dot2<4, MT>(slot, Rg, Rg.r0 + i, Ru, Ru.r0 + i, H, XD, H / 32, lane, acc);
                    if (lane == 0)
#pragma unroll
                        for (int t = 0; t < MT; ++t) {
                            res[i][t] = acc[0][t];
                            res[nr + i][t] = acc[1][t];
                        }
                }
                cbar();
                for (uint32_t e = tid; e < nr * MT; e += kMConsumers) {
                    const uint32_t i = e / MT, t = e % MT;
                    A.S.gated[(size_t)t * I + Rg.r0 + i] = silu_mul_value((float)res[i][t], (float)res[nr + i][t]);
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 3) + 2);
        if (!grid_sync(A, bar_index, &s_fail)) return;

        // ---------------- S5: down + residual -----------------------------------------------
        stamp(A, 3 * (kMegaStages * l + 4));
        {
            const uint32_t nchunk = I / 32;
            for (uint32_t i = tid; i < MT * I; i += kMConsumers)
                Xd[xd_index<4>(i / I, i % I, nchunk)] = (double)__ldcg(A.S.gated + i);
            cbar();
        }
        if (!wait_slice()) return;
        stamp(A, 3 * (kMegaStages * l + 4) + 1);
        {
            const MegaSlice& D = T[slice];
            if (D.nrange) {
                const MegaRange& R = D.range[0];
                const uint8_t* slot = slot_ptr();
                const uint32_t nr = R.r1 - R.r0, nchunk = I / 32;
                const uint32_t parts = nr >= (uint32_t)kMWarps ? 1 : kMWarps / nr;  // split K across warps
                for (uint32_t w = warp; w < nr * parts; w += kMWarps) {
                    const uint32_t i = w / parts, p = w % parts;
                    const uint32_t c0 = nchunk * p / parts, c1 = nchunk * (p + 1) / parts;
                    double acc[MT];
                    row_dot<4, MT>(slot, R, R.r0 + i, I, XD, nchunk, c0, c1, lane, acc);
                    if (lane == 0)
#pragma unroll
                        for (int t = 0; t < MT; ++t) res[w][t] = acc[t];
                }
                cbar();
                for (uint32_t e = tid; e < nr * MT; e += kMConsumers) {
                    const uint32_t i = e / MT, t = e % MT;
                    double v = 0.0;
                    for (uint32_t p = 0; p < parts; ++p) v += res[i * parts + p][t];  // fixed order
                    float* xp = A.S.x + (size_t)t * H + R.r0 + i;
                    *xp = __ldcg(xp) + (float)v;
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 4) + 2);
        if (!grid_sync(A, bar_index, &s_fail)) return;
    }

    // ---------------- final RMSNorm + tied head ---------------------------------------------
    stamp(A, 3 * (kMegaStages * A.layers));
    load_norm<HB, MT>(Xd, A.S.x, false, H, A.final_norm, A.eps, rs, red);
    if (c == 0)
        for (uint32_t i = tid; i < MT * H; i += kMConsumers)
            A.S.normed[i] = norm_value(__ldcg(A.S.x + i), rs[i / H], A.final_norm[i % H]);
    const uint32_t nchunk = H / Geom<HB>::E;
    while (slice < total) {
        if (!wait_slice()) return;
        const MegaSlice& D = T[slice];
        if (D.nrange) {
            const MegaRange& R = D.range[0];
            const uint8_t* slot = slot_ptr();
            for (uint32_t r = R.r0 + 2 * warp; r < R.r1; r += 2 * kMWarps) {
                const uint32_t r2 = r + 1 < R.r1 ? r + 1 : r;
                double acc[2][MT];
                row_dot2<HB, MT>(slot, R, r, R, r2, H, XD, nchunk, lane, acc);
                if (lane < MT) A.S.logits[(size_t)lane * A.vocab + r] = (float)pick<MT>(acc[0], lane);
                if (lane < MT && r2 != r) A.S.logits[(size_t)lane * A.vocab + r2] = (float)pick<MT>(acc[1], lane);
            }
        }
        release_slice();
    }
    stamp(A, 3 * (kMegaStages * A.layers) + 2);
}

// ---------------------------------------------------------------------------------------------
// host side

static uint32_t split_lo(uint32_t total, uint32_t parts, uint32_t i, uint32_t granule) {
    const uint32_t units = total / granule;
    return (uint32_t)(((uint64_t)units * i) / parts) * granule;
}

// Adds the copies and the compute record of rows [r0, r1) of `w` at byte `cursor` of the slot.
static uint32_t plan_range(MegaSlice& S, const QW& w, int bits, uint32_t r0, uint32_t r1, uint32_t tag,
                           uint32_t cursor) {
    auto down16 = [](uint64_t v) { return v & ~uint64_t(15); };
    auto up16 = [](uint64_t v) { return (v + 15) & ~uint64_t(15); };
    MegaRange& R = S.range[S.nrange++];
    R.r0 = r0;
    R.r1 = r1;
    R.tag = tag;
    const uint64_t row_bytes = (uint64_t)w.cols * bits / 8, bpr = w.cols / kBlock, zpw = 32 / bits;
    const uint64_t pb = r0 * row_bytes, pn = (r1 - r0) * row_bytes;  // multiple of 16 (cols % 64 == 0)
    const uint64_t sb = down16(r0 * bpr * 4), se = up16(r1 * bpr * 4);
    const uint64_t zb = down16((r0 * bpr / zpw) * 4), ze = up16(((r1 * bpr + zpw - 1) / zpw) * 4);
    R.off_p = cursor;
    S.copy[S.ncopy++] = MegaCopy{(unsigned long long)(reinterpret_cast<const uint8_t*>(w.packed) + pb), (uint32_t)pn, cursor};
    cursor += (uint32_t)pn;
    R.off_s = cursor;
    R.s_base = (uint32_t)(sb / 4);
    S.copy[S.ncopy++] = MegaCopy{(unsigned long long)(reinterpret_cast<const uint8_t*>(w.scales) + sb), (uint32_t)(se - sb), cursor};
    cursor += (uint32_t)(se - sb);
    R.off_z = cursor;
    R.z_base = (uint32_t)(zb / 4);
    S.copy[S.ncopy++] = MegaCopy{(unsigned long long)(reinterpret_cast<const uint8_t*>(w.zeros) + zb), (uint32_t)(ze - zb), cursor};
    cursor += (uint32_t)(ze - zb);
    S.bytes += (uint32_t)(pn + (se - sb) + (ze - zb));
    return (uint32_t)up16(cursor);
}

void mega_build_table(const MegaArgs& A, const MegaGeometry& g, std::vector<MegaSlice>& table,
                      std::vector<uint32_t>& counts, uint32_t& stride) {
    const uint32_t G = g.grid, L = A.layers;
    uint32_t max_head = 0;
    for (uint32_t c = 0; c < G; ++c) {
        const uint32_t h0 = split_lo(A.vocab, G, c, 1), h1 = split_lo(A.vocab, G, c + 1, 1);
        const uint32_t n = (h1 - h0 + g.head_chunk - 1) / g.head_chunk;
        max_head = n > max_head ? n : max_head;
    }
    stride = 4 * L + max_head;
    table.assign((size_t)G * stride, MegaSlice{});
    counts.assign(G, 0);
    const uint32_t half = A.head_dim / 2, per_slot = half / 4;
    const uint32_t units = (A.heads + 2 * A.kv_heads) * per_slot;
    for (uint32_t c = 0; c < G; ++c) {
        MegaSlice* T = table.data() + (size_t)c * stride;
        for (uint32_t l = 0; l < L; ++l) {
            const LayerArgs& La = A.layer[l];
            {  // S1: units of 4 RoPE pairs of one head slot of the q|k|v row space
                MegaSlice& S = T[4 * l];
                uint32_t cur = 0;
                for (uint32_t u = c; u < units && S.nrange + 2 <= 4; u += G) {
                    const uint32_t hs = u / per_slot, i0 = (u % per_slot) * 4;
                    const QW* w;
                    uint32_t head, kind;
                    if (hs < A.heads) { w = &La.wq; head = hs; kind = 0; }
                    else if (hs < A.heads + A.kv_heads) { w = &La.wk; head = hs - A.heads; kind = 1; }
                    else { w = &La.wv; head = hs - A.heads - A.kv_heads; kind = 2; }
                    const uint32_t b = head * A.head_dim + i0;
                    cur = plan_range(S, *w, 4, b, b + 4, kind, cur);
                    cur = plan_range(S, *w, 4, b + half, b + half + 4, kind, cur);
                }
            }
            {
                const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
                if (r1 > r0) plan_range(T[4 * l + 1], La.wo, 4, r0, r1, 0, 0);
            }
            {
                const uint32_t r0 = split_lo(A.intermediate, G, c, 1), r1 = split_lo(A.intermediate, G, c + 1, 1);
                if (r1 > r0) {
                    const uint32_t cur = plan_range(T[4 * l + 2], La.wg, 4, r0, r1, 0, 0);
                    plan_range(T[4 * l + 2], La.wu, 4, r0, r1, 0, cur);
                }
            }
            {
                const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
                if (r1 > r0) plan_range(T[4 * l + 3], La.wd, 4, r0, r1, 0, 0);
            }
        }
        const uint32_t h0 = split_lo(A.vocab, G, c, 1), h1 = split_lo(A.vocab, G, c + 1, 1);
        uint32_t j = 0;
        for (uint32_t r0 = h0; r0 < h1; r0 += g.head_chunk, ++j) {
            const uint32_t r1 = r0 + g.head_chunk < h1 ? r0 + g.head_chunk : h1;
            plan_range(T[4 * L + j], A.head, A.head_bits, r0, r1, 0, 0);
        }
        counts[c] = 4 * L + j;
    }
}

template <int MT, int HB>
static cudaError_t launch_mega_t(const MegaArgs& A, uint32_t grid, size_t smem, cudaStream_t st) {
    cudaError_t e = cudaFuncSetAttribute(k_mega<MT, HB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_mega<MT, HB>, A);
}

MegaGeometry mega_geometry(uint32_t mt, const MegaArgs& A) {
    MegaGeometry g{};
    int dev = 0, sms = 148, maxsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    g.grid = (uint32_t)sms;
    g.head_chunk = 32;
    const uint32_t x4 = A.intermediate > A.hidden ? A.intermediate : A.hidden;
    g.x4_floats = x4;
    auto range_bytes = [](uint32_t rows, uint32_t cols, uint32_t bits) {
        const uint32_t bpr = cols / 64;
        return rows * cols * bits / 8 + rows * bpr * 4 + 32 + rows * bpr * bits / 8 + 32 + 48;
    };
    const uint32_t rows4 = (A.intermediate + g.grid - 1) / g.grid + 1;
    const uint32_t rows5 = ((A.hidden / 2 + g.grid - 1) / g.grid) * 2 + 2;
    uint32_t slot = 2 * range_bytes(rows4, A.hidden, 4);
    const uint32_t s5 = range_bytes(rows5, A.intermediate, 4);
    const uint32_t s1 = 4 * range_bytes(4, A.hidden, 4);
    const uint32_t hc = range_bytes(g.head_chunk, A.hidden, (uint32_t)A.head_bits);
    if (s5 > slot) slot = s5;
    if (s1 > slot) slot = s1;
    if (hc > slot) slot = hc;
    slot = (slot + 127) & ~127u;
    g.slot_bytes = slot;
    const size_t fixed = 256 + (size_t)mt * x4 * 8 + (size_t)mt * A.hidden * 4 + (size_t)kKvStage * A.kv_heads * A.head_dim * 2;
    const size_t statics = sizeof(double) * (mt + mt * kMWarps + kMaxRes * mt) + 64;
    const int64_t room = (int64_t)maxsm - (int64_t)fixed - (int64_t)statics - 1024;
    int ns = room > 0 ? (int)(room / slot) : 0;
    if (ns > (int)kMegaSlots) ns = kMegaSlots;
    g.nslots = (uint32_t)ns;
    g.smem = fixed + (size_t)g.nslots * slot;
    g.max_positions = mt * x4;  // scores of one head, as doubles, in the activation area
    // shapes the kernel's fixed per-CTA capacities cannot take: report no ring (not eligible)
    const uint32_t s1_units = (A.heads + 2 * A.kv_heads) * (A.head_dim / 8);
    const uint32_t rows_up = (A.intermediate + g.grid - 1) / g.grid + 1;
    if (s1_units > 2 * g.grid || 2 * rows_up > (uint32_t)kMaxRes || rows5 > (uint32_t)kMaxRes ||
        (size_t)mt * A.hidden > 8 * (size_t)kMConsumers ||
        A.hidden > 2 * (uint32_t)kMConsumers || A.head_dim % 8 != 0 || A.heads / A.kv_heads > kMaxGroup)
        g.nslots = 0;
    return g;
}

cudaError_t launch_mega(uint32_t mt, const MegaArgs& A, const MegaGeometry& g, cudaStream_t st) {
    const bool h8 = A.head_bits == 8;
    switch (mt) {
        case 1: return h8 ? launch_mega_t<1, 8>(A, g.grid, g.smem, st) : launch_mega_t<1, 4>(A, g.grid, g.smem, st);
        case 2: return h8 ? launch_mega_t<2, 8>(A, g.grid, g.smem, st) : launch_mega_t<2, 4>(A, g.grid, g.smem, st);
        default: return h8 ? launch_mega_t<4, 8>(A, g.grid, g.smem, st) : launch_mega_t<4, 4>(A, g.grid, g.smem, st);
    }
}

}  // namespace enx
