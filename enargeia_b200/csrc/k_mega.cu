// Persistent decode step: the whole decoder + tied head for MT tokens in ONE cooperative launch.
//
// A batch-1 decode step of this model moves 351 MB (54 us at the measured HBM rate) but is a
// chain of dependent stages.  As separate kernels each stage pays a launch, a cold activation
// read and a cold weight read in sequence.  Here one CTA per SM runs every stage.  A producer
// warp streams the CTA's weight slices for the coming stages into a shared-memory ring with bulk
// copies (cp.async.bulk, full/empty mbarriers), running ahead of the consumers; 16 consumer
// warps compute.  What each CTA copies and computes in every slice is a table built on the host
// (mega_build_table), so no thread plans on the device.
//
// Per layer, four stages hand their outputs on through tagged words (see "Tagged activations"
// below), each reader waiting only for the words it needs, with no grid barrier:
//   A  every CTA: RMSNorm(x) -> its units of q|k|v rows (4 RoPE pairs each) + bias + RoPE; q and
//      the f16 k|v values out as tagged words, k|v into the cache too.  One attention CTA per
//      (token, query head) reads its head's q and its kv head's current k|v row, runs attention
//      over the cached positions (history prefetched with cp.async at the start of the stage) and
//      writes its head's output.
//   O  every CTA: reads the attention output -> its rows of the o-projection + residual (x_mid)
//   C  every CTA: reads x_mid -> RMSNorm -> its gate|up rows -> SiLU(gate)*up (gated)
//   D  every CTA: reads gated -> its down-projection rows + residual (x)
// The final RMSNorm and the tied head follow in a separate kernel (launch_head_tc).  Norm gains
// and q|k|v biases travel in the slices with the weights.
// Arithmetic is the faithful double-sum, float-store scheme of k_matvec.cuh.
//
// Every wait is bounded and reports through `err` instead of hanging; the producer waits for its
// copies in flight before it leaves.

#include "k_decode.cuh"
#include "k_mega.cuh"

namespace enx {

constexpr int kMWarps = 16;                  // consumer warps
constexpr int kMConsumers = kMWarps * 32;    // consumer threads (named barrier 1)
constexpr int kMThreads = kMConsumers + 32;  // + one producer warp
constexpr uint32_t kSpinLimit = 1u << 24;    // bounded waits (well under a minute), then an error

// Spins a wait may take before it gives up (enx_set_wait_limit; per device).  The producer's final
// drain of its copies in flight always uses kSpinLimit.
__device__ uint32_t g_mega_spin = kSpinLimit;
constexpr uint32_t kKvHalfs = 16384;         // f16 staging of cached K and V rows (32 KB)
constexpr int kMaxRes = 96;                  // rows per token exchanged in shared memory (C, D)
constexpr int kHeadDimMax = 64;
constexpr int kMaxChunks = 192;             // chunks of a staged activation row (K <= 6144)

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
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Plain bulk copy global -> this CTA's own shared memory (one destination CTA).
__device__ __forceinline__ void bulk_copy(uint32_t dst_smem, unsigned long long src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 16-byte asynchronous copy global -> shared (L2 only), completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kMConsumers) : "memory"); }

// Stage trace: consumer thread 0 of CTA 0 stamps %globaltimer at the start of a stage (after its
// barrier), when its first weights have landed, and when its compute is done: trace[3*stage + k].
__device__ __forceinline__ void stamp(const MegaArgs& A, uint32_t idx) {
    if (A.trace && blockIdx.x == A.trace_cta && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        A.trace[idx] = t;
    }
}

// Detail stamps of stage A (CTA 0): trace[3*(kMegaStages*layers + 1) + kADetail*l + k].
constexpr uint32_t kADetail = kMegaTraceDetail;
__device__ __forceinline__ void stamp_a(const MegaArgs& A, uint32_t l, uint32_t k) {
    stamp(A, 3 * (kMegaStages * A.layers + 1) + kADetail * l + k);
}


// ---------------------------------------------------------------------------------------------
// Tagged activations between stages (no grid barriers).
//
// Every value one stage hands to the next travels as one 64-bit word {value, tag}, written with a
// single 8-byte store; tag = 32 * epoch + layer, the epoch counting launches (bumped before each
// launch by the step's prep kernel).  A reader polls the words it needs until each carries the
// tag it expects: a word is written whole or not at all, so a matching tag proves its value is
// this layer's, with no fence on the writer's side and no arrival counter to wait for first.
// Buffers alternate between two copies by layer parity, so a writer of layer l can only overwrite
// words of layer l - 2, which every CTA has read before any CTA can reach layer l (each stage
// needs every CTA's output of the stage before it).
// Measured on the whole step (config 0), this beat release/acquire grid barriers with plain data
// (733 -> 642 us per step), arrival counters bumped with relaxed adds before the tagged reads
// (742 us) or with release adds (840 us), and polling every missing word of a batch together
// (1100 us: the polls flood L2); every fence or extra round trip sits on the critical path.

__device__ __forceinline__ uint32_t ll_tag(uint32_t epoch, uint32_t layer) { return epoch * 32u + layer; }
__device__ __forceinline__ uint32_t ll_epoch(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ll_store(unsigned long long* p, uint32_t v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)tag << 32) | v) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Polls one word until it carries `tag` (bounded; gives up early once the error word is set).
__device__ __forceinline__ bool ll_poll(const unsigned long long* p, unsigned long long& v, uint32_t tag, uint32_t spin,
                                        const uint32_t* err) {
    for (uint32_t it = 0; (uint32_t)(v >> 32) != tag; ++it) {
        if (it >= spin || ((it & 63u) == 63u && *reinterpret_cast<const volatile uint32_t*>(err))) return false;
        v = ll_load(p);
    }
    return true;
}
// Consumer thread i reads words i, i + kMConsumers, ... of src[0, n), kLLBatch loads in flight,
// and hands each value to f(index, value); a word without the tag yet is polled alone until it
// lands.  Returns false if a poll gave up (error word set).
constexpr int kLLBatch = 10;
template <class F>
__device__ __forceinline__ bool ll_read(const unsigned long long* src, uint32_t n, uint32_t tag, uint32_t spin,
                                        uint32_t* err, F f) {
    for (uint32_t i0 = threadIdx.x; i0 < n; i0 += kLLBatch * kMConsumers) {
        unsigned long long v[kLLBatch];
#pragma unroll
        for (int k = 0; k < kLLBatch; ++k) {
            const uint32_t i = i0 + k * kMConsumers;
            v[k] = i < n ? ll_load(src + i) : ((unsigned long long)tag << 32);
        }
#pragma unroll
        for (int k = 0; k < kLLBatch; ++k) {
            const uint32_t i = i0 + k * kMConsumers;
            if (i >= n) break;
            if (!ll_poll(src + i, v[k], tag, spin, err)) {
                atomicMax(err, 1u);
                return false;
            }
            f(i, (uint32_t)v[k]);
        }
    }
    return true;
}
// Two arrays of n words at once (a head's k and v rows): both sets of loads in flight together.
template <class F, class G>
__device__ __forceinline__ bool ll_read2(const unsigned long long* a, const unsigned long long* b, uint32_t n, uint32_t tag,
                                         uint32_t spin, uint32_t* err, F fa, G fb) {
    for (uint32_t i = threadIdx.x; i < 2 * n; i += kMConsumers) {
        const unsigned long long* p = i < n ? a + i : b + (i - n);
        unsigned long long v = ll_load(p);
        if (!ll_poll(p, v, tag, spin, err)) {
            atomicMax(err, 1u);
            return false;
        }
        if (i < n) fa(i, (uint32_t)v);
        else fb(i - n, (uint32_t)v);
    }
    return true;
}
// The tagged buffers of one launch: two copies (layer parity) of, per token, x after the down
// stage, q, the f16 k|v row, the attention output, x after the o-projection, and the gated
// activations.
struct LLView {
    unsigned long long* base;
    uint32_t mt, H, kvd, I;
    __device__ __forceinline__ size_t per() const { return (size_t)mt * (4 * H + 2 * kvd + I); }
    __device__ __forceinline__ unsigned long long* at(uint32_t l, size_t off) const { return base + (l & 1) * per() + off; }
    __device__ __forceinline__ unsigned long long* x(uint32_t l) const { return at(l, 0); }
    __device__ __forceinline__ unsigned long long* q(uint32_t l) const { return at(l, (size_t)mt * H); }
    __device__ __forceinline__ unsigned long long* kv(uint32_t l) const { return at(l, (size_t)mt * 2 * H); }
    __device__ __forceinline__ unsigned long long* attn(uint32_t l) const { return at(l, (size_t)mt * (2 * H + 2 * kvd)); }
    __device__ __forceinline__ unsigned long long* xmid(uint32_t l) const { return at(l, (size_t)mt * (3 * H + 2 * kvd)); }
    __device__ __forceinline__ unsigned long long* gated(uint32_t l) const { return at(l, (size_t)mt * (4 * H + 2 * kvd)); }
};

// ---------------------------------------------------------------------------------------------
// dot products against staged rows

// One chunk of R rows against MT tokens with biased codes: (B + q) becomes an exact double in a
// single byte permute (B = 16 for int4, 4096 for int8, the code landing in the top mantissa
// bits), so each element costs one DFMA; the bias comes off once per chunk as (B + z) * sum(x)
// with the chunk sums xsum precomputed for all rows.  Products stay exact ((B + q) * x needs at
// most 37 bits); the sums are double sums like the reference's, in another order.
template <int BITS, int MT, int R>
__device__ __forceinline__ void chunk_dot_b(const uint4 (&q)[R], const float (&s)[R], const uint32_t (&zc)[R],
                                            const double2* __restrict__ XD, const double* __restrict__ xsum,
                                            uint32_t nchunk, uint32_t c, double (&acc)[R][MT]) {
    constexpr int F2 = Geom<BITS>::F2;
    constexpr int NP = 4;
    constexpr double B = BITS == 4 ? 16.0 : 4096.0;
    uint32_t wv[R][BITS == 4 ? 8 : 4];  // int4: per word, even nibbles then odd nibbles as bytes 0x3q
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint32_t w4[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (BITS == 4) {
                wv[r][2 * i] = (w4[i] & 0x0F0F0F0Fu) | 0x30303030u;
                wv[r][2 * i + 1] = ((w4[i] >> 4) & 0x0F0F0F0Fu) | 0x30303030u;
            } else {
                wv[r][i] = w4[i];
            }
        }
    }
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
                const double xe = e == 0 ? xv.x : xv.y;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    uint32_t hi;
                    if (BITS == 4) {  // element el = nibble (el & 7) of word el >> 3
                        const uint32_t src = wv[r][2 * (el >> 3) + (el & 1)];
                        hi = __byte_perm(src, 0x40000000u, 0x7054u | ((uint32_t)((el & 7) >> 1) << 8));
                    } else {  // element el = byte (el & 3) of word el >> 2
                        hi = __byte_perm(wv[r][el >> 2], 0x40B00000u, 0x7604u | ((uint32_t)(el & 3) << 4));
                    }
                    part[r][el % NP] = fma(__hiloint2double((int)hi, 0), xe, part[r][el % NP]);
                }
            }
        }
        const double xs = xsum[t * nchunk + c];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const double p = fma(-(B + (double)zc[r]), xs, (part[r][0] + part[r][1]) + (part[r][2] + part[r][3]));
            acc[r][t] = fma(p, (double)s[r], acc[r][t]);
        }
    }
}

// Chunk sums of the staged activations (for chunk_dot_b): xsum[t * nchunk + c].
template <int BITS, int MT>
__device__ __forceinline__ void stage_xsum(const double* Xd, double* xsum, uint32_t nchunk) {
    constexpr int F2 = Geom<BITS>::F2;
    const double2* XD = reinterpret_cast<const double2*>(Xd);
    for (uint32_t t = 0; t < MT; ++t)
        for (uint32_t c = threadIdx.x; c < nchunk; c += kMConsumers) {
            double sum = 0.0;
#pragma unroll
            for (int j = 0; j < F2; ++j) {
                const double2 v = XD[(t * F2 + j) * nchunk + c];
                sum += v.x + v.y;
            }
            xsum[t * nchunk + c] = sum;
        }
}

// One staged row over chunks [c0, c1): lane l takes chunks c0+l, c0+l+32, ...
template <int BITS, int MT>
__device__ __forceinline__ void row_dot(const uint8_t* slot, const MegaRange& R, uint32_t row, uint32_t cols,
                                        const double2* __restrict__ XD, const double* __restrict__ xsum, uint32_t nchunk,
                                        uint32_t c0, uint32_t c1, int lane, double (&acc)[MT]) {
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
        chunk_dot_b<BITS, MT, 1>(q, s, zc, XD, xsum, nchunk, c, a);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = warp_sum_d(a[0][t]);
}

// Two staged rows at once (each x chunk read from shared memory serves both): acc[r][t].
template <int BITS, int MT>
__device__ __forceinline__ void row_dot2(const uint8_t* slot, const MegaRange& Ra, uint32_t ra, const MegaRange& Rb,
                                         uint32_t rb, uint32_t cols, const double2* __restrict__ XD,
                                         const double* __restrict__ xsum, uint32_t nchunk, int lane, double (&acc)[2][MT]) {
    if constexpr (MT > 2) {  // register budget: one row at a time
        row_dot<BITS, MT>(slot, Ra, ra, cols, XD, xsum, nchunk, 0, nchunk, lane, acc[0]);
        row_dot<BITS, MT>(slot, Rb, rb, cols, XD, xsum, nchunk, 0, nchunk, lane, acc[1]);
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
        chunk_dot_b<BITS, MT, 2>(q, s, zc, XD, xsum, nchunk, c, acc);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
}

// One pass: read MT rows of x (L2 or shared), RMSNorm them in double, stage the float-rounded
// outputs as doubles.  K <= 2 * kMConsumers.
template <int BITS, int MT>
__device__ void load_norm(double* Xd, double* xsum, const float* x, bool from_smem, uint32_t K, const float* gain,
                          float eps, double* rs, double* red, float* keep = nullptr, const MegaArgs* tr = nullptr,
                          uint32_t tl = 0) {
    constexpr int PER = 2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float v[MT][PER], gv[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const uint32_t i = tid + k * kMConsumers;
        gv[k] = i < K ? gain[i] : 0.f;  // shared (staged with the weights) or global
#pragma unroll
        for (int t = 0; t < MT; ++t) v[t][k] = i < K ? (from_smem ? x[t * K + i] : __ldcg(x + t * K + i)) : 0.f;
    }
    if (keep)  // a copy of the raw rows (the residual) in shared memory
#pragma unroll
        for (int k = 0; k < PER; ++k)
#pragma unroll
            for (int t = 0; t < MT; ++t)
                if (tid + k * kMConsumers < K) keep[t * K + tid + k * kMConsumers] = v[t][k];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < PER; ++k) ss = fma((double)v[t][k], (double)v[t][k], ss);
        ss = warp_sum_d(ss);
        if (lane == 0) red[t * kMWarps + warp] = ss;
    }
    cbar();
    if (tr) stamp_a(*tr, tl, 6);
    if (tid < MT) {
        double tot = 0.0;
        for (int w = 0; w < kMWarps; ++w) tot += red[tid * kMWarps + w];
        rs[tid] = 1.0 / sqrt(tot / (double)K + (double)eps);
    }
    cbar();
    if (tr) stamp_a(*tr, tl, 7);
    const uint32_t nchunk = K / Geom<BITS>::E;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const uint32_t i = tid + k * kMConsumers;
        if (i < K)
#pragma unroll
            for (int t = 0; t < MT; ++t) Xd[xd_index<BITS>(t, i, nchunk)] = (double)norm_value(v[t][k], rs[t], gv[k]);
    }
    cbar();
    stage_xsum<BITS, MT>(Xd, xsum, nchunk);
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

// Shared state of an attention CTA (one token, one head).
struct HeadSmem {
    double qd[kHeadDimMax];  // rotated query (float values)
    __align__(16) uint16_t kcur[kHeadDimMax];
    __align__(16) uint16_t vcur[kHeadDimMax];
    double ad[kHeadDimMax];  // attention output (float values)
    float red[kMWarps];
    double redd[kMWarps];
};

// Attention of one query head over positions [0, npos) (test/reference/ops.ts:123-204):
//   score_j = float(sum_d q[d] * K[j][d] / sqrt(hd))          (sum in double)
//   w_j     = float(float(exp(score_j - max)) / sum_j exp(.))  (exp and sum in double)
//   out[d]  = float(sum_j w_j * V[j][d])                       (sum in double)
// Rows [0, min(npos, cap)) of K and V are already staged in kst / vst; longer contexts stream
// further chunks from the cache.  pw (npos doubles) holds the scores, then the weights.  Leaves
// the output in hs.ad.
__device__ void attend(const MegaArgs& A, uint32_t l, uint32_t t, uint32_t g, uint32_t pos, double* pw,
                       uint16_t* kst, uint16_t* vst, uint32_t cap, HeadSmem& hs) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t hd = A.head_dim, kvd = A.kv_heads * hd, row8 = hd / 8, npos = pos + 1;
    const size_t base = A.S.cache_offset(A.S.seq_of(t), l, 0) + g * hd;
    const uint16_t* Kc = A.S.kcache + base;
    const uint16_t* Vc = A.S.vcache + base;
    const double scale = 1.0 / sqrt((double)hd);
    // f16 -> f32 -> double through the conversion units: exact, and in this loop (few
    // conversions per loaded byte, integer pipe busy with addressing) faster than bit moves
    auto h2d = [](uint16_t v) { return (double)__half2float(__ushort_as_half(v)); };
    const uint32_t lr8 = hd == 64 ? 3 : 2;  // row8 = 1 << lr8 (head_dim 32 or 64)
    auto stage_rows = [&](uint16_t* st, const uint16_t* src, const uint16_t* cur, uint32_t j0, uint32_t n) {
        for (uint32_t i = tid; i < (n << lr8); i += kMConsumers) {
            const uint32_t j = j0 + (i >> lr8);
            reinterpret_cast<uint4*>(st)[i] = j == pos ? reinterpret_cast<const uint4*>(cur)[i & (row8 - 1)]
                                                       : __ldcg(reinterpret_cast<const uint4*>(src + (size_t)j * kvd) + (i & (row8 - 1)));
        }
    };
    // scores: 8 threads per position, hd/8 dims each, combined over the 8 lanes
    const uint32_t sub = tid & 7;
    float mloc = -INFINITY;
    for (uint32_t j0 = 0; j0 < npos; j0 += cap) {
        const uint32_t n = min(cap, npos - j0);
        if (j0 > 0) {
            cbar();  // previous chunk consumed
            stage_rows(kst, Kc, hs.kcur, j0, n);
            cbar();
        }
        for (uint32_t jb = 0; jb < n; jb += kMConsumers / 8) {
            const uint32_t j = jb + (tid >> 3);
            double acc = 0.0;
            if (j < n) {
                const uint16_t* kr = kst + (size_t)j * hd + sub * row8;
                for (uint32_t d = 0; d < row8; ++d) acc = fma(hs.qd[sub * row8 + d], h2d(kr[d]), acc);
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
    }
    stamp_a(A, l, 8);
    // softmax over npos
    mloc = warp_max(mloc);
    if (lane == 0) hs.red[warp] = mloc;
    cbar();
    float m = -INFINITY;
    for (int w = 0; w < kMWarps; ++w) m = fmaxf(m, hs.red[w]);
    double sloc = 0.0;
    for (uint32_t j = tid; j < npos; j += kMConsumers) {
        const double e = exp(pw[j] - (double)m);
        pw[j] = (double)(float)e;
        sloc += e;
    }
    sloc = warp_sum_d(sloc);
    if (lane == 0) hs.redd[warp] = sloc;
    cbar();
    double sum = 0.0;
    for (int w = 0; w < kMWarps; ++w) sum += hs.redd[w];
    for (uint32_t j = tid; j < npos; j += kMConsumers) pw[j] = (double)(float)(pw[j] / sum);
    stamp_a(A, l, 9);
    // weighted V: thread (d, slice) sums positions j = slice, slice + S, ... of each chunk
    const uint32_t S = kMConsumers / hd, slice = tid / hd, d = tid % hd;
    double a0 = 0.0, a1 = 0.0;
    for (uint32_t j0 = 0; j0 < npos; j0 += cap) {
        const uint32_t n = min(cap, npos - j0);
        cbar();  // weights final / previous chunk consumed
        if (j0 > 0) {
            stage_rows(vst, Vc, hs.vcur, j0, n);
            cbar();
        }
        if (slice < S) {
            uint32_t j = slice;
            for (; j + S < n; j += 2 * S) {
                a0 = fma(pw[j0 + j], h2d(vst[(size_t)j * hd + d]), a0);
                a1 = fma(pw[j0 + j + S], h2d(vst[(size_t)(j + S) * hd + d]), a1);
            }
            if (j < n) a0 = fma(pw[j0 + j], h2d(vst[(size_t)j * hd + d]), a0);
        }
    }
    cbar();
    stamp_a(A, l, 10);
    double* part = reinterpret_cast<double*>(kst);  // [S][hd]
    if (slice < S) part[slice * hd + d] = a0 + a1;
    cbar();
    if ((uint32_t)tid < hd) {
        double v = 0.0;
        for (uint32_t s2 = 0; s2 < S; ++s2) v += part[s2 * hd + tid];  // fixed order
        hs.ad[tid] = (double)(float)v;
    }
    cbar();
}

// ---------------------------------------------------------------------------------------------
// the kernel

// A consumer leaves early (a bounded wait gave up): its own cp.async copies land first.
#define BAIL()               \
    do {                     \
        cp_async_wait_all(); \
        return;              \
    } while (0)

template <int MT, int HB>
__global__ void __launch_bounds__(kMThreads, 1) k_mega(const __grid_constant__ MegaArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double rs[MT], red[MT * kMWarps];
    __shared__ double res[kMaxRes * MT];  // per-row results of a stage, exchanged between warps
    __shared__ double rope_c[MT][kHeadDimMax / 2], rope_s[MT][kHeadDimMax / 2];  // this step's RoPE rows
    __shared__ HeadSmem hs;
    __shared__ uint32_t spos[MT];  // this step's positions
    __shared__ double xsum[MT * kMaxChunks];  // chunk sums of the staged activations
    __shared__ __align__(16) MegaSlice sdesc[kMegaSlots];  // descriptors of the slices in the ring
    __shared__ volatile int s_fail;
    __shared__ uint32_t s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t c = blockIdx.x;
    const uint32_t H = A.hidden, I = A.intermediate, hd = A.head_dim, half = hd / 2;
    const uint32_t NS = A.nslots, SB = A.slot_bytes;
    const uint32_t group = A.heads / A.kv_heads;
    const uint32_t spin = g_mega_spin;

    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMegaSlots;
    uint8_t* slots = smem + 256;
    double* Xd = reinterpret_cast<double*>(slots + (size_t)NS * SB);  // [MT][x4] activations (doubles)
    const double2* XD = reinterpret_cast<const double2*>(Xd);
    float* xs = reinterpret_cast<float*>(Xd + (size_t)MT * A.x4_floats);  // [MT][H] residual after attention
    uint16_t* kst = reinterpret_cast<uint16_t*>(xs + (((size_t)MT * H + 3) & ~size_t(3)));
    uint16_t* vst = kst + kKvHalfs / 2;
    const uint32_t cap = kKvHalfs / 2 / hd;  // cached positions per staged chunk

    const MegaSlice* T = A.table + (size_t)c * A.table_stride;
    const uint32_t total = A.nslices[c];
    // attention role: (token, query head) for the first MT * heads CTAs
    const bool att = c < MT * A.heads;
    const uint32_t at = att ? c / A.heads : 0, ah = att ? c % A.heads : 0;
    const uint32_t ag = ah / group;

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
    // Lane k issues copy k of a slice; the next slice's descriptor is fetched before waiting for
    // its slot, so the table reads overlap the wait.
    if (warp == kMWarps) {
        static_assert(sizeof(MegaSlice) % 16 == 0 && sizeof(MegaSlice) / 16 <= 32, "descriptor = one uint4 per lane");
        constexpr uint32_t kDescVecs = sizeof(MegaSlice) / 16;
        uint4 dv = make_uint4(0, 0, 0, 0);  // this lane's 16 bytes of the next descriptor
        auto fetch = [&](uint32_t i) {
            if (i < total && (uint32_t)lane < kDescVecs) dv = reinterpret_cast<const uint4*>(T + i)[lane];
            // descriptors further ahead: into L2 now, so the fetch above hits it later
            const uint32_t ahead = i + 2 + lane / 4;
            if ((lane & 3) < 4 && ahead < total && lane < 16)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const uint8_t*>(T + ahead) + (lane & 3) * 128));
        };
        fetch(0);
        uint32_t issued = 0;
        for (uint32_t i = 0; i < total; ++i) {
            const uint32_t slot = i % NS;
            int ok = 1;
            if (lane == 0) {
                if (i >= NS && !mbar_wait_bounded(empty + slot, ((i / NS) - 1) & 1u, spin)) {
                    atomicMax(A.err, 2u);
                    ok = 0;
                }
                if (*reinterpret_cast<volatile uint32_t*>(A.err)) ok = 0;
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            // publish the descriptor next to its data slot; the consumers read it from there
            if ((uint32_t)lane < kDescVecs) reinterpret_cast<uint4*>(sdesc + slot)[lane] = dv;
            __syncwarp();
            const MegaSlice& D = sdesc[slot];
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(full + slot, D.bytes);
            }
            __syncwarp();
            const uint32_t base = smem_u32(slots + (size_t)slot * SB);
            if ((uint32_t)lane < D.ncopy) bulk_copy(base + D.copy[lane].dst, D.copy[lane].src, D.copy[lane].bytes, full + slot);
            for (uint32_t k = lane; k < D.rows.n; k += 32)
                bulk_copy(base + D.rows.dst + k * D.rows.dst_stride, D.rows.src + (unsigned long long)k * D.rows.src_stride,
                          D.rows.bytes, full + slot);
            issued = i + 1;
            fetch(i + 1);
        }
        // no copy may still be writing into shared memory when the CTA retires
        if (lane == 0)
            for (uint32_t i = issued > NS ? issued - NS : 0; i < issued; ++i)
                mbar_wait_bounded(full + i % NS, (i / NS) & 1u, kSpinLimit);
        return;
    }

    // ---------------- consumers ---------------------------------------------------------------
    uint32_t slice = 0;
    // Thread 0 alone waits (bounded) so that every consumer takes the same branch.  Its wait
    // acquires the completed phase (the copied bytes); the barrier after it carries that order to
    // every other consumer, so they read the slot without polling the mbarrier themselves.
    auto wait_slice = [&]() -> bool {
        if (tid == 0 && !mbar_wait_bounded(full + slice % NS, (slice / NS) & 1u, spin)) {
            atomicMax(A.err, 2u);
            s_fail = 1;
        }
        cbar();
        return !s_fail;
    };
    auto release_slice = [&]() {
        cbar();  // every consumer is done with this slot
        if (tid == 0) mbar_arrive(empty + slice % NS);
        ++slice;
    };
    auto slot_ptr = [&]() { return slots + (size_t)(slice % NS) * SB; };
    // After an ll_read: every consumer learns whether any of them gave up.
    auto ll_done = [&](bool ok) -> bool {
        if (!ok) s_fail = 1;
        cbar();
        return !s_fail;
    };

    if (tid == 0) s_epoch = ll_epoch(A.ll_epoch);
    if (tid < MT) spos[tid] = A.S.pos_of(tid);
    cbar();
    const uint32_t epoch = s_epoch;
    const uint32_t apos = att ? spos[at] : 0;
    // the RoPE rows of this step's positions (same for every layer)
    for (uint32_t i = tid; i < MT * half; i += kMConsumers) {
        const uint32_t t = i / half, p = i % half, pos = spos[t];
        rope_c[t][p] = __ldg(A.S.rope_cos + (size_t)pos * half + p);
        rope_s[t][p] = __ldg(A.S.rope_sin + (size_t)pos * half + p);
    }
    const uint32_t kvd = A.kv_heads * hd;
    const LLView V{A.ll, MT, H, kvd, I};

    for (uint32_t l = 0; l < A.layers; ++l) {
        const uint32_t tag = ll_tag(epoch, l), ptag = ll_tag(epoch, l - 1);

        // ---------------- A: q|k|v units, then (attention CTAs) attention --------------------
        stamp(A, 3 * (kMegaStages * l + 0));
        if (att) {  // this head's cached K/V rows [0, min(pos, cap)), in flight during the units
            const uint32_t row8 = hd / 8;
            const size_t base = A.S.cache_offset(A.S.seq_of(at), l, 0) + ag * hd;
            const uint32_t pre = min(apos, cap), lr8 = hd == 64 ? 3 : 2;  // row8 = hd / 8 = 1 << lr8
            for (uint32_t i = tid; i < (pre << lr8); i += kMConsumers) {
                const uint32_t j = i >> lr8, d8 = i & (row8 - 1);
                const size_t off = base + (size_t)j * kvd + d8 * 8;
                cp_async16(kst + (size_t)j * hd + d8 * 8, A.S.kcache + off);
                cp_async16(vst + (size_t)j * hd + d8 * 8, A.S.vcache + off);
            }
            cp_async_commit();
        }
        if (!wait_slice()) BAIL();
        stamp(A, 3 * (kMegaStages * l + 0) + 1);
        {
            const MegaSlice& D = sdesc[slice % NS];
            const uint8_t* slot = slot_ptr();
            const float* gain = reinterpret_cast<const float*>(slot + D.off_v);
            if (l == 0) {
                // embedding rows of the tied table (every CTA: the residual of its o rows)
                const uint32_t bpr = H / kBlock;
                for (uint32_t i = tid; i < MT * H; i += kMConsumers) {
                    const uint32_t t = i / H, k = i % H, row = A.tokens[t];
                    const size_t flat = (size_t)row * H + k;
                    const uint32_t q = HB == 4 ? (A.head.packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu
                                               : (A.head.packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
                    const uint32_t blk = row * bpr + k / kBlock;
                    xs[i] = ((float)q - (float)zero_code<HB>(A.head.zeros, blk)) * A.head.scales[blk];
                }
                cbar();
            } else {  // x of the previous layer's down stage, every row of it
                const bool ok = ll_read(V.x(l - 1), MT * H, ptag, spin, A.err, [&](uint32_t i, uint32_t v) { xs[i] = __uint_as_float(v); });
                if (!ll_done(ok)) BAIL();
            }
            stamp_a(A, l, 7);
            load_norm<4, MT>(Xd, xsum, xs, true, H, gain, A.eps, rs, red);
            stamp_a(A, l, 0);
            // q|k|v units: ranges of 4 rows, (i0..i0+3) then (+half), a warp per row
            const uint32_t nrows = D.nrange * 4;
            for (uint32_t w = warp; w < nrows; w += kMWarps) {
                const MegaRange& Rr = D.range[w / 4];
                double acc[MT];
                row_dot<4, MT>(slot, Rr, Rr.r0 + w % 4, H, XD, xsum, H / 32, 0, H / 32, lane, acc);
                if (lane == 0)
#pragma unroll
                    for (int t = 0; t < MT; ++t) res[w * MT + t] = acc[t];
            }
            cbar();
            // epilogue: a thread per (RoPE pair, token): bias, RoPE (q, k), f16 rounding (k, v);
            // q and the f16 k|v values go out through the tagged buffers, k|v into the cache too
            for (uint32_t e = tid; e < (nrows / 2) * MT; e += kMConsumers) {
                const uint32_t p = e / MT, t = e % MT;
                const uint32_t u = p / 4, i4 = p % 4;
                const MegaRange& Ra = D.range[2 * u];
                const MegaRange& Rb = D.range[2 * u + 1];
                const uint32_t kind = Ra.tag;
                const uint32_t ra = Ra.r0 + i4, rb = Rb.r0 + i4;
                const float ba = reinterpret_cast<const float*>(slot + Ra.off_b)[i4];
                const float bb = reinterpret_cast<const float*>(slot + Rb.off_b)[i4];
                float a = (float)(res[((2 * u) * 4 + i4) * MT + t] + (double)ba);
                float b = (float)(res[((2 * u + 1) * 4 + i4) * MT + t] + (double)bb);
                const uint32_t head = ra / hd, i = ra % hd;
                if (kind != 2) rope_pair(a, b, rope_c[t][i], rope_s[t][i]);
                if (kind == 0) {
                    ll_store(V.q(l) + (size_t)t * H + ra, __float_as_uint(a), tag);
                    ll_store(V.q(l) + (size_t)t * H + rb, __float_as_uint(b), tag);
                } else {
                    uint16_t* cache = (kind == 1 ? A.S.kcache : A.S.vcache) + A.S.cache_offset(A.S.seq_of(t), l, spos[t]);
                    const uint16_t ha = __half_as_ushort(__float2half_rn(a)), hb = __half_as_ushort(__float2half_rn(b));
                    cache[head * hd + i] = ha;
                    cache[head * hd + i + half] = hb;
                    unsigned long long* kv = V.kv(l) + (size_t)t * 2 * kvd + (kind == 1 ? 0 : kvd) + head * hd;
                    ll_store(kv + i, ha, tag);
                    ll_store(kv + i + half, hb, tag);
                }
            }
            release_slice();
        }
        stamp_a(A, l, 1);
        if (att) {
            // this head's rotated query and the step's f16 k|v row of its kv head
            const unsigned long long* qsrc = V.q(l) + (size_t)at * H + ah * hd;
            const unsigned long long* kvsrc = V.kv(l) + (size_t)at * 2 * kvd + ag * hd;
            bool ok = ll_read(qsrc, hd, tag, spin, A.err, [&](uint32_t d, uint32_t v) { hs.qd[d] = (double)__uint_as_float(v); });
            ok = ok && ll_read2(kvsrc, kvsrc + kvd, hd, tag, spin, A.err,
                                [&](uint32_t d, uint32_t v) { hs.kcur[d] = (uint16_t)v; },
                                [&](uint32_t d, uint32_t v) { hs.vcur[d] = (uint16_t)v; });
            if (!ll_done(ok)) BAIL();
            stamp_a(A, l, 2);
            if (apos < cap)  // the row written this step joins the staged history
                for (uint32_t d = tid; d < hd; d += kMConsumers) {
                    kst[(size_t)apos * hd + d] = hs.kcur[d];
                    vst[(size_t)apos * hd + d] = hs.vcur[d];
                }
            cp_async_wait_all();
            cbar();
            stamp_a(A, l, 3);
            attend(A, l, at, ag, apos, Xd, kst, vst, cap, hs);
            for (uint32_t d = tid; d < hd; d += kMConsumers)
                ll_store(V.attn(l) + (size_t)at * H + ah * hd + d, __float_as_uint((float)hs.ad[d]), tag);
            stamp_a(A, l, 4);
        }
        // ---------------- O: every CTA, its rows of the o-projection + residual ---------------
        {
            const bool ok = ll_read(V.attn(l), MT * H, tag, spin, A.err,
                                    [&](uint32_t i, uint32_t v) { Xd[xd_index<4>(i / H, i % H, H / 32)] = (double)__uint_as_float(v); });
            if (!ll_done(ok)) BAIL();
        }
        stamp_a(A, l, 5);
        stage_xsum<4, MT>(Xd, xsum, H / 32);
        if (!wait_slice()) BAIL();
        {
            const MegaSlice& D = sdesc[slice % NS];
            if (D.nrange) {
                const MegaRange& Rr = D.range[0];
                const uint8_t* slot = slot_ptr();
                const uint32_t nr = Rr.r1 - Rr.r0, nchunk = H / 32;
                const uint32_t parts = nr >= (uint32_t)kMWarps ? 1 : kMWarps / nr;  // split K across warps
                for (uint32_t w = warp; w < nr * parts; w += kMWarps) {
                    const uint32_t i = w / parts, p = w % parts;
                    const uint32_t c0 = nchunk * p / parts, c1 = nchunk * (p + 1) / parts;
                    double acc[MT];
                    row_dot<4, MT>(slot, Rr, Rr.r0 + i, H, XD, xsum, nchunk, c0, c1, lane, acc);
                    if (lane == 0)
#pragma unroll
                        for (int t = 0; t < MT; ++t) res[w * MT + t] = acc[t];
                }
                cbar();
                for (uint32_t e = tid; e < nr * MT; e += kMConsumers) {
                    const uint32_t i = e / MT, t = e % MT;
                    double v = 0.0;
                    for (uint32_t p = 0; p < parts; ++p) v += res[(i * parts + p) * MT + t];  // fixed order
                    const float xm = xs[(size_t)t * H + Rr.r0 + i] + (float)v;
                    ll_store(V.xmid(l) + (size_t)t * H + Rr.r0 + i, __float_as_uint(xm), tag);
                }
            }
        }
        release_slice();
        stamp_a(A, l, 6);
        stamp(A, 3 * (kMegaStages * l + 0) + 2);

        // ---------------- C: residual + RMSNorm + gate|up + SiLU ----------------------------
        stamp(A, 3 * (kMegaStages * l + 1));
        {  // x_mid, every row (the residual of D stays in xs)
            const bool ok = ll_read(V.xmid(l), MT * H, tag, spin, A.err, [&](uint32_t i, uint32_t v) { xs[i] = __uint_as_float(v); });
            if (!ll_done(ok)) BAIL();
        }
        if (!wait_slice()) BAIL();
        stamp(A, 3 * (kMegaStages * l + 1) + 1);
        {
            const MegaSlice& D = sdesc[slice % NS];
            const uint8_t* slot = slot_ptr();
            load_norm<4, MT>(Xd, xsum, xs, true, H, reinterpret_cast<const float*>(slot + D.off_v), A.eps, rs, red);
            stamp_a(A, l, 11);
            if (D.nrange) {
                const MegaRange& Rg = D.range[0];
                const MegaRange& Ru = D.range[1];
                const uint32_t nr = Rg.r1 - Rg.r0, nchunk = H / 32;
                if (MT == 1 && 2 * nr * nchunk * MT <= kKvHalfs / 4) {
                    // (row pair, chunk) units spread over every consumer thread: 33 rows of 28
                    // chunks take 2 rounds instead of 3 warp-per-row rounds with 28 of 32 lanes.
                    // Partials land in the K/V staging area (free in this stage) and are summed
                    // per row in chunk order.
                    double* part = reinterpret_cast<double*>(kst);  // [2][nr][nchunk][MT]
                    const uint32_t bpr = H / kBlock;
                    const uint32_t* zg = reinterpret_cast<const uint32_t*>(slot + Rg.off_z);
                    const uint32_t* zu = reinterpret_cast<const uint32_t*>(slot + Ru.off_z);
                    for (uint32_t u = tid; u < nr * nchunk; u += kMConsumers) {
                        const uint32_t i = u / nchunk, c = u % nchunk;
                        const uint32_t bg = (Rg.r0 + i) * bpr + c / Geom<4>::CPB, bu = (Ru.r0 + i) * bpr + c / Geom<4>::CPB;
                        const uint4 q[2] = {(reinterpret_cast<const uint4*>(slot + Rg.off_p) + (size_t)i * nchunk)[c],
                                            (reinterpret_cast<const uint4*>(slot + Ru.off_p) + (size_t)i * nchunk)[c]};
                        const float sv[2] = {reinterpret_cast<const float*>(slot + Rg.off_s)[bg - Rg.s_base],
                                             reinterpret_cast<const float*>(slot + Ru.off_s)[bu - Ru.s_base]};
                        const uint32_t zc[2] = {(zg[(bg >> 3) - Rg.z_base] >> ((bg & 7u) * 4u)) & 0xFu,
                                                (zu[(bu >> 3) - Ru.z_base] >> ((bu & 7u) * 4u)) & 0xFu};
                        double a[2][MT];
#pragma unroll
                        for (int r = 0; r < 2; ++r)
#pragma unroll
                            for (int t = 0; t < MT; ++t) a[r][t] = 0.0;
                        chunk_dot_b<4, MT, 2>(q, sv, zc, XD, xsum, nchunk, c, a);
#pragma unroll
                        for (int r = 0; r < 2; ++r)
#pragma unroll
                            for (int t = 0; t < MT; ++t) part[(((size_t)r * nr + i) * nchunk + c) * MT + t] = a[r][t];
                    }
                    cbar();
                    for (uint32_t e = tid; e < 2 * nr * MT; e += kMConsumers) {
                        const uint32_t ri = e / MT, t = e % MT;  // ri = r * nr + i
                        const double* pp = part + (size_t)ri * nchunk * MT + t;
                        double v = 0.0;
                        for (uint32_t c = 0; c < nchunk; ++c) v += pp[(size_t)c * MT];  // chunk order
                        res[ri * MT + t] = v;
                    }
                } else {
                    for (uint32_t i = warp; i < nr; i += kMWarps) {  // gate row i with up row i
                        double acc[2][MT];
                        row_dot2<4, MT>(slot, Rg, Rg.r0 + i, Ru, Ru.r0 + i, H, XD, xsum, nchunk, lane, acc);
                        if (lane == 0)
#pragma unroll
                            for (int t = 0; t < MT; ++t) {
                                res[i * MT + t] = acc[0][t];
                                res[(nr + i) * MT + t] = acc[1][t];
                            }
                    }
                }
                cbar();
                stamp_a(A, l, 12);
                for (uint32_t e = tid; e < nr * MT; e += kMConsumers) {
                    const uint32_t i = e / MT, t = e % MT;
                    const float gv = silu_mul_value((float)res[i * MT + t], (float)res[(nr + i) * MT + t]);
                    ll_store(V.gated(l) + (size_t)t * I + Rg.r0 + i, __float_as_uint(gv), tag);
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 1) + 2);

        // ---------------- D: down + residual ------------------------------------------------
        stamp(A, 3 * (kMegaStages * l + 2));
        {
            const uint32_t nchunk = I / 32;
            const bool ok = ll_read(V.gated(l), MT * I, tag, spin, A.err,
                                    [&](uint32_t i, uint32_t v) { Xd[xd_index<4>(i / I, i % I, nchunk)] = (double)__uint_as_float(v); });
            if (!ll_done(ok)) BAIL();
            stamp_a(A, l, 13);
            stage_xsum<4, MT>(Xd, xsum, nchunk);
        }
        if (!wait_slice()) BAIL();
        stamp(A, 3 * (kMegaStages * l + 2) + 1);
        {
            const MegaSlice& D = sdesc[slice % NS];
            if (D.nrange) {
                const MegaRange& Rr = D.range[0];
                const uint8_t* slot = slot_ptr();
                const uint32_t nr = Rr.r1 - Rr.r0, nchunk = I / 32;
                const uint32_t parts = nr >= (uint32_t)kMWarps ? 1 : kMWarps / nr;  // split K across warps
                for (uint32_t w = warp; w < nr * parts; w += kMWarps) {
                    const uint32_t i = w / parts, p = w % parts;
                    const uint32_t c0 = nchunk * p / parts, c1 = nchunk * (p + 1) / parts;
                    double acc[MT];
                    row_dot<4, MT>(slot, Rr, Rr.r0 + i, I, XD, xsum, nchunk, c0, c1, lane, acc);
                    if (lane == 0)
#pragma unroll
                        for (int t = 0; t < MT; ++t) res[w * MT + t] = acc[t];
                }
                cbar();
                for (uint32_t e = tid; e < nr * MT; e += kMConsumers) {
                    const uint32_t i = e / MT, t = e % MT;
                    double v = 0.0;
                    for (uint32_t p = 0; p < parts; ++p) v += res[(i * parts + p) * MT + t];  // fixed order
                    const float xn = xs[(size_t)t * H + Rr.r0 + i] + (float)v;
                    ll_store(V.x(l) + (size_t)t * H + Rr.r0 + i, __float_as_uint(xn), tag);
                    if (l + 1 == A.layers) A.S.x[(size_t)t * H + Rr.r0 + i] = xn;  // for the head kernel
                }
            }
        }
        release_slice();
        stamp(A, 3 * (kMegaStages * l + 2) + 2);
    }

    // the final RMSNorm and the tied head run in the next kernel (the tensor-core head, or the
    // CUDA-core head for an int4 table), which reads the last layer's x from S.x
    stamp(A, 3 * (kMegaStages * A.layers));
    stamp(A, 3 * (kMegaStages * A.layers) + 2);
}

// ---------------------------------------------------------------------------------------------
// host side

static uint32_t split_lo(uint32_t total, uint32_t parts, uint32_t i, uint32_t granule) {
    const uint32_t units = total / granule;
    return (uint32_t)(((uint64_t)units * i) / parts) * granule;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static uint32_t up16(uint32_t v) { return (v + 15) & ~15u; }

// Adds a plain copy of `bytes` (a multiple of 16, 16-byte aligned source) at byte `cursor`.
static uint32_t plan_copy(MegaSlice& S, const void* src, uint32_t bytes, uint32_t cursor) {
    S.copy[S.ncopy++] = MegaCopy{(unsigned long long)src, bytes, cursor};
    S.bytes += bytes;
    return up16(cursor + bytes);
}

// Adds the copies and the compute record of rows [r0, r1) of `w` at byte `cursor` of the slot,
// and their biases when `bias` is given (r0 and r1 multiples of 4).  bpr = scales per row (0:
// cols / 64).
static uint32_t plan_range(MegaSlice& S, const QW& w, int bits, uint32_t r0, uint32_t r1, uint32_t tag,
                           uint32_t cursor, uint32_t bpr_override = 0, const float* bias = nullptr) {
    auto down16 = [](uint64_t v) { return v & ~uint64_t(15); };
    auto up16l = [](uint64_t v) { return (v + 15) & ~uint64_t(15); };
    MegaRange& R = S.range[S.nrange++];
    R.r0 = r0;
    R.r1 = r1;
    R.tag = tag;
    const uint64_t row_bytes = (uint64_t)w.cols * bits / 8, zpw = 32 / bits;
    const uint64_t bpr = bpr_override ? bpr_override : w.cols / kBlock;
    const uint64_t pb = r0 * row_bytes, pn = (r1 - r0) * row_bytes;  // multiple of 16 (cols % 32 == 0)
    const uint64_t sb = down16(r0 * bpr * 4), se = up16l(r1 * bpr * 4);
    const uint64_t zb = down16((r0 * bpr / zpw) * 4), ze = up16l(((r1 * bpr + zpw - 1) / zpw) * 4);
    R.off_p = cursor;
    cursor = plan_copy(S, reinterpret_cast<const uint8_t*>(w.packed) + pb, (uint32_t)pn, cursor);
    R.off_s = cursor;
    R.s_base = (uint32_t)(sb / 4);
    cursor = plan_copy(S, reinterpret_cast<const uint8_t*>(w.scales) + sb, (uint32_t)(se - sb), cursor);
    R.off_z = cursor;
    R.z_base = (uint32_t)(zb / 4);
    cursor = plan_copy(S, reinterpret_cast<const uint8_t*>(w.zeros) + zb, (uint32_t)(ze - zb), cursor);
    if (bias) {
        R.off_b = cursor;
        cursor = plan_copy(S, bias + r0, (r1 - r0) * 4, cursor);
    }
    return cursor;
}

void mega_build_table(uint32_t mt, const MegaArgs& A, const MegaGeometry& g,
                      std::vector<MegaSlice>& table, std::vector<uint32_t>& counts, uint32_t& stride) {
    const uint32_t G = g.grid, L = A.layers, hd = A.head_dim, half = hd / 2, per_slot = half / 4;
    const uint32_t units = (A.heads + 2 * A.kv_heads) * per_slot;
    stride = 4 * L;
    table.assign((size_t)G * stride, MegaSlice{});
    counts.assign(G, 0);
    for (uint32_t c = 0; c < G; ++c) {
        MegaSlice* T = table.data() + (size_t)c * stride;
        uint32_t i = 0;
        for (uint32_t l = 0; l < L; ++l) {
            const LayerArgs& La = A.layer[l];
            {  // q|k|v units of 4 RoPE pairs (this CTA's share), after the input-norm gain
                MegaSlice& S = T[i++];
                S.off_v = 0;
                uint32_t cur = plan_copy(S, La.norm_in, A.hidden * 4, 0);
                for (uint32_t u = c; u < units; u += G) {
                    const uint32_t hs = u / per_slot, i0 = (u % per_slot) * 4;
                    const QW* w;
                    const float* bias;
                    uint32_t head, kind;
                    if (hs < A.heads) { w = &La.wq; bias = La.bq; head = hs; kind = 0; }
                    else if (hs < A.heads + A.kv_heads) { w = &La.wk; bias = La.bk; head = hs - A.heads; kind = 1; }
                    else { w = &La.wv; bias = La.bv; head = hs - A.heads - A.kv_heads; kind = 2; }
                    const uint32_t b = head * hd + i0;
                    cur = plan_range(S, *w, 4, b, b + 4, kind, cur, 0, bias);
                    cur = plan_range(S, *w, 4, b + half, b + half + 4, kind, cur, 0, bias);
                }
            }
            {  // this CTA's rows of the o-projection (the rows it owns in D too)
                const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
                if (r1 > r0) plan_range(T[i], La.wo, 4, r0, r1, 0, 0);
                ++i;
            }
            {
                MegaSlice& S = T[i++];
                S.off_v = 0;
                uint32_t cur = plan_copy(S, La.norm_post, A.hidden * 4, 0);
                const uint32_t r0 = split_lo(A.intermediate, G, c, 1), r1 = split_lo(A.intermediate, G, c + 1, 1);
                if (r1 > r0) {
                    cur = plan_range(S, La.wg, 4, r0, r1, 0, cur);
                    plan_range(S, La.wu, 4, r0, r1, 0, cur);
                }
            }
            {
                const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
                if (r1 > r0) plan_range(T[i], La.wd, 4, r0, r1, 0, 0);
                ++i;
            }
        }
        counts[c] = i;
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
    const uint32_t x4 = A.intermediate > A.hidden ? A.intermediate : A.hidden;
    g.x4_floats = x4;
    auto range_bytes = [](uint32_t rows, uint32_t cols, uint32_t bits, uint32_t bpr) {
        return rows * cols * bits / 8 + rows * bpr * 4 + 32 + rows * bpr * bits / 8 + 32 + 48 + rows * 4 + 16;
    };
    const uint32_t bprH = A.hidden / 64, bprI = A.intermediate / 64, gain = A.hidden * 4 + 16;
    const uint32_t rows4 = (A.intermediate + g.grid - 1) / g.grid + 1;
    const uint32_t rows5 = ((A.hidden / 2 + g.grid - 1) / g.grid) * 2 + 2;
    const uint32_t units = (A.heads + 2 * A.kv_heads) * (A.head_dim / 8);
    const uint32_t upc = (units + g.grid - 1) / g.grid;  // q|k|v units per CTA
    uint32_t slot = gain + 2 * range_bytes(rows4, A.hidden, 4, bprH);
    const uint32_t cand[3] = {range_bytes(rows5, A.intermediate, 4, bprI), gain + upc * 2 * range_bytes(4, A.hidden, 4, bprH),
                              range_bytes(rows5, A.hidden, 4, bprH)};
    for (uint32_t v : cand) slot = v > slot ? v : slot;
    slot = (slot + 127) & ~127u;
    g.slot_bytes = slot;
    const size_t fixed = 256 + (size_t)mt * x4 * 8 + (((size_t)mt * A.hidden * 4 + 15) & ~size_t(15)) + (size_t)kKvHalfs * 2;
    const size_t statics = sizeof(double) * (mt + mt * kMWarps + kMaxRes * mt + mt * kHeadDimMax) + sizeof(HeadSmem) +
                           sizeof(MegaSlice) * kMegaSlots + sizeof(double) * mt * kMaxChunks + 64;
    const int64_t room = (int64_t)maxsm - (int64_t)fixed - (int64_t)statics - 1024;
    int ns = room > 0 ? (int)(room / slot) : 0;
    if (ns > (int)kMegaSlots) ns = kMegaSlots;
    g.nslots = (uint32_t)ns;
    g.smem = fixed + (size_t)g.nslots * slot;
    g.max_positions = mt * x4;  // scores of one head, as doubles, in the activation area
    // shapes the kernel's fixed per-CTA capacities cannot take: report no ring (not eligible)
    if (upc > 2 || A.intermediate / 32 > (uint32_t)kMaxChunks || A.hidden / 16 > (uint32_t)kMaxChunks || 2 * rows4 > (uint32_t)kMaxRes || rows5 > (uint32_t)kMaxRes || mt * A.heads > g.grid ||
        (A.head_dim != 32 && A.head_dim != 64) || A.hidden % 64 != 0 || A.intermediate % 64 != 0 ||
        A.hidden > 2 * (uint32_t)kMConsumers || A.kv_heads == 0 || A.heads % A.kv_heads != 0 ||
        A.kv_heads * (size_t)mt + 3 > kMegaBarWords)
        g.nslots = 0;
    return g;
}

cudaError_t mega_set_spin(uint32_t spins) {
    const uint32_t v = spins ? spins : kSpinLimit;
    return cudaMemcpyToSymbol(g_mega_spin, &v, sizeof(v));
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
