// Persistent decode step: the whole decoder + tied head for MT tokens in ONE cooperative launch.
//
// A batch-1 decode step of this model moves 351 MB (54 us at the measured HBM rate) but has
// ~100 dependent stages.  As separate kernels each stage pays a launch, a cold activation read
// and a cold weight read in sequence (7-15 us per kernel, measured with ncu).  Here one CTA per
// SM runs every stage; its weight slices for the coming stages are streamed into a shared-memory
// ring by TMA bulk copies (cp.async.bulk + mbarrier) that run ahead of the grid barriers, so
// after a barrier a stage only pays for reading the activations (L2) and computing.
//
// Stages per layer (a grid barrier after each):
//   S1  RMSNorm(x) -> q|k|v rows (RoPE pairs) + bias + RoPE; q to global, k/v into the f16 cache
//   S23 attention for every head, recomputed by every CTA (short contexts: the scores of all
//       positions must fit the activation area, see mega_geometry) -> this CTA's o-projection
//       rows + residual into x
//   S4  RMSNorm(x) -> gate|up rows -> SiLU(gate)*up into `gated`
//   S5  down-projection rows + residual into x
// then the final RMSNorm and this CTA's slice of the tied head rows, streamed in chunks.
//
// Grid barriers are a monotonic 64-bit arrival counter (zeroed by a memset node before each
// launch); every wait is bounded and reports through `err` instead of hanging.  Activations
// written by other CTAs are read with ld.global.cg (L2), never through L1.

#include "k_decode.cuh"
#include "k_mega.cuh"

namespace enx {

constexpr int kMThreads = 512;
constexpr int kMWarps = kMThreads / 32;
constexpr uint32_t kSpinLimit = 1u << 24;  // bounded waits (well under a minute), then an error
constexpr uint32_t kMaxGroup = 8;          // query heads per kv head handled by the scorer
constexpr uint32_t kKvStage = 64;          // cached positions staged in shared memory at a time

// Stage trace: thread 0 of CTA 0 stamps %globaltimer at the start of a stage (after its barrier),
// when its weights have landed, and when its compute is done: trace[3*stage + {0,1,2}].
__device__ __forceinline__ void stamp(const MegaArgs& A, uint32_t idx) {
    if (A.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        A.trace[idx] = t;
    }
}

// ---------------------------------------------------------------------------------------------
// PTX helpers: mbarrier + bulk copy

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Plain (non-multicast) bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_copy(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// ---------------------------------------------------------------------------------------------
// per-CTA work plan (a pure function of the slice id and blockIdx, so producer and consumer agree)

// A row range [r0, r1) of one quantised tensor staged in shared memory.  The three source byte
// ranges are widened to 16-byte boundaries (bulk-copy alignment); the compute indexes from the
// widened starts.
struct SRange {
    const QW* w;
    uint32_t r0, r1;
    uint32_t off_p, off_s, off_z;     // byte offsets of packed / scales / zeros inside the slot
    uint32_t s_base;                  // global scale index at the start of the staged scales
    uint32_t z_base;                  // global zero-word index at the start of the staged zeros
    uint32_t gp, np, gs, ns, gz, nz;  // source byte offsets and sizes of the three copies
};

__device__ __forceinline__ uint32_t align_down16(uint32_t v) { return v & ~15u; }
__device__ __forceinline__ uint32_t align_up16(uint32_t v) { return (v + 15u) & ~15u; }

__device__ __forceinline__ uint32_t plan_range(SRange& R, const QW* w, int bits, uint32_t r0, uint32_t r1,
                                               uint32_t cursor) {
    R.w = w;
    R.r0 = r0;
    R.r1 = r1;
    const uint32_t row_bytes = w->cols * bits / 8;
    const uint32_t bpr = w->cols / kBlock;
    R.gp = r0 * row_bytes;
    R.np = (r1 - r0) * row_bytes;  // multiple of 16 since cols % 64 == 0
    const uint32_t sb = align_down16(r0 * bpr * 4), se = align_up16(r1 * bpr * 4);
    R.gs = sb;
    R.ns = se - sb;
    R.s_base = sb / 4;
    const uint32_t zpw = 32 / bits;  // zero-points per word
    const uint32_t zb = align_down16((r0 * bpr / zpw) * 4), ze = align_up16(((r1 * bpr + zpw - 1) / zpw) * 4);
    R.gz = zb;
    R.nz = ze - zb;
    R.z_base = zb / 4;
    R.off_p = cursor;
    cursor += R.np;
    R.off_s = cursor;
    cursor += R.ns;
    R.off_z = cursor;
    cursor += R.nz;
    return align_up16(cursor);
}

struct Plan {
    SRange r[4];
    int n;
};

// Start of part i when `total` items (in granules) are split into `parts` contiguous ranges.
__device__ __forceinline__ uint32_t split_lo(uint32_t total, uint32_t parts, uint32_t i, uint32_t granule) {
    uint32_t units = total / granule;
    return (uint32_t)(((uint64_t)units * i) / parts) * granule;
}

// Slice ids: layer l stage s (0..3) -> 4*l + s; head chunk j -> 4*layers + j.
__device__ void plan_slice(const MegaArgs& A, uint32_t slice, Plan& P) {
    const uint32_t G = gridDim.x, c = blockIdx.x;
    P.n = 0;
    uint32_t cur = 0;
    if (slice < 4 * A.layers) {
        const LayerArgs& La = A.layer[slice / 4];
        const uint32_t s = slice % 4;
        if (s == 0) {
            // units of 4 RoPE pairs of one head slot of the concatenated q|k|v row space
            const uint32_t half = A.head_dim / 2, per_slot = half / 4;
            const uint32_t units = (A.heads + 2 * A.kv_heads) * per_slot;
            for (uint32_t u = c; u < units && P.n + 2 <= 4; u += G) {
                const uint32_t hs = u / per_slot, i0 = (u % per_slot) * 4;
                const QW* w;
                uint32_t head;
                if (hs < A.heads) { w = &La.wq; head = hs; }
                else if (hs < A.heads + A.kv_heads) { w = &La.wk; head = hs - A.heads; }
                else { w = &La.wv; head = hs - A.heads - A.kv_heads; }
                const uint32_t b = head * A.head_dim + i0;
                cur = plan_range(P.r[P.n++], w, 4, b, b + 4, cur);
                cur = plan_range(P.r[P.n++], w, 4, b + half, b + half + 4, cur);
            }
        } else if (s == 1) {
            const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
            if (r1 > r0) cur = plan_range(P.r[P.n++], &La.wo, 4, r0, r1, cur);
        } else if (s == 2) {
            const uint32_t r0 = split_lo(A.intermediate, G, c, 1), r1 = split_lo(A.intermediate, G, c + 1, 1);
            if (r1 > r0) {
                cur = plan_range(P.r[P.n++], &La.wg, 4, r0, r1, cur);
                cur = plan_range(P.r[P.n++], &La.wu, 4, r0, r1, cur);
            }
        } else {
            const uint32_t r0 = split_lo(A.hidden, G, c, 2), r1 = split_lo(A.hidden, G, c + 1, 2);
            if (r1 > r0) cur = plan_range(P.r[P.n++], &La.wd, 4, r0, r1, cur);
        }
    } else {
        const uint32_t j = slice - 4 * A.layers;
        const uint32_t h0 = split_lo(A.vocab, G, c, 1), h1 = split_lo(A.vocab, G, c + 1, 1);
        const uint32_t r0 = h0 + j * A.head_chunk, r1 = min(r0 + A.head_chunk, h1);
        if (r1 > r0) cur = plan_range(P.r[P.n++], &A.head, A.head_bits, r0, r1, cur);
    }
}

__device__ __forceinline__ uint32_t num_slices(const MegaArgs& A) {
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t h0 = split_lo(A.vocab, G, c, 1), h1 = split_lo(A.vocab, G, c + 1, 1);
    return 4 * A.layers + (h1 - h0 + A.head_chunk - 1) / A.head_chunk;
}

struct Ring {
    uint8_t* slots;
    uint64_t* bars;
    uint32_t nslots, slot_bytes, total;
};

// Thread 0 only: issue the bulk copies of `slice` into its slot.
__device__ void issue_slice(const MegaArgs& A, const Ring& R, uint32_t slice) {
    if (slice >= R.total) return;
    Plan P;
    plan_slice(A, slice, P);
    const uint32_t slot = slice % R.nslots;
    uint8_t* base = R.slots + (size_t)slot * R.slot_bytes;
    uint64_t* bar = R.bars + slot;
    uint32_t bytes = 0;
    for (int i = 0; i < P.n; ++i) bytes += P.r[i].np + P.r[i].ns + P.r[i].nz;
    fence_proxy_async();         // earlier generic reads of this slot precede the async writes
    mbar_expect_tx(bar, bytes);  // the one arrival of this phase; 0 bytes completes it at once
    for (int i = 0; i < P.n; ++i) {
        const SRange& r = P.r[i];
        const uint8_t* p = reinterpret_cast<const uint8_t*>(r.w->packed);
        const uint8_t* s = reinterpret_cast<const uint8_t*>(r.w->scales);
        const uint8_t* z = reinterpret_cast<const uint8_t*>(r.w->zeros);
        if (r.np) bulk_copy(base + r.off_p, p + r.gp, r.np, bar);
        if (r.ns) bulk_copy(base + r.off_s, s + r.gs, r.ns, bar);
        if (r.nz) bulk_copy(base + r.off_z, z + r.gz, r.nz, bar);
    }
}

// All threads: wait for `slice` to land.  Bounded: on timeout the error is recorded, and the
// caller waits (bounded again) for the copies still in flight before leaving.
__device__ bool wait_slice(const MegaArgs& A, const Ring& R, uint32_t slice) {
    const uint32_t slot = slice % R.nslots, parity = (slice / R.nslots) & 1u;
    uint32_t it = 0;
    while (!mbar_try_wait(R.bars + slot, parity)) {
        if (++it > kSpinLimit) {
            if (threadIdx.x == 0) atomicMax(A.err, 2u);
            return false;
        }
    }
    return true;
}

// On an early exit: give every issued copy a bounded chance to land so no bulk copy is still
// writing into shared memory when the CTA retires.
__device__ void drain(const Ring& R, uint32_t next_issued) {
    for (uint32_t s = next_issued >= R.nslots ? next_issued - R.nslots : 0; s < next_issued && s < R.total; ++s) {
        const uint32_t slot = s % R.nslots, parity = (s / R.nslots) & 1u;
        for (uint32_t it = 0; it < kSpinLimit && !mbar_try_wait(R.bars + slot, parity); ++it) {
        }
    }
}

// ---------------------------------------------------------------------------------------------
// grid barrier (bounded)

__device__ bool grid_sync(const MegaArgs& A, uint32_t& index, int* s_fail) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long target = (unsigned long long)(index + 1) * gridDim.x;
        __threadfence();
        atomicAdd(A.bar, 1ull);
        uint32_t it = 0;
        for (;;) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(A.bar) : "memory");
            if (v >= target) break;
            if (++it > kSpinLimit) {
                atomicMax(A.err, 1u);
                *s_fail = 1;
                break;
            }
            if ((it & 255u) == 0 && *reinterpret_cast<volatile uint32_t*>(A.err)) {
                *s_fail = 1;
                break;
            }
        }
    }
    ++index;
    __syncthreads();
    return !*s_fail;
}

// ---------------------------------------------------------------------------------------------
// dot products over a staged row range (lane per 16-byte chunk, exact (q - z), f32 accumulate)

template <int BITS, int MT, int R>
__device__ __forceinline__ void dot_staged(const uint8_t* slot, const SRange& S, const uint32_t (&rows)[R],
                                           const double2* __restrict__ XD, uint32_t nchunk, int lane,
                                           double (&acc)[R][MT]) {
    constexpr int CPB = Geom<BITS>::CPB;
    const uint32_t bpr = S.w->cols / kBlock;
    const uint4* P = reinterpret_cast<const uint4*>(slot + S.off_p);
    const float* sc = reinterpret_cast<const float*>(slot + S.off_s);
    const uint32_t* zw = reinterpret_cast<const uint32_t*>(slot + S.off_z);
    for (uint32_t c = lane; c < nchunk; c += 32) {
        uint4 q[R];
        float s[R];
        uint32_t zc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            q[r] = P[(size_t)(rows[r] - S.r0) * nchunk + c];
            const uint32_t blk = rows[r] * bpr + c / CPB;
            s[r] = sc[blk - S.s_base];
            zc[r] = BITS == 4 ? (zw[(blk >> 3) - S.z_base] >> ((blk & 7u) * 4u)) & 0xFu
                              : (zw[(blk >> 2) - S.z_base] >> ((blk & 3u) * 8u)) & 0xFFu;
        }
        chunk_dot<BITS, MT, R>(q, s, zc, XD, nchunk, c, acc);
    }
}

template <int MT>
__device__ __forceinline__ double pick(const double (&a)[MT], int t) {
    double v = 0.0;
#pragma unroll
    for (int i = 0; i < MT; ++i)
        if (i == t) v = a[i];
    return v;
}

// ---------------------------------------------------------------------------------------------
// the kernel

template <int MT, int HB>
__global__ void __launch_bounds__(kMThreads, 1) k_mega(const __grid_constant__ MegaArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double rs[MT], red[MT * kMWarps];
    __shared__ int s_fail;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t H = A.hidden, I = A.intermediate, hd = A.head_dim, half = hd / 2;

    Ring R;
    R.bars = reinterpret_cast<uint64_t*>(smem);
    R.nslots = A.nslots;
    R.slot_bytes = A.slot_bytes;
    R.slots = smem + 128;
    R.total = num_slices(A);
    double2* XD = reinterpret_cast<double2*>(smem + 128 + (size_t)A.nslots * A.slot_bytes);
    double* Xd = reinterpret_cast<double*>(XD);   // [MT][x4] activations as doubles
    float* Xf = reinterpret_cast<float*>(XD);     // the same area, as float attention scratch
    float* qs = reinterpret_cast<float*>(Xd + (size_t)MT * A.x4_floats);  // [MT][H] queries / temporary
    uint16_t* kvs = reinterpret_cast<uint16_t*>(qs + (size_t)MT * H);  // [kKvStage][kv_heads*hd] f16

    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < R.nslots; ++i) mbar_init(R.bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // weights do not depend on earlier kernels: start streaming them at once
    if (tid == 0)
        for (uint32_t i = 0; i < R.nslots; ++i) issue_slice(A, R, i);

    uint32_t bar_index = 0, slice = 0;
    auto fail_out = [&]() { if (tid == 0) drain(R, slice + R.nslots); };
    auto next_slice = [&]() {
        __syncthreads();  // every thread is done with this slot
        if (tid == 0) issue_slice(A, R, slice + R.nslots);
        ++slice;
    };

    for (uint32_t l = 0; l < A.layers; ++l) {
        const LayerArgs& La = A.layer[l];
        Plan P;

        // ---------------- S1: RMSNorm + q|k|v + RoPE + cache ---------------------------------
        stamp(A, 3 * (4 * l + 0));
        if (l == 0) {
            // embedding rows of the tied table, for this CTA's norm; the rows this CTA owns in S23
            // and S5 also initialise the residual stream in global memory
            const uint32_t o0 = split_lo(H, G, c, 2), o1 = split_lo(H, G, c + 1, 2);
            const uint32_t bpr = H / kBlock;
            for (uint32_t i = tid; i < MT * H; i += blockDim.x) {
                const uint32_t t = i / H, k = i % H, row = A.tokens[t];
                const size_t flat = (size_t)row * H + k;
                const uint32_t q = HB == 4 ? (A.head.packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu
                                           : (A.head.packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
                const uint32_t blk = row * bpr + k / kBlock;
                const float v = ((float)q - (float)zero_code<HB>(A.head.zeros, blk)) * A.head.scales[blk];
                qs[i] = v;
                if (k >= o0 && k < o1) A.S.x[i] = v;
            }
            __syncthreads();
            rms_scale_d<MT, false>(rs, red, qs, H, A.eps);
            stage_x_d<4, MT, false>(Xd, qs, H, rs, La.norm_in);
        } else {
            rms_scale_d<MT, true>(rs, red, A.S.x, H, A.eps);
            stage_x_d<4, MT, true>(Xd, A.S.x, H, rs, La.norm_in);
        }
        plan_slice(A, slice, P);
        if (!wait_slice(A, R, slice)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 0) + 1);
        {
            const uint8_t* slot = R.slots + (size_t)(slice % R.nslots) * R.slot_bytes;
            const uint32_t nchunk = H / 32;
            // range 2u holds rows i0..i0+3 of a head, range 2u+1 their RoPE partners (+half)
            const int npairs = (P.n / 2) * 4;
            for (int pi = warp; pi < npairs; pi += kMWarps) {
                const SRange& Ra = P.r[(pi / 4) * 2];
                const SRange& Rb = P.r[(pi / 4) * 2 + 1];
                const uint32_t ra = Ra.r0 + pi % 4, rb = Rb.r0 + pi % 4;
                double aa[1][MT] = {}, ab[1][MT] = {};
                const uint32_t rowa[1] = {ra}, rowb[1] = {rb};
                dot_staged<4, MT, 1>(slot, Ra, rowa, XD, nchunk, lane, aa);
                dot_staged<4, MT, 1>(slot, Rb, rowb, XD, nchunk, lane, ab);
#pragma unroll
                for (int t = 0; t < MT; ++t) { aa[0][t] = warp_sum_d(aa[0][t]); ab[0][t] = warp_sum_d(ab[0][t]); }
                if (lane < MT) {
                    const int kind = Ra.w == &La.wq ? 0 : Ra.w == &La.wk ? 1 : 2;
                    const float* bias = kind == 0 ? La.bq : kind == 1 ? La.bk : La.bv;
                    float a = (float)(pick<MT>(aa[0], lane) + (double)bias[ra]);
                    float b = (float)(pick<MT>(ab[0], lane) + (double)bias[rb]);
                    const uint32_t head = ra / hd, i = ra % hd;
                    const uint32_t pos = A.S.pos_of(lane);
                    if (kind != 2)  // half-rotation RoPE (src/kernels/rope.wgsl:42-52)
                        rope_pair(a, b, A.S.rope_cos[(size_t)pos * half + i], A.S.rope_sin[(size_t)pos * half + i]);
                    if (kind == 0) {
                        A.S.q[(size_t)lane * H + ra] = a;
                        A.S.q[(size_t)lane * H + rb] = b;
                    } else {
                        uint16_t* cache = (kind == 1 ? A.S.kcache : A.S.vcache) +
                                          A.S.cache_offset(A.S.seq_of(lane), l, pos);
                        cache[head * hd + i] = __half_as_ushort(__float2half_rn(a));
                        cache[head * hd + i + half] = __half_as_ushort(__float2half_rn(b));
                    }
                }
            }
        }
        stamp(A, 3 * (4 * l + 0) + 2);
        next_slice();
        if (!grid_sync(A, bar_index, &s_fail)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 1));

        // ---------------- S23: attention (all heads) + o-projection + residual ---------------
        {
            const uint32_t group = A.heads / A.kv_heads, kvd = A.kv_heads * hd;
            for (uint32_t i = tid; i < MT * H; i += blockDim.x) qs[i] = ldcg(A.S.q + i);
            __syncthreads();
            float* sc = Xf;  // scores [heads][npos], aliasing the activation area
            float out_v[2 * MT];
#pragma unroll
            for (int i = 0; i < 2 * MT; ++i) out_v[i] = 0.f;
            for (int t = 0; t < MT; ++t) {
                const uint32_t npos = A.S.pos_of(t) + 1;
                const uint16_t* Kc = A.S.kcache + A.S.cache_offset(A.S.seq_of(t), l, 0);
                const uint16_t* Vc = A.S.vcache + A.S.cache_offset(A.S.seq_of(t), l, 0);
                const float* qt = qs + (size_t)t * H;
                // K and V pass through shared memory kKvStage positions at a time: all threads load
                // a chunk with independent 16-byte reads, then compute.  Arithmetic and rounding
                // follow test/reference/ops.ts:123-204 (double sums, float scores and weights).
                const uint32_t row16 = kvd / 8;  // uint4 per cached position
                const double scale = 1.0 / sqrt((double)hd);
                for (uint32_t j0 = 0; j0 < npos; j0 += kKvStage) {
                    const uint32_t n = min(kKvStage, npos - j0);
                    for (uint32_t i = tid; i < n * row16; i += blockDim.x)
                        reinterpret_cast<uint4*>(kvs)[i] = __ldcg(reinterpret_cast<const uint4*>(Kc + (size_t)j0 * kvd) + i);
                    __syncthreads();
                    for (uint32_t w = tid; w < n * A.heads; w += blockDim.x) {
                        const uint32_t j = w / A.heads, h = w % A.heads, g = h / group;
                        const uint16_t* kr = kvs + (size_t)j * kvd + g * hd;
                        const float* qh = qt + h * hd;
                        double acc = 0.0;
                        for (uint32_t d = 0; d < hd; ++d)
                            acc = fma((double)qh[d], (double)__half2float(__ushort_as_half(kr[d])), acc);
                        sc[h * npos + j0 + j] = (float)(acc * scale);
                    }
                    __syncthreads();
                }
                for (uint32_t h = warp; h < A.heads; h += kMWarps) {  // softmax, a warp per head
                    float m = -INFINITY;
                    for (uint32_t j = lane; j < npos; j += 32) m = fmaxf(m, sc[h * npos + j]);
                    m = warp_max(m);
                    double s = 0.0;
                    for (uint32_t j = lane; j < npos; j += 32) {
                        const double e = exp((double)sc[h * npos + j] - (double)m);
                        sc[h * npos + j] = (float)e;
                        s += e;
                    }
                    s = warp_sum_d(s);
                    for (uint32_t j = lane; j < npos; j += 32) sc[h * npos + j] = (float)((double)sc[h * npos + j] / s);
                }
                __syncthreads();
                double acc2[2] = {0.0, 0.0};
                for (uint32_t j0 = 0; j0 < npos; j0 += kKvStage) {
                    const uint32_t n = min(kKvStage, npos - j0);
                    for (uint32_t i = tid; i < n * row16; i += blockDim.x)
                        reinterpret_cast<uint4*>(kvs)[i] = __ldcg(reinterpret_cast<const uint4*>(Vc + (size_t)j0 * kvd) + i);
                    __syncthreads();
                    uint32_t k = 0;
                    for (uint32_t o = tid; o < H; o += blockDim.x, ++k) {  // V apply, a thread per output
                        const uint32_t h = o / hd, d = o % hd, g = h / group;
                        const float* wv = sc + h * npos + j0;
                        const uint16_t* vp = kvs + g * hd + d;
                        double a = acc2[k & 1];
                        for (uint32_t j = 0; j < n; ++j)
                            a = fma((double)wv[j], (double)__half2float(__ushort_as_half(vp[(size_t)j * kvd])), a);
                        acc2[k & 1] = a;
                    }
                    __syncthreads();
                }
                out_v[t * 2 + 0] = (float)acc2[0];
                out_v[t * 2 + 1] = (float)acc2[1];
            }
            for (int t = 0; t < MT; ++t) {
                uint32_t k = 0;
                for (uint32_t o = tid; o < H; o += blockDim.x, ++k)
                    Xd[xd_index<4>(t, o, H / 32)] = (double)out_v[t * 2 + k];
            }
            __syncthreads();
        }
        plan_slice(A, slice, P);
        if (!wait_slice(A, R, slice)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 1) + 1);
        if (P.n) {
            const uint8_t* slot = R.slots + (size_t)(slice % R.nslots) * R.slot_bytes;
            const SRange& S = P.r[0];
            for (uint32_t r = S.r0 + warp; r < S.r1; r += kMWarps) {
                double acc[1][MT] = {};
                const uint32_t rows[1] = {r};
                dot_staged<4, MT, 1>(slot, S, rows, XD, H / 32, lane, acc);
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[0][t] = warp_sum_d(acc[0][t]);
                if (lane < MT) {
                    float* xp = A.S.x + (size_t)lane * H + r;
                    *xp = ldcg(xp) + (float)pick<MT>(acc[0], lane);
                }
            }
        }
        stamp(A, 3 * (4 * l + 1) + 2);
        next_slice();
        if (!grid_sync(A, bar_index, &s_fail)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 2));

        // ---------------- S4: RMSNorm + gate|up + SiLU --------------------------------------
        rms_scale_d<MT, true>(rs, red, A.S.x, H, A.eps);
        stage_x_d<4, MT, true>(Xd, A.S.x, H, rs, La.norm_post);
        plan_slice(A, slice, P);
        if (!wait_slice(A, R, slice)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 2) + 1);
        if (P.n) {
            const uint8_t* slot = R.slots + (size_t)(slice % R.nslots) * R.slot_bytes;
            const SRange& Sg = P.r[0];
            const SRange& Su = P.r[1];
            for (uint32_t r = Sg.r0 + warp; r < Sg.r1; r += kMWarps) {
                double ag[1][MT] = {}, au[1][MT] = {};
                const uint32_t rows[1] = {r};
                dot_staged<4, MT, 1>(slot, Sg, rows, XD, H / 32, lane, ag);
                dot_staged<4, MT, 1>(slot, Su, rows, XD, H / 32, lane, au);
#pragma unroll
                for (int t = 0; t < MT; ++t) { ag[0][t] = warp_sum_d(ag[0][t]); au[0][t] = warp_sum_d(au[0][t]); }
                if (lane < MT)
                    A.S.gated[(size_t)lane * I + r] =
                        silu_mul_value((float)pick<MT>(ag[0], lane), (float)pick<MT>(au[0], lane));
            }
        }
        stamp(A, 3 * (4 * l + 2) + 2);
        next_slice();
        if (!grid_sync(A, bar_index, &s_fail)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 3));

        // ---------------- S5: down + residual -----------------------------------------------
        stage_x_d<4, MT, true>(Xd, A.S.gated, I, nullptr, nullptr);
        plan_slice(A, slice, P);
        if (!wait_slice(A, R, slice)) { fail_out(); return; }
        stamp(A, 3 * (4 * l + 3) + 1);
        if (P.n) {
            const uint8_t* slot = R.slots + (size_t)(slice % R.nslots) * R.slot_bytes;
            const SRange& S = P.r[0];
            for (uint32_t r = S.r0 + warp; r < S.r1; r += kMWarps) {
                double acc[1][MT] = {};
                const uint32_t rows[1] = {r};
                dot_staged<4, MT, 1>(slot, S, rows, XD, I / 32, lane, acc);
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[0][t] = warp_sum_d(acc[0][t]);
                if (lane < MT) {
                    float* xp = A.S.x + (size_t)lane * H + r;
                    *xp = ldcg(xp) + (float)pick<MT>(acc[0], lane);
                }
            }
        }
        stamp(A, 3 * (4 * l + 3) + 2);
        next_slice();
        if (!grid_sync(A, bar_index, &s_fail)) { fail_out(); return; }
    }

    // ---------------- final RMSNorm + tied head ---------------------------------------------
    stamp(A, 3 * (4 * A.layers));
    rms_scale_d<MT, true>(rs, red, A.S.x, H, A.eps);
    stage_x_d<HB, MT, true>(Xd, A.S.x, H, rs, A.final_norm);
    if (c == 0)
        for (uint32_t i = tid; i < MT * H; i += blockDim.x)
            A.S.normed[i] = norm_value(ldcg(A.S.x + i), rs[i / H], A.final_norm[i % H]);
    const uint32_t nchunk = H / Geom<HB>::E;
    while (slice < R.total) {
        Plan P;
        plan_slice(A, slice, P);
        if (!wait_slice(A, R, slice)) { fail_out(); return; }
        if (P.n) {
            const uint8_t* slot = R.slots + (size_t)(slice % R.nslots) * R.slot_bytes;
            const SRange& S = P.r[0];
            for (uint32_t r0 = S.r0 + 2 * warp; r0 < S.r1; r0 += 2 * kMWarps) {
                const uint32_t rows[2] = {r0, min(r0 + 1, S.r1 - 1)};
                double acc[2][MT] = {};
                dot_staged<HB, MT, 2>(slot, S, rows, XD, nchunk, lane, acc);
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_d(acc[r][t]);
                if (lane < MT) {
                    A.S.logits[(size_t)lane * A.vocab + r0] = (float)pick<MT>(acc[0], lane);
                    if (r0 + 1 < S.r1) A.S.logits[(size_t)lane * A.vocab + r0 + 1] = (float)pick<MT>(acc[1], lane);
                }
            }
        }
        next_slice();
    }
    stamp(A, 3 * (4 * A.layers) + 2);
}

// ---------------------------------------------------------------------------------------------
// host side

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
    auto range_bytes = [](uint32_t rows, uint32_t cols, uint32_t bits) {
        const uint32_t bpr = cols / 64;
        return rows * cols * bits / 8 + rows * bpr * 4 + 32 + rows * bpr * bits / 8 + 32 + 16;
    };
    const uint32_t rows4 = (A.intermediate + g.grid - 1) / g.grid + 1;
    const uint32_t rows5 = ((A.hidden / 2 + g.grid - 1) / g.grid) * 2 + 2;
    uint32_t slot = 2 * range_bytes(rows4, A.hidden, 4);
    const uint32_t s5 = range_bytes(rows5, A.intermediate, 4);
    const uint32_t s1 = 4 * range_bytes(4, A.hidden, 4);
    const uint32_t hc = range_bytes(A.head_chunk, A.hidden, (uint32_t)A.head_bits);
    if (s5 > slot) slot = s5;
    if (s1 > slot) slot = s1;
    if (hc > slot) slot = hc;
    slot = (slot + 127) & ~127u;
    g.slot_bytes = slot;
    const size_t fixed = 128 + (size_t)mt * x4 * 8 + (size_t)mt * A.hidden * 4 +
                         (size_t)kKvStage * A.kv_heads * A.head_dim * 2;
    const int64_t room = (int64_t)maxsm - (int64_t)fixed - 2048;  // static shared memory and slack
    int ns = room > 0 ? (int)(room / slot) : 0;
    if (ns > 8) ns = 8;
    g.nslots = (uint32_t)ns;
    g.smem = fixed + (size_t)g.nslots * slot;
    g.max_positions = (uint32_t)(((size_t)mt * x4 * 2) / A.heads);  // float scores share the double area
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
