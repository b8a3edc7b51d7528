// CPU oracle for the enargeia decode hot path.  TEST INFRASTRUCTURE ONLY.
//
// This file is a plain restatement of the reference's CPU path and WGSL semantics.  It is the
// checker that the CUDA library is compared against: only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline leg may load it.  Nothing in the product links it.
//
// What it restates, and from where (paths inside the reference project):
//   * int4/int8 block dequantisation      test/reference/quant.ts:77-84,
//                                         src/kernels/embedding_variants.ts:56-63
//   * linear / linearQ4                   test/reference/ops.ts:59-78, test/reference/quant.ts:95-112
//   * rmsNorm                             test/reference/ops.ts:30-51
//   * rope (half rotation)                test/reference/ops.ts:87-114
//   * attentionScores/softmaxRows/apply   test/reference/ops.ts:123-204
//   * silu / siluMul / add / embed        test/reference/ops.ts:207-235
//   * argmax (lowest index wins ties)     test/reference/ops.ts:238-244
//   * layer order                         tools/check_cpu_reference.ts:122-192
//   * f16 KV cache (post-RoPE K, and V)   src/kernels/cache_variants.ts:269-301,
//                                         src/runtime/kvcache.ts:9-21
//   * incremental decode and prefill      src/model/graph_decode.ts:268-386, src/model/graph.ts:386-460
//   * sampler                             src/kernels/sample.wgsl:91-331
//   * mulberry32                          src/runtime/session.ts:75-83, test/reference/rng.ts:2-10
//
// Arithmetic follows the TypeScript reference: every reduction accumulates in double and every
// stage stores float.  The reference has no CPU sampler; its WGSL one sums in f32 in an order
// the browser picks.  The oracle pins the sampler to exact arithmetic, approximated in double:
// the per-token probabilities, the bisection masses, the kept mass and the running draw total
// are doubles, while the penalty, the temperature division and the bisection midpoints stay in
// float exactly as the shader computes them.  The CUDA sampler follows the same rule.
//
// Parallelism: OpenMP over independent outputs only, so results are bit-identical at any
// thread count.

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// ---------------------------------------------------------------------------------------------
// helpers

static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int e = -1;
            do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// float -> half, round to nearest even, with subnormals, overflow to inf and NaN kept quiet.
static inline uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) {  // inf or nan
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477FF000u) {  // rounds to >= 65520 -> inf
        return (uint16_t)(sign | 0x7C00u);
    }
    if (absx < 0x38800000u) {  // below the smallest normal half (2^-14): subnormal or zero
        if (absx < 0x33000000u) return (uint16_t)sign;  // < 2^-25 rounds to zero
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
        // value = m * 2^(e-150); half subnormal unit is 2^-24 -> shift by (126 - e)
        uint32_t shift = 126u - e;
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 127 + 15;
    uint32_t m = absx & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

static inline float round_f16(float v) { return f16_to_f32(f32_to_f16(v)); }

void orc_f32_to_f16(const float* in, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16(in[i]);
}

void orc_f16_to_f32(const uint16_t* in, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(in[i]);
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// mulberry32 (src/runtime/session.ts:75-83).  `state` is advanced in place.
double orc_mulberry32_next(uint32_t* state) {
    uint32_t s = *state + 0x6D2B79F5u;
    *state = s;
    uint32_t t = (s ^ (s >> 15)) * (1u | s);
    t = (t + ((t ^ (t >> 7)) * (61u | t))) ^ t;
    return (double)(t ^ (t >> 14)) / 4294967296.0;
}

void orc_mulberry32_fill(uint32_t seed, int64_t n, double* out) {
    uint32_t s = seed;
    for (int64_t i = 0; i < n; ++i) out[i] = orc_mulberry32_next(&s);
}

// ---------------------------------------------------------------------------------------------
// quantised weights.  Element (row, col) of an R x C tensor: flat = row*C + col,
// block = row*(C/64) + col/64 (test/reference/quant.ts:77-84).

static inline double dq4(const uint32_t* packed, const float* scales, const uint32_t* zeros,
                         int64_t cols, int64_t block_size, int64_t row, int64_t col) {
    int64_t flat = row * cols + col;
    uint32_t nib = (packed[flat >> 3] >> ((flat & 7) * 4)) & 0xFu;
    int64_t block = row * (cols / block_size) + col / block_size;
    uint32_t zero = (zeros[block >> 3] >> ((block & 7) * 4)) & 0xFu;
    return ((double)nib - (double)zero) * (double)scales[block];
}

static inline double dq8(const uint32_t* packed, const float* scales, const uint32_t* zeros,
                         int64_t cols, int64_t block_size, int64_t row, int64_t col) {
    int64_t flat = row * cols + col;
    uint32_t q = (packed[flat >> 2] >> ((flat & 3) * 8)) & 0xFFu;
    int64_t block = row * (cols / block_size) + col / block_size;
    uint32_t zero = (zeros[block >> 2] >> ((block & 3) * 8)) & 0xFFu;
    return ((double)q - (double)zero) * (double)scales[block];
}

void orc_dequant(int bits, const uint32_t* packed, const float* scales, const uint32_t* zeros,
                 int64_t rows, int64_t cols, int64_t block_size, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            out[r * cols + c] = (float)(bits == 4 ? dq4(packed, scales, zeros, cols, block_size, r, c)
                                                  : dq8(packed, scales, zeros, cols, block_size, r, c));
}

// out[row*out_stride + out_offset + col] = sum_i x[row*k+i] * W[col, i] + bias[col]
// (test/reference/quant.ts:95-112 with the matmulQ4Dims outStride/outOffset of
// src/kernels/matmul_q4.ts:50-64).  bits 4 or 8 (the tied head, embedding_variants.ts:135-180).
void orc_linear_q(int bits, const float* x, const uint32_t* packed, const float* scales,
                  const uint32_t* zeros, const float* bias, int64_t m, int64_t k, int64_t n,
                  int64_t block_size, int64_t out_stride, int64_t out_offset, float* out) {
#pragma omp parallel
    {
        std::vector<double> wrow(k);
#pragma omp for schedule(static)
        for (int64_t col = 0; col < n; ++col) {
            // The dequantised row is the same double for every input row, so it is built once.
            for (int64_t i = 0; i < k; ++i)
                wrow[i] = bits == 4 ? dq4(packed, scales, zeros, k, block_size, col, i)
                                    : dq8(packed, scales, zeros, k, block_size, col, i);
            for (int64_t row = 0; row < m; ++row) {
                double acc = bias ? (double)bias[col] : 0.0;
                const float* xr = x + row * k;
                for (int64_t i = 0; i < k; ++i) acc += (double)xr[i] * wrow[i];
                out[row * out_stride + out_offset + col] = (float)acc;
            }
        }
    }
}

// Plain fp32 linear (test/reference/ops.ts:59-78).
void orc_linear_f32(const float* x, const float* w, const float* bias, int64_t m, int64_t k,
                    int64_t n, float* out) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t row = 0; row < m; ++row)
        for (int64_t col = 0; col < n; ++col) {
            double acc = bias ? (double)bias[col] : 0.0;
            for (int64_t i = 0; i < k; ++i) acc += (double)x[row * k + i] * (double)w[col * k + i];
            out[row * n + col] = (float)acc;
        }
}

// ---------------------------------------------------------------------------------------------
// small ops

void orc_rmsnorm(const float* x, const float* w, int64_t seq, int64_t features, float eps,
                 float* out) {
    for (int64_t s = 0; s < seq; ++s) {
        double sum = 0.0;
        for (int64_t f = 0; f < features; ++f) {
            double v = x[s * features + f];
            sum += v * v;
        }
        double scale = 1.0 / std::sqrt(sum / (double)features + (double)eps);
        for (int64_t f = 0; f < features; ++f)
            out[s * features + f] = (float)((double)x[s * features + f] * scale * (double)w[f]);
    }
}

// Half-rotation RoPE, element i pairs with i + headDim/2, positions offset by pos_offset.
void orc_rope(const float* x, int64_t seq, int64_t heads, int64_t head_dim, double theta,
              int64_t pos_offset, float* out) {
    int64_t half = head_dim / 2;
    for (int64_t i = 0; i < seq * heads * head_dim; ++i) out[i] = x[i];
    for (int64_t s = 0; s < seq; ++s) {
        double position = (double)(s + pos_offset);
        for (int64_t h = 0; h < heads; ++h) {
            int64_t base = (s * heads + h) * head_dim;
            for (int64_t i = 0; i < half; ++i) {
                double freq = 1.0 / std::pow(theta, (2.0 * (double)i) / (double)head_dim);
                double angle = position * freq;
                double c = std::cos(angle), sn = std::sin(angle);
                double a = x[base + i], b = x[base + i + half];
                out[base + i] = (float)(a * c - b * sn);
                out[base + i + half] = (float)(b * c + a * sn);
            }
        }
    }
}

// cos/sin table, f64-computed, f32-stored: [position][half] each.  The CUDA library builds the
// identical table on the host so rotation matches the oracle to one rounding.
void orc_rope_table(int64_t max_pos, int64_t head_dim, double theta, float* cos_out,
                    float* sin_out) {
    int64_t half = head_dim / 2;
    for (int64_t p = 0; p < max_pos; ++p)
        for (int64_t i = 0; i < half; ++i) {
            double freq = 1.0 / std::pow(theta, (2.0 * (double)i) / (double)head_dim);
            double angle = (double)p * freq;
            cos_out[p * half + i] = (float)std::cos(angle);
            sin_out[p * half + i] = (float)std::sin(angle);
        }
}

static inline float silu_mul1(float g, float u) {
    double gd = g;
    return (float)((gd / (1.0 + std::exp(-gd))) * (double)u);
}

void orc_silu_mul(const float* gate, const float* up, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = silu_mul1(gate[i], up[i]);
}

void orc_add(const float* a, const float* b, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)a[i] + (double)b[i]);
}

// Embedding gather through the int8 (or int4) table: out[s,:] = dequant(table[ids[s], :]).
void orc_embed_q(int bits, const uint32_t* ids, int64_t seq, const uint32_t* packed,
                 const float* scales, const uint32_t* zeros, int64_t hidden, int64_t block_size,
                 float* out) {
    for (int64_t s = 0; s < seq; ++s)
        for (int64_t c = 0; c < hidden; ++c)
            out[s * hidden + c] =
                (float)(bits == 4 ? dq4(packed, scales, zeros, hidden, block_size, ids[s], c)
                                  : dq8(packed, scales, zeros, hidden, block_size, ids[s], c));
}

uint32_t orc_argmax(const float* x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return (uint32_t)best;
}

// ---------------------------------------------------------------------------------------------
// attention over an f16 cache laid out [position][kvHeads][headDim] (cache stride = kvHeads*hd).
//
// Queries q[i][heads][hd] at absolute positions begin+i attend keys 0..begin+i.  Scores are
// f64-accumulated dot products times 1/sqrt(hd), stored float; softmax is f64 over the stored
// scores; the weighted V sum is f64 of float weights.  Decode is the queries=1 case.

void orc_attention_f16(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                       int64_t queries, int64_t begin, int64_t heads, int64_t kv_heads,
                       int64_t head_dim, float* out) {
    int64_t group = heads / kv_heads;
    int64_t stride = kv_heads * head_dim;
    double scale = 1.0 / std::sqrt((double)head_dim);
#pragma omp parallel for schedule(dynamic) collapse(2)
    for (int64_t i = 0; i < queries; ++i) {
        for (int64_t h = 0; h < heads; ++h) {
            int64_t keys = begin + i + 1;
            int64_t kvh = h / group;
            std::vector<float> sc(keys), w(keys);
            const float* qh = q + (i * heads + h) * head_dim;
            for (int64_t j = 0; j < keys; ++j) {
                double acc = 0.0;
                const uint16_t* kr = kcache + j * stride + kvh * head_dim;
                for (int64_t d = 0; d < head_dim; ++d) acc += (double)qh[d] * (double)f16_to_f32(kr[d]);
                sc[j] = (float)(acc * scale);
            }
            float mx = -INFINITY;
            for (int64_t j = 0; j < keys; ++j) mx = std::max(mx, sc[j]);
            double sum = 0.0;
            std::vector<double> e(keys);
            for (int64_t j = 0; j < keys; ++j) {
                e[j] = std::exp((double)sc[j] - (double)mx);
                w[j] = (float)e[j];
                sum += e[j];
            }
            for (int64_t j = 0; j < keys; ++j) w[j] = (float)((double)w[j] / sum);
            float* oh = out + (i * heads + h) * head_dim;
            for (int64_t d = 0; d < head_dim; ++d) {
                double acc = 0.0;
                for (int64_t j = 0; j < keys; ++j)
                    acc += (double)w[j] * (double)f16_to_f32(vcache[j * stride + kvh * head_dim + d]);
                oh[d] = (float)acc;
            }
        }
    }
}

// Write `count` positions of f32 rows [count][stride] into the f16 cache at position `begin`.
void orc_cache_pack(const float* src, int64_t count, int64_t stride, int64_t begin,
                    uint16_t* cache) {
    for (int64_t i = 0; i < count * stride; ++i) cache[begin * stride + i] = f32_to_f16(src[i]);
}

// ---------------------------------------------------------------------------------------------
// sampler (src/kernels/sample.wgsl:91-331), exact-arithmetic form described at the top.

typedef struct {
    uint32_t vocab;
    uint32_t history_length;
    float temperature;
    float top_p;
    float repetition_penalty;
    float random;
    uint32_t pad0, pad1;
} orc_sample_dims;

typedef struct {
    double top1_gap;          // greedy: best minus runner-up logit (ties -> 0)
    double max_prob;
    double sum;               // sum of exp(s - max)
    double min_mass_margin;   // min over bisection steps of |mass - topP|
    double threshold;         // bisection result (0 when topP >= 1)
    double kept;
    double target;
    double cross_margin;      // running - target at the crossing token (>= 0)
    double prev_margin;       // target - running just before the crossing token (> 0)
    uint32_t kept_count;
    uint32_t fallback;        // 1 when no crossing was found and the argmax was returned
} orc_sample_trace;

static void apply_penalty(float* logits, const uint32_t* history, uint32_t hlen, uint32_t vocab,
                          float rp) {
    if (rp == 1.0f) return;
    std::vector<uint8_t> seen(vocab, 0);
    for (uint32_t h = 0; h < hlen; ++h) {
        uint32_t id = history[h];
        if (id >= vocab || seen[id]) continue;  // first occurrence only; out-of-range ignored
        seen[id] = 1;
        float v = logits[id];
        logits[id] = v > 0.0f ? v / rp : v * rp;
    }
}

uint32_t orc_sample(float* logits, const uint32_t* history, const orc_sample_dims* dims,
                    orc_sample_trace* trace) {
    const uint32_t V = dims->vocab;
    orc_sample_trace tr;
    std::memset(&tr, 0, sizeof(tr));
    apply_penalty(logits, history, dims->history_length, V, dims->repetition_penalty);

    if (dims->temperature <= 0.0f) {
        float best = -1.0e30f, second = -1.0e30f;
        uint32_t idx = 0;
        for (uint32_t i = 0; i < V; ++i) {
            float v = logits[i];
            if (v > best) { second = best; best = v; idx = i; }
            else if (v > second) second = v;
        }
        tr.top1_gap = (double)best - (double)second;
        if (trace) *trace = tr;
        return idx;
    }

    const float T = dims->temperature;
    std::vector<float> s(V);
    float m = -1.0e30f;
    uint32_t arg = 0;
    for (uint32_t i = 0; i < V; ++i) {
        s[i] = logits[i] / T;
        if (s[i] > m) { m = s[i]; arg = i; }
    }
    std::vector<double> p(V);
    double sum = 0.0;
    for (uint32_t i = 0; i < V; ++i) {
        p[i] = std::exp((double)s[i] - (double)m);
        sum += p[i];
    }
    double maxp = 0.0;
    for (uint32_t i = 0; i < V; ++i) {
        p[i] = p[i] / sum;
        maxp = std::max(maxp, p[i]);
    }
    tr.sum = sum;
    tr.max_prob = maxp;

    float lo = 0.0f, hi = 1.0f;
    double margin = INFINITY;
    if (dims->top_p < 1.0f) {
        for (int step = 0; step < 32; ++step) {
            float mid = (lo + hi) * 0.5f;
            double mass = 0.0;
            for (uint32_t i = 0; i < V; ++i)
                if (p[i] >= (double)mid) mass += p[i];
            margin = std::min(margin, std::fabs(mass - (double)dims->top_p));
            if (mass < (double)dims->top_p) hi = mid; else lo = mid;
        }
    }
    double thr = dims->top_p < 1.0f ? (double)lo : 0.0;
    tr.threshold = thr;
    tr.min_mass_margin = margin;

    double kept = 0.0;
    uint32_t kc = 0;
    for (uint32_t i = 0; i < V; ++i)
        if (p[i] >= thr) { kept += p[i]; ++kc; }
    double target = (double)dims->random * std::max(kept, 1.0e-20);
    tr.kept = kept;
    tr.kept_count = kc;
    tr.target = target;

    double running = 0.0;
    uint32_t picked = 0xFFFFFFFFu;
    for (uint32_t i = 0; i < V; ++i) {
        if (p[i] >= thr) {
            double before = running;
            running += p[i];
            if (running >= target) {
                picked = i;
                tr.cross_margin = running - target;
                tr.prev_margin = target - before;
                break;
            }
        }
    }
    if (picked == 0xFFFFFFFFu) { picked = arg; tr.fallback = 1; }
    if (trace) *trace = tr;
    return picked;
}

// ---------------------------------------------------------------------------------------------
// whole model (Qwen2 decoder with a tied int8/int4 head), prefill in chunks + incremental decode

typedef struct {
    uint32_t layers, hidden, heads, kv_heads, head_dim, intermediate, vocab;
    float rms_norm_eps;
    float rope_theta;
} orc_config;

typedef struct {
    const uint32_t* packed;
    const float* scales;
    const uint32_t* zeros;
    int32_t bits;
    int32_t rows, cols;
} orc_qtensor;

typedef struct {
    const float* input_norm;
    const float* post_norm;
    orc_qtensor q, k, v, o, gate, up, down;
    const float* q_bias;
    const float* k_bias;
    const float* v_bias;
} orc_layer;

typedef struct {
    orc_qtensor embed;     // tied embedding / LM head
    const float* final_norm;
    const orc_layer* layers;  // array of cfg.layers
} orc_weights;

struct orc_model {
    orc_config cfg;
    orc_weights w;
    std::vector<orc_layer> layers;
    int64_t max_context;
    int64_t filled;
    std::vector<uint16_t> kcache, vcache;  // [layers][max_context][kv*hd]
};

orc_model* orc_model_create(const orc_config* cfg, const orc_weights* w, int64_t max_context) {
    orc_model* m = new orc_model();
    m->cfg = *cfg;
    m->w = *w;
    m->layers.assign(w->layers, w->layers + cfg->layers);
    m->w.layers = m->layers.data();
    m->max_context = max_context;
    m->filled = 0;
    int64_t per = max_context * (int64_t)cfg->kv_heads * cfg->head_dim;
    m->kcache.assign((size_t)per * cfg->layers, 0);
    m->vcache.assign((size_t)per * cfg->layers, 0);
    return m;
}

void orc_model_destroy(orc_model* m) { delete m; }
// A copy of `src` with the same weights and the same cache contents and fill: one shared prompt
// prefilled once, then continued as several independent sequences (test speed only).
orc_model* orc_model_fork(const orc_model* src) {
    orc_model* m = new orc_model(*src);
    m->w.layers = m->layers.data();
    return m;
}
void orc_model_reset(orc_model* m) { m->filled = 0; }
int64_t orc_model_filled(const orc_model* m) { return m->filled; }

static void lin(const orc_qtensor& t, const float* x, const float* bias, int64_t m, float* out) {
    orc_linear_q(t.bits, x, t.packed, t.scales, t.zeros, bias, m, t.cols, t.rows, 64, t.rows, 0, out);
}

// Runs `count` tokens at positions filled..filled+count-1 through the decoder, appends their K/V,
// and writes the final-norm hidden state of the LAST token to `last_normed` (hidden floats).
static int forward_chunk(orc_model* M, const uint32_t* ids, int64_t count, float* last_normed) {
    const orc_config& C = M->cfg;
    const int64_t H = C.hidden, kv = (int64_t)C.kv_heads * C.head_dim, I = C.intermediate;
    const int64_t begin = M->filled;
    if (begin + count > M->max_context) return -1;
    std::vector<float> hidden(count * H), normed(count * H), q(count * H), k(count * kv),
        v(count * kv), qr(count * H), kr(count * kv), att(count * H), proj(count * H),
        gate(count * I), up(count * I), gated(count * I), down(count * H);
    orc_embed_q(M->w.embed.bits, ids, count, M->w.embed.packed, M->w.embed.scales,
                M->w.embed.zeros, H, 64, hidden.data());
    const int64_t per_layer = M->max_context * kv;
    for (uint32_t l = 0; l < C.layers; ++l) {
        const orc_layer& L = M->layers[l];
        uint16_t* kc = M->kcache.data() + l * per_layer;
        uint16_t* vc = M->vcache.data() + l * per_layer;
        orc_rmsnorm(hidden.data(), L.input_norm, count, H, C.rms_norm_eps, normed.data());
        lin(L.q, normed.data(), L.q_bias, count, q.data());
        lin(L.k, normed.data(), L.k_bias, count, k.data());
        lin(L.v, normed.data(), L.v_bias, count, v.data());
        orc_rope(q.data(), count, C.heads, C.head_dim, C.rope_theta, begin, qr.data());
        orc_rope(k.data(), count, C.kv_heads, C.head_dim, C.rope_theta, begin, kr.data());
        orc_cache_pack(kr.data(), count, kv, begin, kc);
        orc_cache_pack(v.data(), count, kv, begin, vc);
        orc_attention_f16(qr.data(), kc, vc, count, begin, C.heads, C.kv_heads, C.head_dim, att.data());
        lin(L.o, att.data(), nullptr, count, proj.data());
        orc_add(hidden.data(), proj.data(), count * H, hidden.data());
        orc_rmsnorm(hidden.data(), L.post_norm, count, H, C.rms_norm_eps, normed.data());
        lin(L.gate, normed.data(), nullptr, count, gate.data());
        lin(L.up, normed.data(), nullptr, count, up.data());
        orc_silu_mul(gate.data(), up.data(), count * I, gated.data());
        lin(L.down, gated.data(), nullptr, count, down.data());
        orc_add(hidden.data(), down.data(), count * H, hidden.data());
    }
    orc_rmsnorm(hidden.data() + (count - 1) * H, M->w.final_norm, 1, H, C.rms_norm_eps, last_normed);
    M->filled += count;
    return 0;
}

static void head(orc_model* M, const float* normed, float* logits) {
    const orc_qtensor& E = M->w.embed;
    orc_linear_q(E.bits, normed, E.packed, E.scales, E.zeros, nullptr, 1, E.cols, E.rows, 64,
                 E.rows, 0, logits);
}

// Prefill `n` prompt ids in chunks of `chunk` (src/model/graph.ts:610-621); logits of the last
// prompt position go to `logits` (vocab floats).  Returns 0, or -1 if the context is exhausted.
int orc_prefill(orc_model* M, const uint32_t* ids, int64_t n, int64_t chunk, float* logits) {
    if (n < 1 || M->filled + n > M->max_context) return -1;
    if (chunk < 1) chunk = n;
    std::vector<float> normed(M->cfg.hidden);
    for (int64_t b = 0; b < n; b += chunk) {
        int64_t c = std::min(chunk, n - b);
        if (forward_chunk(M, ids + b, c, normed.data()) != 0) return -1;
    }
    if (logits) head(M, normed.data(), logits);
    return 0;
}

// One decode step: append `token` at position `filled`, logits of the next token to `logits`.
int orc_decode(orc_model* M, uint32_t token, float* logits, float* final_normed) {
    std::vector<float> normed(M->cfg.hidden);
    if (forward_chunk(M, &token, 1, normed.data()) != 0) return -1;
    if (final_normed) std::memcpy(final_normed, normed.data(), sizeof(float) * M->cfg.hidden);
    if (logits) head(M, normed.data(), logits);
    return 0;
}

// -log softmax(logits)[target] as the reference's perplexity harness computes it
// (test/parity/quality.test.ts:93-99): max of the float logits, a sequential double sum of
// exp(logit - max), then -((logit[target] - max) - log(sum)).
double orc_nll(const float* logits, int64_t n, uint32_t target) {
    float m = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
        if (logits[i] > m) m = logits[i];
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += std::exp((double)logits[i] - (double)m);
    return -(((double)logits[target] - (double)m) - std::log(sum));
}

// Copies of the f16 cache, for parity checks: [max_context][kv*hd] of one layer.
void orc_model_kv(const orc_model* M, uint32_t layer, uint16_t* k_out, uint16_t* v_out) {
    int64_t per = M->max_context * (int64_t)M->cfg.kv_heads * M->cfg.head_dim;
    std::memcpy(k_out, M->kcache.data() + layer * per, per * 2);
    std::memcpy(v_out, M->vcache.data() + layer * per, per * 2);
}

}  // extern "C"
