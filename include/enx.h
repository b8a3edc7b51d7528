/*
 * enx.h — C ABI of the B200 decode hot path (libenx.so).
 *
 * Replaces, for CUDA hosts, the WebGPU kernels and graph of the reference engine
 * (src/kernels/*.wgsl, src/model/graph_decode.ts, src/model/graph.ts, src/runtime/session.ts).
 * Plain pointers and sizes only.  Device pointers are CUDA global-memory addresses; `stream`
 * is a cudaStream_t passed as void* (NULL = the legacy default stream).
 *
 * Conventions, mirroring src/kernels/kernel.ts:20-112:
 *   - every kernel entry point takes its inputs, then its output, then a dims struct whose
 *     layout is byte-identical to the reference's uniform block for that kernel;
 *   - kernels never allocate: outputs and workspaces are caller-owned (the reference's
 *     BufferPool is the only scratch owner, src/gpu/pool.ts:1-12);
 *   - every call returns an enx_status; enx_last_error() gives the message of the last
 *     failure on the calling thread (the reference throws RangeError / EnargeiaError instead).
 *
 * Two levels:
 *   1. raw kernels (enx_matmul_q4, enx_lm_head_q8, enx_embed_gather_q8, enx_sample,
 *      enx_attn_decode, enx_rmsnorm, enx_rope, enx_cache_pack, enx_silu_mul, enx_add), each the
 *      drop-in for one WGSL dispatch;
 *   2. a model context (enx_create ... enx_destroy) holding the weights, KV caches and the
 *      captured decode step, the drop-in for WeightStore + KVCache + DecodeGraph/ForwardGraph.
 */
#ifndef ENX_H
#define ENX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ENX_API __attribute__((visibility("default")))
#else
#define ENX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t enx_status;
#define ENX_OK 0
#define ENX_ERR_INVALID 1   /* bad argument, size or pointer (kernel.ts:70-75 bind mismatch) */
#define ENX_ERR_CUDA 2      /* a CUDA runtime error; the message names the call */
#define ENX_ERR_RANGE 3     /* RangeError: grid limits, context exhausted, prompt too long */
#define ENX_ERR_FORMAT 4    /* EnargeiaError: malformed or unsupported .enargeia */
#define ENX_ERR_TIMEOUT 5   /* a bounded device-side wait gave up (no GPU hang) */
#define ENX_ERR_NOMEM 6
#define ENX_ERR_STATE 7     /* call order: e.g. decode before load */

/* Last error message of the calling thread ("" when none). */
ENX_API const char* enx_last_error(void);
/* Library version string, and the compute capability it was built for ("sm_100a"). */
ENX_API const char* enx_version(void);

/* ------------------------------------------------------------------------------------------
 * Raw kernels.  Dims structs are the reference's uniform blocks, byte for byte.
 * ---------------------------------------------------------------------------------------- */

/* matmulQ4Dims, 48 bytes (src/kernels/matmul_q4.ts:50-64). */
typedef struct {
    uint32_t m, n, k, use_bias;
    uint32_t block_size, blocks_per_row, out_stride, out_offset;
    uint32_t grid_width, pad0, pad1, pad2;
} enx_matmul_q4_dims;

/* out[row*out_stride + out_offset + col] = sum_i x[row*k + i] * (q - z) * s + bias[col]
 * Replaces matmul_q4_decode (m == 1, src/kernels/matmul_q4_decode.wgsl:56-101) and
 * matmul_q4_prefill (m > 1, src/kernels/matmul_q4_prefill.wgsl:77-162).  Bindings in the
 * reference's order: x, packed, scales, zeros, bias, out, dims.  `bias` may be NULL when
 * use_bias is 0.  Requires k % 64 == 0 and block_size == 64. */
ENX_API enx_status enx_matmul_q4(const float* x, const uint32_t* packed, const float* scales,
                         const uint32_t* zeros, const float* bias, float* out,
                         const enx_matmul_q4_dims* dims, void* stream);

/* The raw tensor-core paths of enx_matmul_q4 (m >= 16) and enx_lm_head_q8 (seq >= 16) share one
 * library-owned workspace per device (activation limbs, split-K partials, int8 weight codes),
 * grown on demand: calls that overlap on the GPU (other streams, other threads) race on it, so
 * serialise them.  Their bounded device waits record a sticky error word instead of hanging;
 * enx_raw_check reads it. */

/* Report (then clear) the sticky error word of the raw tensor-core entry points:
 * ENX_ERR_TIMEOUT if a bounded wait gave up since the last check, whose outputs are then
 * invalid.  It first waits for ALL work on the current device (cudaDeviceSynchronize), including
 * the streams of other enx contexts and of other libraries on that device, so it must not be
 * called while any stream of the device is being captured into a CUDA graph.  No reference
 * counterpart (WebGPU kernels have no device waits). */
ENX_API enx_status enx_raw_check(void);

/* How many polls a bounded device-side wait (grid barrier, readiness counter, ring or pipeline
 * mbarrier of the persistent decode kernel and of the tensor-core GEMM) makes on `device` before
 * it gives up and the call reports ENX_ERR_TIMEOUT; 0 restores the default (2^24 polls, well
 * under a minute).  A waiting CTA that gives up still waits, with the default limit, for the
 * copies and MMAs it issued before it exits.  Applies to launches made after the call (CUDA graphs
 * already captured included).  No reference counterpart: a hook to exercise the timeout path. */
ENX_API enx_status enx_set_wait_limit(int device, uint32_t spins);

/* Peer-memory exchange between the GPUs of one box (the vocab-sharded sampler's per-phase
 * all-gather without a collective library).  enx_peer_alloc allocates an exchange buffer of 512
 * header bytes + `bytes` on the current device and returns its CUDA IPC handle (64 bytes);
 * other ranks map it with enx_peer_open (lazy peer access) and unmap it with
 * enx_peer_close(ptr, 1); the owner frees it with enx_peer_close(ptr, 0).  enx_peer_allgather
 * copies `bytes` (a multiple of 16, 16-byte aligned) of `send` into slot `rank` of every rank's
 * buffer (peers: device array of the world buffers' addresses as mapped here, peers[rank] =
 * this rank's own), raises arrival word `rank` of every buffer to `seq`, and waits (bounded;
 * *err raised to 4 on giving up) until all arrival words of this rank's buffer reach `seq`; the
 * gathered region (world x bytes, rank-major) then starts 512 bytes into the own buffer.  `seq`
 * must grow by one per exchange on every rank.  Replaces the NCCL all_gather_into_tensor of
 * enargeia_b200/vocab_shard.py's protocol (no reference counterpart: the reference runs on one
 * device). */
ENX_API enx_status enx_peer_alloc(size_t bytes, void** ptr, uint8_t* handle);
ENX_API enx_status enx_peer_open(const uint8_t* handle, void** ptr);
ENX_API enx_status enx_peer_close(void* ptr, int opened);
ENX_API enx_status enx_peer_allgather(const void* send, size_t bytes, const unsigned long long* peers, uint32_t world,
                                      uint32_t rank, unsigned long long seq, uint32_t* err, void* stream);

/* embeddingDims, 48 bytes (src/kernels/embedding_variants.ts:76-90, 207-221). */
typedef struct {
    uint32_t seq, hidden, row_begin, row_count;
    uint32_t block_size, blocks_per_row, out_stride, out_offset;
    uint32_t grid_width, pad0, pad1, pad2;
} enx_embedding_dims;

/* Tied LM head over the int8 table: out[col + out_offset] = sum_k x[k] * W[col, k] for
 * col < row_count (lm_head_q8, src/kernels/embedding_variants.ts:135-180).  `packed`, `scales`
 * and `zeros` are the rows of this call (a vocab shard passes its own rows).  seq > 1 is this
 * library's batched extension: row s of x (hidden floats) goes to out + s*out_stride
 * (out_stride 0 means row_count); from 16 rows it runs on the tensor-core GEMM.
 * Bindings: x, packed, scales, zeros, out, dims. */
ENX_API enx_status enx_lm_head_q8(const float* x, const uint32_t* packed, const float* scales,
                          const uint32_t* zeros, float* out, const enx_embedding_dims* dims,
                          void* stream);

/* out[s, :] = dequant(table[ids[s] - row_begin, :]) for ids inside [row_begin, row_begin +
 * row_count) (embed_gather_q8, src/kernels/embedding_variants.ts:100-130).  Bindings: ids,
 * packed, scales, zeros, out, dims. */
ENX_API enx_status enx_embed_gather_q8(const uint32_t* ids, const uint32_t* packed, const float* scales,
                               const uint32_t* zeros, float* out, const enx_embedding_dims* dims,
                               void* stream);

/* sampleDims, 32 bytes (src/kernels/sample.ts:35-50). */
typedef struct {
    uint32_t vocab, history_length;
    float temperature, top_p, repetition_penalty, random;
    uint32_t pad0, pad1;
} enx_sample_dims;

/* The sampler of src/kernels/sample.wgsl:143-332: in-place repetition penalty on `logits`,
 * then greedy argmax (temperature <= 0) or temperature / top-p / seeded draw; writes one id to
 * out[0].  Bindings: logits (read_write), history, out, dims.  Probabilities, bisection masses
 * and the running draw total are computed in double (the oracle's exact-arithmetic rule).
 * `workspace` is an EXTENSION of the reference's binding list (logits, history, out, dims;
 * src/kernels/sample.ts:24-52): it is unused and may be NULL (the kernel keeps its state in
 * shared memory), and is kept so the raw entry points share one call shape (inputs, output,
 * dims, workspace, stream). */
ENX_API enx_status enx_sample(float* logits, const uint32_t* history, uint32_t* out,
                      const enx_sample_dims* dims, void* workspace, void* stream);

/* Batched form: rows b = 0..batch-1 of logits [batch][vocab] with their own histories
 * (history + b*history_stride, history_length[b]) and params; out[b].  All pointers device. */
typedef struct {
    float temperature, top_p, repetition_penalty, random;
} enx_sampling_row;

ENX_API enx_status enx_sample_batched(float* logits, uint32_t vocab, uint32_t batch,
                              const uint32_t* history, uint32_t history_stride,
                              const uint32_t* history_length, const enx_sampling_row* rows,
                              uint32_t* out, void* stream);

/* attnDecodeDims, 32 bytes (src/kernels/attn_decode.ts:23-32). */
typedef struct {
    uint32_t position, heads, kv_heads, head_dim;
    uint32_t score_stride, cache_stride, pad0, pad1;
} enx_attn_decode_dims;

/* Decode attention of one query over the f16 cache, fused: attn_scores_decode_f16 +
 * softmax + attn_apply_decode_parallel_f16 (src/kernels/cache_variants.ts:147-179,
 * src/kernels/softmax.wgsl:30-81, src/kernels/cache_variants.ts:353-399).
 * q f32[heads*head_dim]; k_cache/v_cache f16 bits [position+1][cache_stride]; out
 * f32[heads*head_dim].  `workspace` holds split partials: enx_attn_decode_workspace_bytes(). */
ENX_API enx_status enx_attn_decode(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                           float* out, const enx_attn_decode_dims* dims, void* workspace,
                           void* stream);
/* Same computation as enx_attn_decode, for callers that cannot allocate device memory (for
 * example code running where cudaMalloc's implicit synchronisation is not allowed, or hosts that
 * only hand over fixed buffers).  No counterpart in the reference: its WebGPU path always has a
 * buffer pool.  The attention scores live in one library-owned device array (512 KB, held on
 * every GPU that loads the library until exit); limits: position < 4096, heads <= 32,
 * head_dim <= 64, else ENX_ERR_RANGE.  The first call on each device looks up that array's
 * device address (cudaGetSymbolAddress, with the device current): make that first call before
 * any stream capture.  All calls share the array, so calls that overlap on the GPU (other
 * streams, other threads) race; serialise them.  Allocates nothing. */
ENX_API enx_status enx_attn_decode_noalloc(const float* q, const uint16_t* k_cache,
                                           const uint16_t* v_cache, float* out,
                                           const enx_attn_decode_dims* dims, void* stream);
ENX_API size_t enx_attn_decode_workspace_bytes(uint32_t max_context, uint32_t heads, uint32_t head_dim);

/* Prefill attention of a chunk: queries i = 0..queries-1 at absolute positions begin+i attend
 * cached keys 0..begin+i (attn_scores_f16 / softmax / attn_apply_f16,
 * src/kernels/cache_variants.ts:81-144).  q f32[queries][heads*hd]; out likewise. */
ENX_API enx_status enx_attn_prefill(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            float* out, uint32_t queries, uint32_t begin, uint32_t heads,
                            uint32_t kv_heads, uint32_t head_dim, void* workspace, void* stream);
ENX_API size_t enx_attn_prefill_workspace_bytes(uint32_t queries, uint32_t keys, uint32_t heads,
                                        uint32_t head_dim);

/* RMSNorm rows (src/kernels/rmsnorm.wgsl:27-63): out = x * rsqrt(mean(x^2) + eps) * w. */
ENX_API enx_status enx_rmsnorm(const float* x, const float* weight, float* out, uint32_t seq,
                       uint32_t features, float eps, void* stream);

/* Half-rotation RoPE (src/kernels/rope.wgsl:28-53) from a cos/sin table
 * ([max_pos][head_dim/2] each, f32); out[out_offset + ...].  Rows s at position
 * position_offset + s. */
ENX_API enx_status enx_rope(const float* x, float* out, const float* cos_table, const float* sin_table,
                    uint32_t seq, uint32_t heads, uint32_t head_dim, uint32_t position_offset,
                    uint32_t out_offset, void* stream);

/* f32 -> f16 (round to nearest even) pack into a cache at element offset dst_offset
 * (cache_pack_f16, src/kernels/cache_variants.ts:269-301, cachePackDims). */
ENX_API enx_status enx_cache_pack(const float* src, uint16_t* dst, uint32_t count, uint32_t dst_offset,
                          void* stream);
ENX_API enx_status enx_silu_mul(const float* gate, const float* up, float* out, uint32_t count,
                        void* stream);
ENX_API enx_status enx_add(const float* a, const float* b, float* out, uint32_t count, void* stream);

/* ------------------------------------------------------------------------------------------
 * Model context: WeightStore + KVCache + DecodeGraph + ForwardGraph + Session's step.
 * One context is used from one host thread and owns one CUDA stream.
 * ---------------------------------------------------------------------------------------- */

/* ModelConfig (src/model/graph.ts:57-67). */
typedef struct {
    uint32_t layers, hidden, heads, kv_heads, head_dim, intermediate, vocab;
    float rms_norm_eps, rope_theta;
} enx_model_config;

/* SamplingParams (src/kernels/sample.ts:24-33). */
typedef struct {
    float temperature, top_p, repetition_penalty;
} enx_sampling;

typedef struct enx_ctx enx_ctx;

/* Create a context on CUDA device `device`. */
ENX_API enx_status enx_create(const enx_model_config* cfg, int device, enx_ctx** out);
ENX_API enx_status enx_destroy(enx_ctx* ctx);

/* Load every tensor of a .enargeia file (WeightStore.loadQuantized, src/model/weights.ts:
 * 299-471): the file is parsed here (magic, version, JSON header, 256-aligned ranges,
 * src/model/enargeia.ts:112-240) and each range is copied to the device verbatim. */
ENX_API enx_status enx_load_enargeia(enx_ctx* ctx, const char* path);
/* Same, from a host buffer holding the whole file. */
ENX_API enx_status enx_load_enargeia_memory(enx_ctx* ctx, const void* data, size_t size);

/* Preallocate f16 KV caches for `batch` sequences of `max_context` positions each
 * (KVCache constructor, src/runtime/kvcache.ts:59-88).  Also sizes the decode scratch. */
ENX_API enx_status enx_kv_alloc(enx_ctx* ctx, uint32_t max_context, uint32_t batch);
/* Forget sequence `seq` without freeing (KVCache.reset, src/runtime/kvcache.ts:135-137). */
ENX_API enx_status enx_kv_reset(enx_ctx* ctx, uint32_t seq);
/* Positions filled in sequence `seq` (KVCache.filled). */
ENX_API enx_status enx_kv_filled(enx_ctx* ctx, uint32_t seq, uint32_t* filled);

/* Chunked prefill of `n` ids into sequence `seq` (Session.runPrefill + ForwardGraph.
 * encodeChunks, src/runtime/session.ts:326-344, src/model/graph.ts:610-621).  The ids become
 * the sequence's history; the logits of the last prompt position are kept on the device for
 * enx_sample_prefill / enx_logits.  ENX_ERR_RANGE if the prompt exceeds the remaining context. */
ENX_API enx_status enx_prefill(enx_ctx* ctx, uint32_t seq, const uint32_t* ids, uint32_t n,
                       uint32_t chunk);

/* Session.sampleFromPrefill (src/runtime/session.ts:472-495): sample the first token from the
 * prefill logits with `params` and draw `random`; the id is written to *out_id (host). */
ENX_API enx_status enx_sample_prefill(enx_ctx* ctx, uint32_t seq, const enx_sampling* params,
                              float random, uint32_t* out_id);

/* One decode step for sequences 0..batch-1 (Session.decodeStep, src/runtime/session.ts:
 * 347-375): append tokens[b] at each sequence's next position, run the whole decoder and the
 * sampler, write the next ids to out_ids[b].  tokens/params/randoms/out_ids are HOST arrays
 * of `batch` entries; params may hold one entry (shared) when params_count == 1.  The fed token
 * joins the sequence's history before sampling, as in the reference. */
ENX_API enx_status enx_decode_step(enx_ctx* ctx, uint32_t batch, const uint32_t* tokens,
                           const enx_sampling* params, uint32_t params_count,
                           const float* randoms, uint32_t* out_ids);

/* Decode `steps` tokens for sequences 0..batch-1 with no host round trip between steps (the
 * loop of Session.generate, src/runtime/session.ts:440-452, kept on the device): step 0 feeds
 * first_tokens[b], step i feeds the id sampled at step i-1; step i of sequence b draws
 * randoms[i*batch + b].  Each step is one launch of the captured decode graph.  With sync != 0
 * the call waits and writes steps*batch ids to out_ids (host); with sync == 0 it only enqueues
 * on the context stream, and enx_synchronize + enx_loop_ids fetch the ids later (out_ids may
 * then be NULL).  ENX_ERR_RANGE if a sequence would run past its context. */
ENX_API enx_status enx_decode_loop(enx_ctx* ctx, uint32_t batch, const uint32_t* first_tokens,
                                   const enx_sampling* params, uint32_t params_count,
                                   uint32_t steps, const float* randoms, uint32_t* out_ids,
                                   int sync);
/* Wait for all work queued on the context's stream. */
ENX_API enx_status enx_synchronize(enx_ctx* ctx);
/* Ids of the last enx_decode_loop (count = steps*batch), after enx_synchronize. */
ENX_API enx_status enx_loop_ids(enx_ctx* ctx, uint32_t* out_ids, uint32_t count);

/* Logits of the last step of sequence `seq` (Session.logitsAfter's readback,
 * src/runtime/session.ts:385-401), copied to host `out` (vocab floats).  Valid after
 * enx_prefill or enx_decode_step; a sampled step with a repetition penalty has modified them in
 * place, as in the reference. */
ENX_API enx_status enx_logits(enx_ctx* ctx, uint32_t seq, float* out);

/* Negative log-likelihood of `target` under the softmax of sequence `seq`'s current logits, in
 * double: -((logit[target] - max) - log(sum_i exp(logit[i] - max))), the per-position term of the
 * reference's perplexity harness (test/parity/quality.test.ts:93-99, over the logits that
 * Session.logitsAfter returns, src/runtime/session.ts:385-401).  Computed on the device, so a
 * perplexity evaluation reads 8 bytes per position instead of the whole logits row. */
ENX_API enx_status enx_nll(enx_ctx* ctx, uint32_t seq, uint32_t target, double* out);

/* Final-norm hidden state of the last step of sequence `seq` (hidden floats, host). */
ENX_API enx_status enx_hidden(enx_ctx* ctx, uint32_t seq, float* out);

/* Device view of one layer's cache of sequence `seq` (f16 bits, [max_context][kv_heads*hd]),
 * for parity checks. */
ENX_API enx_status enx_kv_view(enx_ctx* ctx, uint32_t seq, uint32_t layer, const uint16_t** k,
                       const uint16_t** v);

/* Device pointers of one loaded tensor (packed/scales/zeros for Q4/Q8, data in `packed` for
 * F32).  Shapes are returned in rows/cols (cols = 1 for 1-D). */
ENX_API enx_status enx_tensor_view(enx_ctx* ctx, const char* name, int32_t* dtype_bits, uint32_t* rows,
                           uint32_t* cols, const void** packed, const float** scales,
                           const uint32_t** zeros);

/* Stage telemetry (Session.setInstrumented + the per-kernel timestamp queries of
 * src/runtime/session.ts:162-308).  With tracing on, the persistent decode kernel stamps the
 * device clock (ns) three times per stage: when the stage starts (its barrier released), when its
 * weights have landed in shared memory, and when its compute is done; stages are 3 per layer
 * (q|k|v + attention + o partial, gate/up, down) then the head.  After those 3 * (3*layers + 1)
 * values come 8 per layer inside the attention stage and 2 head totals (waiting, computing), all
 * of the first CTA.  enx_trace copies the stamps of the last step (unused slots are 0).  Turning
 * tracing on or off re-captures the decode graphs on the next step. */
ENX_API enx_status enx_set_tracing(enx_ctx* ctx, int on);
ENX_API enx_status enx_trace(enx_ctx* ctx, uint64_t* out, uint32_t capacity, uint32_t* count);

/* The CUDA stream the context runs on (cudaStream_t as void*). */
ENX_API enx_status enx_stream(enx_ctx* ctx, void** stream);

/* Kernel launches issued by the last enx_decode_step (the captured step's node count). */
ENX_API enx_status enx_step_launches(enx_ctx* ctx, uint32_t* launches);

/* Measurement hook: enqueue on the context stream, `count` times, the weight-streaming kernels of
 * a decode step -- the persistent layer kernel (after its tag-epoch bump) and the tied-head kernel
 * -- for the `batch` tokens and positions of the last decode step, without the sampler or any
 * host copy.  Re-running a step rewrites the same cache rows and
 * logits.  ENX_ERR_STATE if no step ran yet or the step did not use the persistent kernel. */
ENX_API enx_status enx_launch_step_kernel(enx_ctx* ctx, uint32_t batch, uint32_t count);

/* Measurement hook for batched decode (more than 4 sequences): runs the last batched step's body
 * once, outside its graph, with CUDA events between sections, and writes each section's total
 * time in ms to ms[0..9]: embed, RMSNorms, q|k|v GEMMs, RoPE + cache rows, attention, o GEMM +
 * residual, gate/up GEMMs + SiLU, down GEMM + residual, head GEMM, sampler.  With count >= 14 the
 * many-token attention is also timed stage by stage into ms[10..13]: scores, softmax rows,
 * weighted V, combine.  It rewrites the same cache rows and logits.  count must be at least 10. */
ENX_API enx_status enx_batch_profile(enx_ctx* ctx, uint32_t batch, float* ms, uint32_t count);

/* ------------------------------------------------------------------------------------------
 * Vocab-sharded sampling (the sampler of src/kernels/sample.wgsl:143-332 over a head split by
 * contiguous id ranges across GPUs; the reference samples one unsplit vocabulary).
 *
 * Rank r of `world` holds logits [rows][n] for ids [row_begin, row_begin + n); ranks' ranges are
 * in ascending id order.  `split` CTAs per row each own a contiguous part of the shard; a "unit"
 * is (rank, cta) and units in rank-major order cover the vocabulary in id order.  Each phase
 * writes a send buffer of one record per (row, cta) - [rows][split] - and the caller allgathers
 * every rank's send buffer into [world][rows][split] (rank-major: NCCL all_gather_into_tensor)
 * before the next phase reads it:
 *   prepare -> cand u32[4]  | probs -> sum f64 | buckets x4 -> bucket u64[256] | kept -> kept f64
 *   | pick -> pick u32 | finish -> out[rows]
 * Bucket masses are round(p * 2^62) summed as integers (exact, order-free).  With topp_rounds 0
 * (no row has top_p < 1) the bucket phases are skipped and kept normalises.
 * `state` (enx_shard_state_bytes(rows), device) and `probs` (f64 [rows][n], device) stay on the
 * rank between phases.  Every rank computes the same ids in `out`.  All pointers device.
 * ---------------------------------------------------------------------------------------- */
ENX_API size_t enx_shard_state_bytes(uint32_t rows);
ENX_API enx_status enx_shard_prepare(float* logits, uint32_t n, uint32_t row_begin, uint32_t rows,
                                     uint32_t split, const uint32_t* history, uint32_t history_stride,
                                     const uint32_t* history_length, const enx_sampling_row* params,
                                     uint32_t* cand, void* stream);
ENX_API enx_status enx_shard_probs(const float* logits, uint32_t n, uint32_t rows, uint32_t split,
                                   uint32_t world, const enx_sampling_row* params,
                                   const uint32_t* cand_all, void* state, double* probs, double* sum,
                                   void* stream);
ENX_API enx_status enx_shard_buckets(uint32_t n, uint32_t rows, uint32_t split, uint32_t world,
                                     uint32_t round, const enx_sampling_row* params,
                                     const double* sum_all, const uint64_t* bucket_prev, void* state,
                                     double* probs, uint64_t* bucket, void* stream);
ENX_API enx_status enx_shard_kept(uint32_t n, uint32_t rows, uint32_t split, uint32_t world,
                                  uint32_t topp_rounds, const enx_sampling_row* params,
                                  const double* sum_all, const uint64_t* bucket_last, void* state,
                                  double* probs, double* kept, void* stream);
ENX_API enx_status enx_shard_pick(uint32_t n, uint32_t row_begin, uint32_t rows, uint32_t split,
                                  uint32_t world, uint32_t rank, const enx_sampling_row* params,
                                  const double* kept_all, const void* state, const double* probs,
                                  uint32_t* pick, void* stream);
ENX_API enx_status enx_shard_finish(uint32_t rows, uint32_t split, uint32_t world,
                                    const enx_sampling_row* params, const uint32_t* cand_all,
                                    const uint32_t* pick_all, const void* state, uint32_t* out,
                                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ENX_H */
