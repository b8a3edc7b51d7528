// Launchers of the row-wise / elementwise kernels (k_small.cu) and of the sampler (k_sample.cu).
#pragma once

#include "enx_internal.cuh"

namespace enx {

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, uint32_t seq,
                           uint32_t features, float eps, cudaStream_t st);
cudaError_t launch_rope(const float* x, float* out, const float* ct, const float* sn, uint32_t seq,
                        uint32_t heads, uint32_t hd, uint32_t pos0, uint32_t out_offset,
                        cudaStream_t st);
cudaError_t launch_rope_d(const float* x, float* out, const double* ct, const double* sn, uint32_t seq,
                          uint32_t heads, uint32_t hd, uint32_t pos0, uint32_t out_offset, cudaStream_t st);
cudaError_t launch_cache_pack(const float* src, uint16_t* dst, uint32_t count, uint32_t dst_offset,
                              cudaStream_t st);
cudaError_t launch_silu_mul(const float* g, const float* u, float* out, uint32_t n, cudaStream_t st);
cudaError_t launch_add(const float* a, const float* b, float* out, uint32_t n, cudaStream_t st);

// -log softmax(logits)[target] in double (one row, one block): the perplexity harness's nll.
cudaError_t launch_nll(const float* logits, uint32_t vocab, uint32_t target, double* out, cudaStream_t st);

// Per-row sampling parameters on the device.
struct SampleRow {
    float temperature, top_p, repetition_penalty, random;
};

// Samples rows b = 0..batch-1 of logits [batch][vocab] (in-place penalty), histories at
// history + b*history_stride with lengths hist_len[b] (device; when null every row's length is
// history_stride), params rows[b] (device; rows[0] for all when rows_shared; row0 by value when
// rows is null), ids to out[b] (device).
cudaError_t launch_sample(float* logits, uint32_t vocab, uint32_t batch, const uint32_t* history,
                          uint32_t history_stride, const uint32_t* hist_len, const SampleRow* rows,
                          bool rows_shared, SampleRow row0, uint32_t* out, cudaStream_t st,
                          bool pdl);
// Largest vocabulary the sampler keeps on chip.
uint32_t sample_max_vocab();

}  // namespace enx
