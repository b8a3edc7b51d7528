// Arguments and launcher of the persistent decode kernel (k_mega.cu).
#pragma once

#include "k_decode.cuh"

namespace enx {

constexpr uint32_t kMaxLayers = 32;

struct MegaArgs {
    uint32_t hidden, heads, kv_heads, head_dim, intermediate, vocab, layers;
    float eps, attn_scale;
    LayerArgs layer[kMaxLayers];
    QW head;
    int head_bits;
    const float* final_norm;
    StepArgs S;                  // activations, caches, RoPE table, positions
    const uint32_t* tokens;      // [MT] ids fed this step (device)
    unsigned long long* bar;     // grid-barrier arrival counter, zeroed before each launch
    uint32_t* err;               // sticky error: 1 barrier timeout, 2 copy timeout
    uint32_t nslots, slot_bytes, head_chunk, x4_floats;
    unsigned long long* trace;   // optional: globaltimer stamps of CTA 0, 3 per stage (see k_mega.cu)
};

struct MegaGeometry {
    uint32_t grid, nslots, slot_bytes, x4_floats, max_positions;
    size_t smem;
};

MegaGeometry mega_geometry(uint32_t mt, const MegaArgs& A);
cudaError_t launch_mega(uint32_t mt, const MegaArgs& A, const MegaGeometry& g, cudaStream_t st);

}  // namespace enx
