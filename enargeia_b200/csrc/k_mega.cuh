// Arguments, schedule table and launcher of the persistent decode kernel (k_mega.cu).
#pragma once

#include <vector>

#include "k_decode.cuh"

namespace enx {

constexpr uint32_t kMaxLayers = 32;
constexpr uint32_t kMegaSlots = 8;   // upper bound on ring slots
constexpr uint32_t kMegaStages = 5;  // grid-barrier stages per layer (qkv, attention, o, gate/up, down)

// One bulk copy of a slice: global source, size, destination offset inside the slot.
struct MegaCopy {
    unsigned long long src;
    uint32_t bytes, dst;
};

// A row range [r0, r1) of one quantised tensor as staged in a slot: where its packed codes,
// scales and zero words start inside the slot, and the global scale / zero-word index of the
// first staged scale / zero word (the copies are widened to 16-byte boundaries).
struct MegaRange {
    uint32_t r0, r1;
    uint32_t off_p, off_s, off_z;
    uint32_t s_base, z_base;
    uint32_t tag;  // stage-specific: q/k/v kind for the q|k|v stage
};

// Everything one CTA needs for one slice (one stage of one layer, or one chunk of head rows).
struct MegaSlice {
    uint32_t ncopy, nrange, bytes, pad;
    MegaCopy copy[12];
    MegaRange range[4];
};

struct MegaArgs {
    uint32_t hidden, heads, kv_heads, head_dim, intermediate, vocab, layers;
    float eps;
    LayerArgs layer[kMaxLayers];
    QW head;
    int head_bits;
    const float* final_norm;
    StepArgs S;                   // activations, caches, RoPE table, positions
    const uint32_t* tokens;       // [MT] ids fed this step (device)
    unsigned long long* bar;      // grid-barrier arrival counter, zeroed before each launch
    uint32_t* err;                // sticky error: 1 barrier timeout, 2 copy timeout
    const MegaSlice* table;       // [grid][table_stride] slices, built on the host
    const uint32_t* nslices;      // [grid] slices per CTA
    uint32_t table_stride;
    uint32_t nslots, slot_bytes, x4_floats;
    unsigned long long* trace;    // optional: globaltimer stamps of CTA 0, 3 per stage
};

struct MegaGeometry {
    uint32_t grid, nslots, slot_bytes, x4_floats, max_positions, head_chunk;
    size_t smem;
};

// Grid, ring and shared-memory geometry for `mt` tokens.
MegaGeometry mega_geometry(uint32_t mt, const MegaArgs& A);
// The per-CTA slice table for that geometry (host side): table[c * stride + i], counts[c].
void mega_build_table(const MegaArgs& A, const MegaGeometry& g, std::vector<MegaSlice>& table,
                      std::vector<uint32_t>& counts, uint32_t& stride);
cudaError_t launch_mega(uint32_t mt, const MegaArgs& A, const MegaGeometry& g, cudaStream_t st);

}  // namespace enx
