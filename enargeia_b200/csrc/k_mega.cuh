// Arguments, schedule table and launcher of the persistent decode kernel (k_mega.cu).
#pragma once

#include <vector>

#include "k_decode.cuh"

namespace enx {

constexpr uint32_t kMaxLayers = 32;
constexpr uint32_t kMegaSlots = 8;   // upper bound on ring slots
constexpr uint32_t kMegaStages = 3;  // traced stages per layer (attention + o, gate/up, down)
constexpr uint32_t kMegaTraceDetail = 14;  // extra stamps per layer inside stage A
constexpr uint32_t kMegaBarWords = 64;    // u64 words of step counters (word 0: the tag epoch, then arrival counters)
constexpr uint32_t kMegaMaxTokens = 4;    // tokens per launch the tagged buffers are sized for

// 64-bit words of the tagged stage outputs for `mt` tokens: two layer-parity copies of x, q, k|v,
// attention output, x after the o-projection and the gated activations.
inline size_t mega_ll_words(uint32_t mt, uint32_t hidden, uint32_t kv_dim, uint32_t intermediate) {
    return 2 * (size_t)mt * (4 * (size_t)hidden + 2 * (size_t)kv_dim + intermediate);
}

// One bulk copy of a slice: global source, size, destination offset inside the slot.
struct MegaCopy {
    unsigned long long src;
    uint32_t bytes, dst;
};

// A row range [r0, r1) of one quantised tensor as staged in a slot: where its packed codes,
// scales, zero words and (q|k|v units) biases start inside the slot, and the global scale /
// zero-word index of the first staged scale / zero word (copies are widened to 16 bytes).
struct MegaRange {
    uint32_t r0, r1;
    uint32_t off_p, off_s, off_z, off_b;
    uint32_t s_base, z_base;
    uint32_t tag;  // q|k|v units: 0 q, 1 k, 2 v
};

// Rows copied one by one to a padded stride in the slot (conflict-free row-per-lane reads).
struct MegaRows {
    unsigned long long src;
    uint32_t n, bytes, src_stride, dst, dst_stride, pad;
};

// Everything one CTA needs for one slice (one weight group of one stage, or a chunk of head rows):
// the bulk copies and, for stages that start with an RMSNorm, the slot offset of its gain vector.
struct MegaSlice {
    uint32_t ncopy, nrange, bytes, off_v;
    MegaCopy copy[18];
    MegaRows rows;
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
    unsigned long long* ll;       // tagged stage outputs (mega_ll_words(kMaxStepTokens, ...) words, zeroed once)
    const uint32_t* ll_epoch;     // launch counter of the tags, bumped before each launch
    uint32_t* err;                // sticky error: 1 activation wait timeout, 2 copy timeout
    const MegaSlice* table;       // [grid][table_stride] slices, built on the host
    const uint32_t* nslices;      // [grid] slices per CTA
    uint32_t table_stride;
    uint32_t nslots, slot_bytes, x4_floats;
    unsigned long long* trace;    // optional: globaltimer stamps of CTA trace_cta, 3 per stage
    uint32_t trace_cta;
};

struct MegaGeometry {
    uint32_t grid, nslots, slot_bytes, x4_floats, max_positions;
    size_t smem;
};

// Grid, ring and shared-memory geometry for `mt` tokens; nslots < 2 means the shape is not supported.
MegaGeometry mega_geometry(uint32_t mt, const MegaArgs& A);
// The per-CTA slice table for `mt` tokens (host side): table[c * stride + i], counts[c].
void mega_build_table(uint32_t mt, const MegaArgs& A, const MegaGeometry& g, std::vector<MegaSlice>& table,
                      std::vector<uint32_t>& counts, uint32_t& stride);
// Spins a bounded wait of the persistent kernel takes before it gives up (current device; 0 = the
// default 2^24).
cudaError_t mega_set_spin(uint32_t spins);
cudaError_t launch_mega(uint32_t mt, const MegaArgs& A, const MegaGeometry& g, cudaStream_t st);

}  // namespace enx
