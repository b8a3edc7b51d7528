// Tensor-core (tcgen05) quantised projection GEMM for M >= 16 tokens (k_gemm_tc.cu).
#pragma once

#include "k_matvec.cuh"

namespace enx {

// Bytes of one (32-token group, 64-element block) limb tile: 192 rows (limb l of token t in row
// 32 l + t) x 64 int8 values, then per token the block sum of the scaled activations (int64) and
// its scale 2^-F (double).
constexpr uint32_t kTcLimbTileBytes = 192 * 64 + 32 * 16;

// Workspace for launch_gemm_tc: the limb tiles of m tokens over k and the split-K partials.
size_t gemm_tc_workspace_bytes(uint32_t m, uint32_t k);
// Extra workspace when an int4 call passes no prepared code matrix (converted per call).
size_t gemm_tc_codes_bytes(uint32_t rows, uint32_t k);

// The byte matrix [rows][cols] the GEMM reads for int4 weights: q - z per element, in the GEMM's
// slot order (gemm_tc_codes_bytes(rows, cols) bytes).  Prepared once per weight by callers that
// reuse it.
cudaError_t launch_codes_i8(const QW& w, uint8_t* out, cudaStream_t st);

// Output segments of a GEMM over stacked int4 weights (q|k|v, gate|up): rows [end[s-1], end[s]) of w
// (end[-1] = 0) go to out[s][t * stride[s] + row - end[s-1]] with bias[s] (may be null).
struct TcSeg {
    float* out[3];
    const float* bias[3];
    uint32_t stride[3];
    uint32_t end[3];
    uint32_t n;  // 0: the single output of launch_gemm_tc's out / bias / out_stride / out_offset
};

// out[t * out_stride + out_offset + n] = float(x[t] . W[n] (+ bias[n])) for t < m, n < w.rows;
// x rows ld floats apart.  bits 4 or 8; w.cols a multiple of 64.  codes8: the prepared int4 byte
// matrix, or null to convert into the workspace (which then needs gemm_tc_codes_bytes more).
// *err is raised to 3 if a bounded wait inside the kernel gives up.  limbs_ready: the previous
// call on this workspace had the same x, ld, m and w.cols, so its activation limbs are reused.
// residual: added in float to each rounded output (same layout as out; may be out itself).
cudaError_t launch_gemm_tc(int bits, const float* x, uint32_t ld, const QW& w, const uint8_t* codes8, const float* bias,
                           float* out, uint32_t m, uint32_t out_stride, uint32_t out_offset, uint8_t* workspace,
                           uint32_t* err, cudaStream_t st, bool limbs_ready = false, const float* residual = nullptr,
                           const TcSeg* seg = nullptr);

// The tied int8 head for 1-4 tokens on the tensor cores (exact limbs, like launch_gemm_tc):
// out[t * out_stride + row] = float(x_t . W[row]) for row < w.rows, t < ntok; with `gain`, x is
// first RMS-normalised in the kernel (and CTA 0 writes the normalised rows to normed_out).
// w.cols <= 1024, a multiple of 64.  pdl: launched as a programmatic dependent of the previous
// kernel (the weight stream starts before it finishes).  *err is raised to 3 if a bounded wait
// gives up.
struct HeadTcArgs {
    const float* x;                 // [ntok][K] activations
    const float* gain;              // final-norm gain: RMSNorm x here first; null: x is normalised
    float eps;
    float* normed_out;              // with gain: CTA 0 writes the normalised rows here (may be null)
    QW w;                           // int8 table (rows of this call)
    float* out;
    uint32_t out_stride, ntok;
    uint32_t* err;
};
cudaError_t launch_head_tc(const HeadTcArgs& args, cudaStream_t st, bool pdl);

// Spins a bounded wait of the tensor-core GEMM takes before it gives up (current device; 0 = the
// default 2^24).
cudaError_t tc_set_spin(uint32_t spins);

}  // namespace enx
