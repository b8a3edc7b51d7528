// Tensor-core (tcgen05) quantised projection GEMM for M >= 16 tokens (k_gemm_tc.cu).
#pragma once

#include "k_matvec.cuh"

namespace enx {

// Bytes of one (32-token group, 64-element block) limb tile: 256 rows x 64 int8 limbs, then per
// token the block sum of the scaled activations (int64) and its scale 2^-F (double).
constexpr uint32_t kTcLimbTileBytes = 256 * 64 + 32 * 16;

// Workspace for launch_gemm_tc: the limb tiles of m tokens over k.
size_t gemm_tc_workspace_bytes(uint32_t m, uint32_t k);

// out[t * out_stride + out_offset + n] = float(x[t] . W[n] (+ bias[n])) for t < m, n < w.rows;
// x rows ld floats apart.  bits 4 or 8; w.cols a multiple of 64.  *err is raised to 3 if a
// bounded wait inside the kernel gives up.
cudaError_t launch_gemm_tc(int bits, const float* x, uint32_t ld, const QW& w, const float* bias, float* out,
                           uint32_t m, uint32_t out_stride, uint32_t out_offset, uint8_t* workspace, uint32_t* err,
                           cudaStream_t st);

}  // namespace enx
