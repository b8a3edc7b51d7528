// Internal helpers shared by the libenx translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/enx.h"

namespace enx {

// ---- error state (thread-local message, status return) ------------------------------------
void set_error(const std::string& msg);
enx_status fail(enx_status code, const std::string& msg);
enx_status cuda_fail(cudaError_t err, const char* what);

#define ENX_CUDA(call)                                                  \
    do {                                                                \
        cudaError_t _e = (call);                                        \
        if (_e != cudaSuccess) return ::enx::cuda_fail(_e, #call);      \
    } while (0)

#define ENX_TRY(call)                                                   \
    do {                                                                \
        enx_status _s = (call);                                         \
        if (_s != ENX_OK) return _s;                                    \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- numeric helpers ------------------------------------------------------------------------

// 2^23 + v as a float, for 0 <= v < 2^23: the exponent trick that turns a small unsigned code
// into a float without an int->float conversion.  (2^23 + q) - (2^23 + z) is exactly q - z.
__device__ __forceinline__ float magic_u(uint32_t v) { return __uint_as_float(0x4B000000u | v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read exactly once).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue now,
// and wait here until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

constexpr int kBlock = 64;  // quantisation block along the reduction axis

}  // namespace enx
