// Shared device/host helpers for the ARGUS B200 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "argus_b200.h"

#define ARGUS_CHECK_LAUNCH()                                    \
    do {                                                        \
        cudaError_t e__ = cudaGetLastError();                   \
        if (e__ != cudaSuccess) return argus_set_cuda_error(e__); \
    } while (0)

// Records the CUDA error text for argus_last_error() and returns ARGUS_ERR_CUDA.
int argus_set_cuda_error(cudaError_t e);
// Records a message for argus_last_error() and returns `status`.
int argus_set_error(int status, const char* msg);
// Read and clear the device status words of the JL contraction (jl.cu), the JL attention
// (jl_attention.cu) and the outlier-correction builder (sidecar.cu) after synchronising `st`.
int argus_jl_take_status(int* status, cudaStream_t st);
int argus_jla_take_status(int* status, cudaStream_t st);
int argus_side_take_status(int* status, cudaStream_t st);

static inline bool argus_aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static inline int argus_grid_cap(int64_t blocks) {
    // Grid-stride kernels: a few waves over 148 SMs is enough to saturate HBM.
    const int64_t cap = 148 * 32;
    return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// ------------------------------------------------------------------ device helpers
namespace argus {

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
// fp32 op followed by round-to-nearest-even to fp16, as torch's CPU fp16 ops do.
__device__ __forceinline__ float rh(float v) { return __half2float(__float2half_rn(v)); }

// torch's CPU float->int8/uint8 cast: truncate to int32, keep the low byte; NaN -> 0.
__device__ __forceinline__ uint32_t w8(float v) {
    if (v != v) return 0u;
    return (uint32_t)((int32_t)v) & 0xffu;  // callers clamp to |v| <= 240 first
}

// clamp that lets NaN through (torch.clamp semantics).
__device__ __forceinline__ float clamp_nan(float v, float lo, float hi) {
    return (v != v) ? v : fminf(fmaxf(v, lo), hi);
}

__device__ __forceinline__ float round_even(float v) { return rintf(v); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace argus
