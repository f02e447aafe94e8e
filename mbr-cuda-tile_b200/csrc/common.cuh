// common.cuh — device helpers (conversions, warp reductions, activations).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"

namespace mbr {

// ---------------------------------------------------------------------------
// element conversions
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// torch / Tensor::pad_reflect index (no edge repeat), valid for pad < n.
__host__ __device__ __forceinline__ int64_t reflect_idx(int64_t p, int64_t n) {
    if (n <= 1) return 0;
    while (p < 0 || p >= n) {
        if (p < 0) p = -p;
        if (p >= n) p = 2 * (n - 1) - p;
    }
    return p;
}

// Dispatch a compute dtype to a C++ element type.
#define MBR_DISPATCH_DTYPE(dt, T, ...)                                        \
    do {                                                                      \
        if ((dt) == ::mbr::DT_F32) {                                          \
            using T = float;                                                  \
            __VA_ARGS__;                                                      \
        } else if ((dt) == ::mbr::DT_F16) {                                   \
            using T = __half;                                                 \
            __VA_ARGS__;                                                      \
        } else if ((dt) == ::mbr::DT_BF16) {                                  \
            using T = __nv_bfloat16;                                          \
            __VA_ARGS__;                                                      \
        } else {                                                              \
            throw ::mbr::Error(::mbr::ERR_UNSUPPORTED, "unsupported dtype");  \
        }                                                                     \
    } while (0)

}  // namespace mbr
