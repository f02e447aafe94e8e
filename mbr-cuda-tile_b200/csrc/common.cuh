// common.cuh — device helpers (conversions, warp reductions, activations).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

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

// complex value (two floats) <-> a pair of elements of T stored together
// (one 8-byte word for float, one 4-byte word for the 16-bit types)
template <typename T>
struct PairOf {
    using type = uint32_t;
};
template <>
struct PairOf<float> {
    using type = float2;
};
template <typename T>
__device__ __forceinline__ float2 pair_to_f32(typename PairOf<T>::type p) {
    if constexpr (std::is_same_v<T, float>) {
        return p;
    } else if constexpr (std::is_same_v<T, __half>) {
        return __half22float2(*reinterpret_cast<const __half2*>(&p));
    } else {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&p));
    }
}
template <typename T>
__device__ __forceinline__ void store_pair(T* dst, float2 v) {
    if constexpr (std::is_same_v<T, float>) {
        *reinterpret_cast<float2*>(dst) = v;
    } else if constexpr (std::is_same_v<T, __half>) {
        *reinterpret_cast<__half2*>(dst) = __float22half2_rn(v);
    } else {
        *reinterpret_cast<__nv_bfloat162*>(dst) = __float22bfloat162_rn(v);
    }
}

// asynchronous global -> shared copy of N (4, 8 or 16) bytes, both addresses
// N-byte aligned; cp_async_wait_all() waits for all of this thread's copies
template <int N>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem) {
    static_assert(N == 4 || N == 8 || N == 16, "cp.async copies 4, 8 or 16 bytes");
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(s), "l"(gmem), "n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
// GELU as the reference computes it: 0.5 x (1 + erf(x)) = x Phi(sqrt(2) x).
// Its erf-based kernels take erf of x itself, not of x / sqrt(2)
// (add_bias_gelu_kernel, src/mbr_cuda_tile.cu:5536-5558; gelu_erf_approx,
// :565-583; gelu_erf_poly9_l30, src/mbr_ffn12_cutile.cu:33-66), so it is not
// torch's nn.GELU; the outputs here follow the reference.
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x)); }

// Single-instruction approximations (PTX rcp.approx / ex2.approx, ~1-2 ulp).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The reference's GELU 0.5 x (1 + erf(x)) (see gelu_erf) of N values (N even)
// with one exponential each: gelu(x) = x - x Q(u) for x >= 0 and x Q(u) for
// x < 0, u = |x|, where the tail Q(u) = erfc(u) / 2 is evaluated as 2^P(u).
// P comes from a degree-7 least-squares Chebyshev fit of log2 of the normal
// tail, log2(erfc(t / sqrt 2) / 2) on t in [0, 5.5] (fitted in double
// precision from the log of the normal CDF, converted to monomial form), with
// t = sqrt(2) u folded into the coefficients (c_i sqrt(2)^i) and rounded to
// fp32; u is clamped to 5.5 / sqrt(2), where Q < 2e-8.  Evaluated in fp32 the
// GELU error stays below 5e-7 absolute (Q within 1.1e-5 relative), under a
// 16-bit output's rounding.  The Horner steps run on packed f32x2 pairs, all
// N/2 chains advanced together so consecutive instructions are independent.
template <int N>
__device__ __forceinline__ void gelu_tail(float (&v)[N]) {
    constexpr float kC[8] = {-9.999850392e-01f, -1.628247229e+00f, -9.164922238e-01f, -1.532212642e-01f,
                             3.443936631e-02f,  -5.409059366e-03f, 5.186771159e-04f,  -2.258130597e-05f};
    constexpr float kClamp = 3.8890873f;  // 5.5 / sqrt(2)
    float2 t[N / 2], p[N / 2];
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
        t[j] = make_float2(fminf(fabsf(v[2 * j]), kClamp), fminf(fabsf(v[2 * j + 1]), kClamp));
        p[j] = make_float2(kC[7], kC[7]);
    }
#pragma unroll
    for (int i = 6; i >= 0; --i)
#pragma unroll
        for (int j = 0; j < N / 2; ++j) p[j] = __ffma2_rn(p[j], t[j], make_float2(kC[i], kC[i]));
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
        const float x0 = v[2 * j], x1 = v[2 * j + 1];
        const float r0 = x0 * ex2_approx(p[j].x), r1 = x1 * ex2_approx(p[j].y);
        v[2 * j] = x0 >= 0.0f ? x0 - r0 : r0;
        v[2 * j + 1] = x1 >= 0.0f ? x1 - r1 : r1;
    }
}

// tanh(x) = sign(x) (1 - 2 / (e^{2|x|} + 1)); absolute error ~1e-7.
__device__ __forceinline__ float tanh_fast(float x) {
    const float e = ex2_approx(fabsf(x) * 2.8853900817779268f);  // e^{2|x|}
    const float r = fmaf(-2.0f, rcp_approx(e + 1.0f), 1.0f);
    return copysignf(r, x);
}

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
