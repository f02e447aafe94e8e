// tensor_kernels.cu — kernels behind the Tensor API: copy / dtype conversion,
// fill, broadcast binary ops, scalar ops, reductions over one dim, reflect
// padding, index_select, arange.
//
// Restates the elementwise, broadcast and reduction kernels of the reference
// tensor library (src/tensor_cuda_tile.cu:264-338, src/tensor_cuda_glue.cu:57-559)
// for sm_100a:
//  * contiguous operands of one floating dtype (the common case) take
//    vectorised kernels: every thread moves 16-byte vectors (8 x 16-bit or
//    2 x 4 x fp32 per step), grid-stride, with the dtype and the operation as
//    template parameters, so the inner loop has no branches or conversions
//    other than the element's own; a [D] operand broadcast over rows and a
//    scalar operand have their own vector paths;
//  * reductions over a contiguous last dim give a warp 8 rows at a time:
//    16-byte loads along the rows, fp32 accumulation, a reduce-scatter
//    shuffle butterfly at the end;
//    reductions over the leading dim of a contiguous [len][n] tensor with few
//    outputs (column sums) split the rows over CTAs (coalesced rows, a shared
//    memory combine, fp32 partials from the stream-ordered pool, then a
//    second pass); other reductions keep one thread per output, whose strided
//    walk is coalesced across neighbouring outputs;
//  * the contiguous copy of a transposed 2-D view goes through shared-memory
//    tiles (64 x 64 for 4-byte elements, 32-bit pairs for 16-bit ones);
//  * everything else (views with arbitrary strides, mixed dtypes) takes the
//    generic strided kernels, with 32-bit index arithmetic when the element
//    count allows.
// Shapes and strides travel by value in the launch parameters (the reference
// uploads them with a blocking cudaMemcpy per call, src/tensor_cuda_glue.cu:47-55),
// so no op synchronises the host.
#include <type_traits>

#include "common.cuh"
#include "memory_pool.h"
#include "tensor_kernels.h"

namespace cudasep {
namespace tk {

namespace {

enum Dt { F32 = 0, F16 = 1, I64 = 2, BF16 = 3 };

struct Geo {
    int nd;
    int64_t shape[kMaxDims];
    int64_t s[3][kMaxDims];  // strides of up to three operands
};

Geo make_geo(int nd, const int64_t* shape, const int64_t* s0, const int64_t* s1, const int64_t* s2) {
    if (nd > kMaxDims) throw mbr::Error(mbr::ERR_UNSUPPORTED, "tensor: more than 8 dims");
    Geo g{};
    g.nd = nd;
    for (int i = 0; i < nd; ++i) {
        g.shape[i] = shape[i];
        g.s[0][i] = s0 ? s0[i] : 0;
        g.s[1][i] = s1 ? s1[i] : 0;
        g.s[2][i] = s2 ? s2[i] : 0;
    }
    return g;
}

// Element offsets of linear index `lin` (row-major over g.shape) in the three
// operands; I is the index type (uint32_t when every offset fits).
template <typename I>
__device__ __forceinline__ void offsets(const Geo& g, I lin, int64_t& o0, int64_t& o1, int64_t& o2) {
    o0 = o1 = o2 = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
        const I n = (I)g.shape[d];
        const I q = lin / n;
        const I i = lin - q * n;
        lin = q;
        o0 += (int64_t)i * g.s[0][d];
        o1 += (int64_t)i * g.s[1][d];
        o2 += (int64_t)i * g.s[2][d];
    }
}

// ---- scalar element access (generic paths) ----
__device__ __forceinline__ float ldf(const void* p, int dt, int64_t off) {
    switch (dt) {
        case F32: return ((const float*)p)[off];
        case F16: return __half2float(((const __half*)p)[off]);
        case I64: return (float)((const int64_t*)p)[off];
        default: return __bfloat162float(((const __nv_bfloat16*)p)[off]);
    }
}
__device__ __forceinline__ void stf(void* p, int dt, int64_t off, float v) {
    switch (dt) {
        case F32: ((float*)p)[off] = v; break;
        case F16: ((__half*)p)[off] = __float2half_rn(v); break;
        case I64: ((int64_t*)p)[off] = (int64_t)v; break;
        default: ((__nv_bfloat16*)p)[off] = __float2bfloat16_rn(v); break;
    }
}

// ---- 8-element vectors: one 16-byte access for 16-bit types, two for fp32 ----
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}
template <typename T>
__device__ __forceinline__ float tof(T x) {
    return mbr::to_f32(x);
}
template <typename T>
__device__ __forceinline__ T fromf(float x) {
    return mbr::from_f32<T>(x);
}

template <int OP>
__device__ __forceinline__ float bin(float x, float y) {
    if constexpr (OP == BIN_ADD) return x + y;
    else if constexpr (OP == BIN_SUB) return x - y;
    else if constexpr (OP == BIN_MUL) return x * y;
    else return x / y;
}
template <int OP>
__device__ __forceinline__ float un(float x, float p0, float p1) {
    if constexpr (OP == UN_ADD_SCALAR) return x + p0;
    else if constexpr (OP == UN_MUL_SCALAR) return x * p0;
    else if constexpr (OP == UN_CLAMP) return fminf(fmaxf(x, p0), p1);
    else if constexpr (OP == UN_NEG) return -x;
    else return x > p0 ? 1.0f : 0.0f;  // UN_GT
}

#define GRID_STRIDE(i, n) for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); \
                               i += (int64_t)gridDim.x * blockDim.x)

// Two independent 8-element vectors in flight per thread per step: units
// i and i + stride of the grid-stride loop.
#define VEC_LOOP(n8, ...)                                                              \
    do {                                                                               \
        const int64_t stride_ = (int64_t)gridDim.x * blockDim.x;                       \
        int64_t i_ = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;                   \
        for (; i_ + stride_ < (n8); i_ += 2 * stride_) {                               \
            { const int64_t u = i_; __VA_ARGS__; }                                     \
            { const int64_t u = i_ + stride_; __VA_ARGS__; }                           \
        }                                                                              \
        if (i_ < (n8)) { const int64_t u = i_; __VA_ARGS__; }                          \
    } while (0)

// Unit u of the vector loops is the 8 elements one lane moves per step.  A
// warp's 32 consecutive units form one 256-element block: for 16-bit types
// lane l takes elements 8l .. 8l+7 (one 16-byte access); for fp32 it takes
// 4l .. 4l+3 and 128+4l .. 128+4l+3, so each of its two 16-byte accesses is a
// fully used 512-byte run across the warp (two 32-byte halves of every sector
// coming from different instructions would leave sectors partly written).  The
// fp32 units past the last whole block keep 8 contiguous elements.
template <typename T>
__device__ __forceinline__ int64_t unit_elem(int64_t u, int64_t full_units, int half) {
    if constexpr (sizeof(T) == 4) {
        if (u < full_units) return 256 * (u >> 5) + 4 * (u & 31) + 128 * half;
    }
    return 8 * u + 4 * half;
}
template <typename T>
__device__ __forceinline__ void load_unit(const T* p, int64_t u, int64_t full_units, float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p + unit_elem<T>(u, full_units, 0)));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p + unit_elem<T>(u, full_units, 1)));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        load8(p + 8 * u, v);
    }
}
template <typename T>
__device__ __forceinline__ void store_unit(T* p, int64_t u, int64_t full_units, const float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(p + unit_elem<T>(u, full_units, 0)) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(p + unit_elem<T>(u, full_units, 1)) = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        store8(p + 8 * u, v);
    }
}
// the [D] broadcast operand's values for unit u (D % 8 == 0): element e uses b[e % D]
template <typename T>
__device__ __forceinline__ void load_unit_bcast(const T* b, int64_t u, int64_t full_units, int64_t D, bool m32,
                                                float (&v)[8]) {
    auto col = [&](int64_t e) { return m32 ? (int64_t)((uint32_t)e % (uint32_t)D) : e % D; };
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(b + col(unit_elem<T>(u, full_units, 0))));
        const float4 c = __ldg(reinterpret_cast<const float4*>(b + col(unit_elem<T>(u, full_units, 1))));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = c.x, v[5] = c.y, v[6] = c.z, v[7] = c.w;
    } else {
        load8(b + col(8 * u), v);
    }
}

// y = convert(a), contiguous (S == D: a vector copy).  The units of source and
// destination must cover the same elements: fp32 on either side uses the fp32
// layout for both.
template <typename S, typename D>
__global__ void __launch_bounds__(256) cvt_vec_kernel(const S* __restrict__ a, D* __restrict__ y, int64_t n) {
    const int64_t n8 = n >> 3, full = 32 * (n >> 8);
    using L = std::conditional_t<sizeof(S) == 4 || sizeof(D) == 4, float, S>;  // unit layout
    VEC_LOOP(n8, {
        float v[8];
        if constexpr (sizeof(L) == 4 && sizeof(S) != 4) {  // 16-bit source, fp32 layout: 8-byte loads
            const int64_t e0 = unit_elem<L>(u, full, 0), e1 = unit_elem<L>(u, full, 1);
            const uint2 q0 = __ldg(reinterpret_cast<const uint2*>(a + e0));
            const uint2 q1 = __ldg(reinterpret_cast<const uint2*>(a + e1));
            const S* h0 = reinterpret_cast<const S*>(&q0);
            const S* h1 = reinterpret_cast<const S*>(&q1);
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = tof(h0[k]), v[4 + k] = tof(h1[k]);
        } else {
            load_unit(a, u, full, v);
        }
        if constexpr (sizeof(L) == 4 && sizeof(D) != 4) {  // 16-bit destination, fp32 layout
            const int64_t e0 = unit_elem<L>(u, full, 0), e1 = unit_elem<L>(u, full, 1);
            D o0[4], o1[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) o0[k] = fromf<D>(v[k]), o1[k] = fromf<D>(v[4 + k]);
            *reinterpret_cast<uint2*>(y + e0) = *reinterpret_cast<uint2*>(o0);
            *reinterpret_cast<uint2*>(y + e1) = *reinterpret_cast<uint2*>(o1);
        } else {
            store_unit(y, u, full, v);
        }
    });
    if (blockIdx.x == 0 && threadIdx.x < (n & 7)) {
        const int64_t i = 8 * n8 + threadIdx.x;
        y[i] = fromf<D>(tof(a[i]));
    }
}

template <typename T>
__global__ void __launch_bounds__(256) fill_vec_kernel(T* __restrict__ y, int64_t n, float val) {
    const int64_t n8 = n >> 3, full = 32 * (n >> 8);
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = val;
    VEC_LOOP(n8, store_unit(y, u, full, v));
    if (blockIdx.x == 0 && threadIdx.x < (n & 7)) y[8 * n8 + threadIdx.x] = fromf<T>(val);
}

template <typename T, int OP>
__global__ void __launch_bounds__(256) unary_vec_kernel(const T* __restrict__ a, T* __restrict__ y, int64_t n,
                                                        float p0, float p1) {
    const int64_t n8 = n >> 3, full = 32 * (n >> 8);
    VEC_LOOP(n8, {
        float v[8];
        load_unit(a, u, full, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = un<OP>(v[k], p0, p1);
        store_unit(y, u, full, v);
    });
    if (blockIdx.x == 0 && threadIdx.x < (n & 7)) {
        const int64_t i = 8 * n8 + threadIdx.x;
        y[i] = fromf<T>(un<OP>(tof(a[i]), p0, p1));
    }
}

// y = a (op) b, a and y contiguous [n]; BM 0: b contiguous [n]; 1: b [D]
// broadcast over rows (D % 8 == 0); 2: b a scalar.
template <typename T, int OP, int BM>
__global__ void __launch_bounds__(256) binary_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                         T* __restrict__ y, int64_t n, int64_t D) {
    const int64_t n8 = n >> 3, full = 32 * (n >> 8);
    const bool m32 = n < ((int64_t)1 << 32);  // 32-bit column arithmetic
    const float bs = BM == 2 ? tof(b[0]) : 0.f;
    VEC_LOOP(n8, {
        float v[8], w[8];
        load_unit(a, u, full, v);
        if constexpr (BM == 0) load_unit(b, u, full, w);
        else if constexpr (BM == 1) load_unit_bcast(b, u, full, D, m32, w);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = bin<OP>(v[k], BM == 2 ? bs : w[k]);
        store_unit(y, u, full, v);
    });
    if (blockIdx.x == 0 && threadIdx.x < (n & 7)) {
        const int64_t i = 8 * n8 + threadIdx.x;
        const float bv = BM == 0 ? tof(b[i]) : BM == 1 ? tof(b[i % D]) : bs;
        y[i] = fromf<T>(bin<OP>(tof(a[i]), bv));
    }
}

// ---- 16-byte units of the reductions: 16 / sizeof(T) elements, kept raw
// (4 registers) until they are folded into fp32 accumulators ----
template <int OP>
__device__ __forceinline__ float red(float a, float b) {
    return OP == RED_MAX ? fmaxf(a, b) : a + b;
}
template <typename T, int OP>
__device__ __forceinline__ float fold16(const uint4& u) {
    if constexpr (sizeof(T) == 4) {
        const float* f = reinterpret_cast<const float*>(&u);
        return red<OP>(red<OP>(f[0], f[1]), red<OP>(f[2], f[3]));
    } else {
        float2 p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, __half>::value) p[i] = __half22float2(reinterpret_cast<const __half2*>(&u)[i]);
            else p[i] = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&u)[i]);
        }
        return red<OP>(red<OP>(red<OP>(p[0].x, p[0].y), red<OP>(p[1].x, p[1].y)),
                       red<OP>(red<OP>(p[2].x, p[2].y), red<OP>(p[3].x, p[3].y)));
    }
}
// per-element fold of one unit into VE column accumulators
template <typename T, int OP>
__device__ __forceinline__ void fold16_cols(const uint4& u, float (&acc)[16 / sizeof(T)]) {
    if constexpr (sizeof(T) == 4) {
        const float* f = reinterpret_cast<const float*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = red<OP>(acc[e], f[e]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 p;
            if constexpr (std::is_same<T, __half>::value) p = __half22float2(reinterpret_cast<const __half2*>(&u)[i]);
            else p = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&u)[i]);
            acc[2 * i] = red<OP>(acc[2 * i], p.x);
            acc[2 * i + 1] = red<OP>(acc[2 * i + 1], p.y);
        }
    }
}

// out[r] = reduce(src[r][0..len)), contiguous rows whose length is a whole
// number of 16-byte units (16-byte aligned).  A warp takes 8 consecutive rows
// per step and each lane loads one 16-byte unit of each of them, so 8 loads
// are in flight per lane even for the short rows (192 to 512 elements) of the
// activations; the raw units stay in 4 registers each until folded, which
// keeps enough warps resident.  The 8 row sums leave the warp through a
// reduce-scatter butterfly (4 + 2 + 1 + 1 + 1 shuffles instead of 8 x 5):
// after it, lanes 4q .. 4q+3 hold row q's total.
template <typename T, int OP>
__global__ void __launch_bounds__(256, 4) reduce_rows_kernel(const T* __restrict__ src, T* __restrict__ out,
                                                             int64_t rows, int64_t len) {
    constexpr int R = 8, VE = 16 / (int)sizeof(T);
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t units = len / VE;
    const uint4* s = reinterpret_cast<const uint4*>(src);
    const float init = OP == RED_MAX ? -INFINITY : 0.f;
    for (int64_t r0 = warp0 * R; r0 < rows; r0 += nwarps * R) {
        float acc[R];
#pragma unroll
        for (int q = 0; q < R; ++q) acc[q] = init;
        for (int64_t k = lane; k < units; k += 32) {
            uint4 raw[R];
#pragma unroll
            for (int q = 0; q < R; ++q)
                if (r0 + q < rows) raw[q] = __ldcs(s + (r0 + q) * units + k);
#pragma unroll
            for (int q = 0; q < R; ++q)
                if (r0 + q < rows) acc[q] = red<OP>(acc[q], fold16<T, OP>(raw[q]));
        }
        // reduce-scatter: each stage halves the rows a lane carries
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool hi = lane & 16;
            const float send = hi ? acc[i] : acc[i + 4], keep = hi ? acc[i + 4] : acc[i];
            acc[i] = red<OP>(keep, __shfl_xor_sync(0xffffffffu, send, 16));
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool hi = lane & 8;
            const float send = hi ? acc[i] : acc[i + 2], keep = hi ? acc[i + 2] : acc[i];
            acc[i] = red<OP>(keep, __shfl_xor_sync(0xffffffffu, send, 8));
        }
        {
            const bool hi = lane & 4;
            const float send = hi ? acc[0] : acc[1], keep = hi ? acc[1] : acc[0];
            acc[0] = red<OP>(keep, __shfl_xor_sync(0xffffffffu, send, 4));
        }
        acc[0] = red<OP>(acc[0], __shfl_xor_sync(0xffffffffu, acc[0], 2));
        acc[0] = red<OP>(acc[0], __shfl_xor_sync(0xffffffffu, acc[0], 1));
        const int q = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        if ((lane & 3) == 0 && r0 + q < rows) out[r0 + q] = fromf<T>(OP == RED_MEAN ? acc[0] / (float)len : acc[0]);
    }
}

// Rows of any length or alignment: one warp per row, scalar loads.
template <typename T, int OP>
__global__ void __launch_bounds__(256) reduce_rows_scalar_kernel(const T* __restrict__ src, T* __restrict__ out,
                                                                 int64_t rows, int64_t len) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp0; r < rows; r += nwarps) {
        float acc = OP == RED_MAX ? -INFINITY : 0.f;
        for (int64_t q = lane; q < len; q += 32) {
            const float v = tof(src[r * len + q]);
            acc = OP == RED_MAX ? fmaxf(acc, v) : acc + v;
        }
        acc = OP == RED_MAX ? mbr::warp_max(acc) : mbr::warp_sum(acc);
        if (lane == 0) out[r] = fromf<T>(OP == RED_MEAN ? acc / (float)len : acc);
    }
}

// Column partials of a contiguous [len][n] (n a whole number of 16-byte
// units, 16-byte aligned): CTA (bx, by) covers the W = 32 units' columns
// [W bx, W bx + W) (256 columns for 16-bit types, 128 for fp32), each lane
// one unit's columns, over rows by, by + gridDim.y, ... split among its 8
// warps with 16 rows' units in flight per lane; the warps' partials are
// combined in shared memory into part[by][col].
template <typename T, int OP>
__global__ void __launch_bounds__(256, 2) reduce_cols_partial_kernel(const T* __restrict__ src,
                                                                     float* __restrict__ part, int64_t len,
                                                                     int64_t n) {
    constexpr int VE = 16 / (int)sizeof(T), W = 32 * VE, U = 16;
    __shared__ float sm[8][W];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t c0 = (int64_t)blockIdx.x * W + VE * lane;
    const float init = OP == RED_MAX ? -INFINITY : 0.f;
    float acc[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) acc[e] = init;
    if (c0 < n) {
        const int64_t step = (int64_t)gridDim.y * 8, nu = n / VE;
        const uint4* col = reinterpret_cast<const uint4*>(src + c0);
        int64_t r = (int64_t)blockIdx.y * 8 + w;
        for (; r + (U - 1) * step < len; r += U * step) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) raw[u] = __ldcs(col + (r + u * step) * nu);
#pragma unroll
            for (int u = 0; u < U; ++u) fold16_cols<T, OP>(raw[u], acc);
        }
        for (; r < len; r += step) fold16_cols<T, OP>(__ldcs(col + r * nu), acc);
    }
#pragma unroll
    for (int e = 0; e < VE; ++e) sm[w][VE * lane + e] = acc[e];
    __syncthreads();
    for (int c = threadIdx.x; c < W; c += 256) {
        float a = sm[0][c];
#pragma unroll
        for (int k = 1; k < 8; ++k) a = red<OP>(a, sm[k][c]);
        const int64_t gc = (int64_t)blockIdx.x * W + c;
        if (gc < n) part[(int64_t)blockIdx.y * n + gc] = a;
    }
}
// part [splits][n] -> out [n]: CTA of 256 threads per 32 columns, its 8 warps
// summing interleaved subsets of the splits (four loads in flight per lane),
// combined in shared memory.
template <typename T, int OP>
__global__ void __launch_bounds__(256) reduce_cols_final_kernel(const float* __restrict__ part, T* __restrict__ out,
                                                                int splits, int64_t len, int64_t n) {
    __shared__ float sm[8][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t c = (int64_t)blockIdx.x * 32 + lane;
    const float init = OP == RED_MAX ? -INFINITY : 0.f;
    float a4[4] = {init, init, init, init};
    if (c < n) {
        int k = w;
        for (; k + 24 < splits; k += 32) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = part[(int64_t)(k + 8 * u) * n + c];
#pragma unroll
            for (int u = 0; u < 4; ++u) a4[u] = red<OP>(a4[u], v[u]);
        }
        for (; k < splits; k += 8) a4[0] = red<OP>(a4[0], part[(int64_t)k * n + c]);
    }
    float acc = red<OP>(red<OP>(a4[0], a4[1]), red<OP>(a4[2], a4[3]));
    sm[w][lane] = acc;
    __syncthreads();
    if (w == 0 && c < n) {
#pragma unroll
        for (int k = 1; k < 8; ++k) acc = OP == RED_MAX ? fmaxf(acc, sm[k][lane]) : acc + sm[k][lane];
        out[c] = fromf<T>(OP == RED_MEAN ? acc / (float)len : acc);
    }
}

// dst[c][r] = src[r][c]: the contiguous copy of a transposed 2-D view
// (source element (i, j) at src[j * ld_src + i]), through 32 x 32 shared-memory
// tiles so both the reads and the writes are coalesced.
template <typename E>
__global__ void __launch_bounds__(256) transpose2d_kernel(const E* __restrict__ src, E* __restrict__ dst,
                                                          int64_t rows, int64_t cols) {
    // dst is [rows][cols] (rows = the view's dim 0); src holds it as [cols][rows]
    __shared__ E tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int64_t tb = blockIdx.x; tb < ((rows + 31) / 32) * ((cols + 31) / 32); tb += gridDim.x) {
        const int64_t tr = tb / ((cols + 31) / 32), tc = tb % ((cols + 31) / 32);
        const int64_t r0 = tr * 32, c0 = tc * 32;
        // read: source rows are the view's columns; lanes along the view's rows (contiguous in src)
#pragma unroll
        for (int k = ty; k < 32; k += 8) {
            const int64_t c = c0 + k, r = r0 + tx;
            if (c < cols && r < rows) tile[k][tx] = src[c * rows + r];
        }
        __syncthreads();
#pragma unroll
        for (int k = ty; k < 32; k += 8) {
            const int64_t r = r0 + k, c = c0 + tx;
            if (r < rows && c < cols) dst[r * cols + c] = tile[tx][k];
        }
        __syncthreads();
    }
}

// The same copy for 4-byte elements through 64 x 64 tiles: each thread has
// 16 loads in flight (a 32 x 32 tile gives 4, too few bytes in flight per SM
// to cover HBM latency).
__global__ void __launch_bounds__(256) transpose64_u32_kernel(const uint32_t* __restrict__ src,
                                                              uint32_t* __restrict__ dst, int64_t rows, int64_t cols) {
    __shared__ uint32_t tile[64][65];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t tcn = (cols + 63) / 64, ntiles = ((rows + 63) / 64) * tcn;
    for (int64_t tb = blockIdx.x; tb < ntiles; tb += gridDim.x) {
        const int64_t r0 = (tb / tcn) * 64, c0 = (tb % tcn) * 64;
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int k = ty + 8 * (i >> 1), x = tx + 32 * (i & 1);
            const int64_t c = c0 + k, r = r0 + x;
            v[i] = (c < cols && r < rows) ? __ldcs(src + c * rows + r) : 0u;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) tile[ty + 8 * (i >> 1)][tx + 32 * (i & 1)] = v[i];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int k = ty + 8 * (i >> 1), x = tx + 32 * (i & 1);
            const int64_t r = r0 + k, c = c0 + x;
            if (r < rows && c < cols) __stcs(dst + r * cols + c, tile[x][k]);
        }
        __syncthreads();
    }
}

// 16-bit elements with even rows and cols, moved as 32-bit pairs.  Source
// words A = src[2p][2q .. 2q+1] and B = src[2p+1][2q .. 2q+1] (two
// neighbouring source rows) give the destination words dst[2q][2p .. 2p+1] =
// (A.lo, B.lo) and dst[2q+1][2p .. 2p+1] = (A.hi, B.hi), so every global
// access is a full 4-byte word and a warp moves 128 contiguous bytes.  A tile
// is 32 p x 64 q (64 source rows x 128 source columns); each thread has 16
// loads in flight.
__global__ void __launch_bounds__(256) transpose_pairs16_kernel(const uint32_t* __restrict__ src,
                                                                uint32_t* __restrict__ dst, int64_t rows,
                                                                int64_t cols) {
    __shared__ uint32_t lo[32][65], hi[32][65];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t np = cols / 2, nq = rows / 2;  // words per dst row, words per src row
    const int64_t tpn = (np + 31) / 32, ntiles = ((nq + 63) / 64) * tpn;
    for (int64_t tb = blockIdx.x; tb < ntiles; tb += gridDim.x) {
        const int64_t q0 = (tb / tpn) * 64, p0 = (tb % tpn) * 32;
        uint32_t a[8], b[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int pl = ty + 8 * (i >> 1), ql = tx + 32 * (i & 1);
            const int64_t p = p0 + pl, q = q0 + ql;
            const bool ok = p < np && q < nq;
            a[i] = ok ? __ldcs(src + (2 * p) * nq + q) : 0u;
            b[i] = ok ? __ldcs(src + (2 * p + 1) * nq + q) : 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int pl = ty + 8 * (i >> 1), ql = tx + 32 * (i & 1);
            lo[pl][ql] = __byte_perm(a[i], b[i], 0x5410);
            hi[pl][ql] = __byte_perm(a[i], b[i], 0x7632);
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int ql = ty + 8 * j;
            const int64_t q = q0 + ql, p = p0 + tx;
            if (q < nq && p < np) {
                __stcs(dst + (2 * q) * np + p, lo[tx][ql]);
                __stcs(dst + (2 * q + 1) * np + p, hi[tx][ql]);
            }
        }
        __syncthreads();
    }
}

// ---- generic strided kernels ----
template <typename I>
__global__ void copy_kernel(Geo g, const void* src, int sdt, void* dst, int ddt, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t os, od, unused;
        offsets<I>(g, (I)i, os, od, unused);
        if (sdt == ddt) {
            switch (sdt) {
                case F32: ((float*)dst)[od] = ((const float*)src)[os]; break;
                case I64: ((int64_t*)dst)[od] = ((const int64_t*)src)[os]; break;
                default: ((uint16_t*)dst)[od] = ((const uint16_t*)src)[os]; break;
            }
        } else {
            stf(dst, ddt, od, ldf(src, sdt, os));
        }
    }
}

template <typename I>
__global__ void fill_kernel(Geo g, void* dst, int dt, double v, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t od, u1, u2;
        offsets<I>(g, (I)i, od, u1, u2);
        if (dt == I64) ((int64_t*)dst)[od] = (int64_t)v;
        else stf(dst, dt, od, (float)v);
    }
}

template <typename I>
__global__ void binary_kernel(Geo g, int op, const void* a, int adt, const void* b, int bdt, void* out, int odt,
                              int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t oa, ob, oo;
        offsets<I>(g, (I)i, oa, ob, oo);
        // fp32 arithmetic (the reference computes its elementwise ops in fp32)
        const float x = ldf(a, adt, oa), y = ldf(b, bdt, ob);
        float r;
        switch (op) {
            case BIN_ADD: r = x + y; break;
            case BIN_SUB: r = x - y; break;
            case BIN_MUL: r = x * y; break;
            default: r = x / y; break;
        }
        stf(out, odt, oo, r);
    }
}

template <typename I>
__global__ void unary_kernel(Geo g, int op, const void* a, int adt, void* out, int odt, float p0, float p1,
                             int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t oa, oo, u;
        offsets<I>(g, (I)i, oa, oo, u);
        const float x = ldf(a, adt, oa);
        float r;
        switch (op) {
            case UN_ADD_SCALAR: r = x + p0; break;
            case UN_MUL_SCALAR: r = x * p0; break;
            case UN_CLAMP: r = fminf(fmaxf(x, p0), p1); break;
            case UN_NEG: r = -x; break;
            default: r = x > p0 ? 1.0f : 0.0f; break;  // UN_GT
        }
        stf(out, odt, oo, r);
    }
}

// One thread per output element; the reduced dim is walked with its stride.
template <typename I>
__global__ void reduce_kernel(Geo g, int op, const void* src, int sdt, int64_t len, int64_t rstride, void* out,
                              int odt, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t os, oo, u;
        offsets<I>(g, (I)i, os, oo, u);
        float acc = op == RED_MAX ? -INFINITY : 0.f;
        for (int64_t k = 0; k < len; ++k) {
            const float v = ldf(src, sdt, os + k * rstride);
            acc = op == RED_MAX ? fmaxf(acc, v) : acc + v;
        }
        if (op == RED_MEAN) acc /= (float)len;
        stf(out, odt, oo, acc);
    }
}

__global__ void pad_reflect_kernel(const void* src, int dt, int64_t L, int64_t left, int64_t Lo, void* dst,
                                   int64_t n) {
    GRID_STRIDE(i, n) {
        const int64_t r = i / Lo, q = i % Lo;
        const int64_t p = mbr::reflect_idx(q - left, L);
        if (dt == F32) ((float*)dst)[i] = ((const float*)src)[r * L + p];
        else if (dt == I64) ((int64_t*)dst)[i] = ((const int64_t*)src)[r * L + p];
        else ((uint16_t*)dst)[i] = ((const uint16_t*)src)[r * L + p];
    }
}

__global__ void index_select_kernel(const void* src, int dt, int64_t dsrc, int64_t inner, const int64_t* idx,
                                    int64_t nidx, void* dst, int64_t n, int* bad) {
    GRID_STRIDE(i, n) {
        const int64_t in = i % inner;
        const int64_t j = (i / inner) % nidx;
        const int64_t o = i / (inner * nidx);
        int64_t k = idx[j];
        if (k < 0) k += dsrc;
        if (k < 0 || k >= dsrc) {
            *bad = 1;
            continue;
        }
        const int64_t s = (o * dsrc + k) * inner + in;
        if (dt == F32) ((float*)dst)[i] = ((const float*)src)[s];
        else if (dt == I64) ((int64_t*)dst)[i] = ((const int64_t*)src)[s];
        else ((uint16_t*)dst)[i] = ((const uint16_t*)src)[s];
    }
}

__global__ void arange_kernel(void* dst, int dt, int64_t start, int64_t n) {
    GRID_STRIDE(i, n) {
        if (dt == I64) ((int64_t*)dst)[i] = start + i;
        else stf(dst, dt, i, (float)(start + i));
    }
}

// ---- host-side classification and dispatch ----
int sm_count() {
    static int n = [] {
        int dev = 0, v = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}
// grid of the generic kernels: one element per thread, at most 32 CTAs per SM
unsigned grid(int64_t n) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 32));
}
// grid of the vector kernels (256 threads, two 8-element units per thread
// per step): enough CTAs to fill every SM several times over
unsigned vgrid(int64_t n8) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n8 + 511) / 512, (int64_t)sm_count() * 8));
}

bool is_contig(int nd, const int64_t* shape, const int64_t* st) {
    int64_t e = 1;
    for (int d = nd - 1; d >= 0; --d) {
        if (shape[d] != 1 && st[d] != e) return false;
        e *= shape[d];
    }
    return true;
}
// b is a [D] vector along the last dim broadcast over all other dims
bool is_row_bcast(int nd, const int64_t* shape, const int64_t* st) {
    if (nd < 1 || st[nd - 1] != 1) return false;
    for (int d = 0; d < nd - 1; ++d)
        if (shape[d] != 1 && st[d] != 0) return false;
    return true;
}
bool is_scalar_bcast(int nd, const int64_t* shape, const int64_t* st) {
    for (int d = 0; d < nd; ++d)
        if (shape[d] != 1 && st[d] != 0) return false;
    return true;
}
bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }
bool fits32(int64_t n, int nd, const int64_t* shape) {
    (void)shape;
    (void)nd;
    return n < (int64_t)1 << 31;
}

// Calls f with the C++ type of a floating dtype (f32 / f16 / bf16); false for i64.
template <class F>
bool with_float_type(int dt, F&& f) {
    switch (dt) {
        case F32: f((float*)nullptr); return true;
        case F16: f((__half*)nullptr); return true;
        case BF16: f((__nv_bfloat16*)nullptr); return true;
        default: return false;
    }
}

}  // namespace

void copy(const void* src, int sdt, const int64_t* sstride, void* dst, int ddt, const int64_t* dstride, int nd,
          const int64_t* shape, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    if (is_contig(nd, shape, sstride) && is_contig(nd, shape, dstride) && aligned16(src) && aligned16(dst) &&
        sdt != I64 && ddt != I64) {
        with_float_type(sdt, [&](auto* s) {
            using S = std::remove_pointer_t<decltype(s)>;
            with_float_type(ddt, [&](auto* d) {
                using D = std::remove_pointer_t<decltype(d)>;
                cvt_vec_kernel<S, D><<<vgrid(n >> 3), 256, 0, st>>>((const S*)src, (D*)dst, n);
            });
        });
        MBR_CUDA(cudaGetLastError());
        return;
    }
    // the contiguous copy of a transposed 2-D view: tiled through shared memory
    {
        int64_t sh2[2], ss2[2];
        int k = 0;
        for (int d = 0; d < nd && k <= 2; ++d)
            if (shape[d] != 1) {
                if (k < 2) sh2[k] = shape[d], ss2[k] = sstride[d];
                ++k;
            }
        if (k == 2 && sdt == ddt && ss2[0] == 1 && ss2[1] == sh2[0] && is_contig(nd, shape, dstride)) {
            const int64_t tiles = ((sh2[0] + 31) / 32) * ((sh2[1] + 31) / 32);
            const unsigned gr = (unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sm_count() * 16));
            const auto grid_for = [&](int64_t t) {
                return (unsigned)std::max<int64_t>(1, std::min<int64_t>(t, (int64_t)sm_count() * 8));
            };
            const bool words = ((uintptr_t)src & 3) == 0 && ((uintptr_t)dst & 3) == 0;
            if (sdt == F32)
                transpose64_u32_kernel<<<grid_for(((sh2[0] + 63) / 64) * ((sh2[1] + 63) / 64)), 256, 0, st>>>(
                    (const uint32_t*)src, (uint32_t*)dst, sh2[0], sh2[1]);
            else if (sdt != I64 && words && sh2[0] % 2 == 0 && sh2[1] % 2 == 0)
                transpose_pairs16_kernel<<<grid_for(((sh2[0] / 2 + 63) / 64) * ((sh2[1] / 2 + 31) / 32)), 256, 0,
                                           st>>>((const uint32_t*)src, (uint32_t*)dst, sh2[0], sh2[1]);
            else if (sdt == I64)
                transpose2d_kernel<int64_t><<<gr, 256, 0, st>>>((const int64_t*)src, (int64_t*)dst, sh2[0], sh2[1]);
            else
                transpose2d_kernel<uint16_t><<<gr, 256, 0, st>>>((const uint16_t*)src, (uint16_t*)dst, sh2[0], sh2[1]);
            MBR_CUDA(cudaGetLastError());
            return;
        }
    }
    const Geo g = make_geo(nd, shape, sstride, dstride, nullptr);
    if (fits32(n, nd, shape)) copy_kernel<uint32_t><<<grid(n), 256, 0, st>>>(g, src, sdt, dst, ddt, n);
    else copy_kernel<uint64_t><<<grid(n), 256, 0, st>>>(g, src, sdt, dst, ddt, n);
    MBR_CUDA(cudaGetLastError());
}

void fill(void* dst, int dt, const int64_t* stride, int nd, const int64_t* shape, int64_t n, double v,
          cudaStream_t st) {
    if (n <= 0) return;
    if (is_contig(nd, shape, stride) && aligned16(dst) &&
        with_float_type(dt, [&](auto* t) {
            using T = std::remove_pointer_t<decltype(t)>;
            fill_vec_kernel<T><<<vgrid(n >> 3), 256, 0, st>>>((T*)dst, n, (float)v);
        })) {
        MBR_CUDA(cudaGetLastError());
        return;
    }
    const Geo g = make_geo(nd, shape, stride, nullptr, nullptr);
    if (fits32(n, nd, shape)) fill_kernel<uint32_t><<<grid(n), 256, 0, st>>>(g, dst, dt, v, n);
    else fill_kernel<uint64_t><<<grid(n), 256, 0, st>>>(g, dst, dt, v, n);
    MBR_CUDA(cudaGetLastError());
}

void binary(int op, const void* a, int adt, const int64_t* sa, const void* b, int bdt, const int64_t* sb, void* out,
            int odt, const int64_t* so, int nd, const int64_t* shape, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    if (adt == bdt && adt == odt && is_contig(nd, shape, sa) && is_contig(nd, shape, so) && aligned16(a) &&
        aligned16(out) && op >= BIN_ADD && op <= BIN_DIV) {
        int bm = -1;
        const int64_t D = nd > 0 ? shape[nd - 1] : 1;
        if (is_contig(nd, shape, sb) && aligned16(b)) bm = 0;
        else if (is_scalar_bcast(nd, shape, sb)) bm = 2;
        else if (is_row_bcast(nd, shape, sb) && D % 8 == 0 && aligned16(b)) bm = 1;
        if (bm >= 0 && with_float_type(adt, [&](auto* t) {
                using T = std::remove_pointer_t<decltype(t)>;
                const T* A = (const T*)a;
                const T* B = (const T*)b;
                T* Y = (T*)out;
                const unsigned gr = vgrid(n >> 3);
                auto go = [&](auto opc) {
                    constexpr int OP = decltype(opc)::value;
                    if (bm == 0) binary_vec_kernel<T, OP, 0><<<gr, 256, 0, st>>>(A, B, Y, n, D);
                    else if (bm == 1) binary_vec_kernel<T, OP, 1><<<gr, 256, 0, st>>>(A, B, Y, n, D);
                    else binary_vec_kernel<T, OP, 2><<<gr, 256, 0, st>>>(A, B, Y, n, D);
                };
                switch (op) {
                    case BIN_ADD: go(std::integral_constant<int, BIN_ADD>()); break;
                    case BIN_SUB: go(std::integral_constant<int, BIN_SUB>()); break;
                    case BIN_MUL: go(std::integral_constant<int, BIN_MUL>()); break;
                    default: go(std::integral_constant<int, BIN_DIV>()); break;
                }
            })) {
            MBR_CUDA(cudaGetLastError());
            return;
        }
    }
    const Geo g = make_geo(nd, shape, sa, sb, so);
    if (fits32(n, nd, shape)) binary_kernel<uint32_t><<<grid(n), 256, 0, st>>>(g, op, a, adt, b, bdt, out, odt, n);
    else binary_kernel<uint64_t><<<grid(n), 256, 0, st>>>(g, op, a, adt, b, bdt, out, odt, n);
    MBR_CUDA(cudaGetLastError());
}

void unary(int op, const void* a, int adt, const int64_t* sa, void* out, int odt, const int64_t* so, int nd,
           const int64_t* shape, int64_t n, float p0, float p1, cudaStream_t st) {
    if (n <= 0) return;
    if (adt == odt && is_contig(nd, shape, sa) && is_contig(nd, shape, so) && aligned16(a) && aligned16(out) &&
        with_float_type(adt, [&](auto* t) {
            using T = std::remove_pointer_t<decltype(t)>;
            const T* A = (const T*)a;
            T* Y = (T*)out;
            const unsigned gr = vgrid(n >> 3);
            switch (op) {
                case UN_ADD_SCALAR: unary_vec_kernel<T, UN_ADD_SCALAR><<<gr, 256, 0, st>>>(A, Y, n, p0, p1); break;
                case UN_MUL_SCALAR: unary_vec_kernel<T, UN_MUL_SCALAR><<<gr, 256, 0, st>>>(A, Y, n, p0, p1); break;
                case UN_CLAMP: unary_vec_kernel<T, UN_CLAMP><<<gr, 256, 0, st>>>(A, Y, n, p0, p1); break;
                case UN_NEG: unary_vec_kernel<T, UN_NEG><<<gr, 256, 0, st>>>(A, Y, n, p0, p1); break;
                default: unary_vec_kernel<T, UN_GT><<<gr, 256, 0, st>>>(A, Y, n, p0, p1); break;
            }
        })) {
        MBR_CUDA(cudaGetLastError());
        return;
    }
    const Geo g = make_geo(nd, shape, sa, so, nullptr);
    if (fits32(n, nd, shape)) unary_kernel<uint32_t><<<grid(n), 256, 0, st>>>(g, op, a, adt, out, odt, p0, p1, n);
    else unary_kernel<uint64_t><<<grid(n), 256, 0, st>>>(g, op, a, adt, out, odt, p0, p1, n);
    MBR_CUDA(cudaGetLastError());
}

void reduce(int op, const void* src, int sdt, const int64_t* s_outer, int nd, const int64_t* outer_shape,
            int64_t n_outer, int64_t len, int64_t rstride, void* out, int odt, cudaStream_t st) {
    if (n_outer <= 0) return;
    std::vector<int64_t> so(nd);
    int64_t acc = 1;
    for (int d = nd - 1; d >= 0; --d) {
        so[d] = acc;
        acc *= outer_shape[d];
    }
    // rows of `len` contiguous elements laid one after another: warp per row
    std::vector<int64_t> row_st(nd);
    for (int d = 0; d < nd; ++d) row_st[d] = so[d] * len;
    if (rstride == 1 && sdt == odt &&
        [&] {
            for (int d = 0; d < nd; ++d)
                if (outer_shape[d] != 1 && s_outer[d] != row_st[d]) return false;
            return true;
        }() &&
        with_float_type(sdt, [&](auto* t) {
            using T = std::remove_pointer_t<decltype(t)>;
            const bool vec = aligned16(src) && len % 8 == 0;
            const unsigned gr = (unsigned)std::max<int64_t>(
                1, std::min<int64_t>((n_outer + 31) / 32, (int64_t)sm_count() * 16));
            auto go = [&](auto opc) {
                constexpr int OP = decltype(opc)::value;
                if (vec) reduce_rows_kernel<T, OP><<<gr, 256, 0, st>>>((const T*)src, (T*)out, n_outer, len);
                else reduce_rows_scalar_kernel<T, OP><<<gr, 256, 0, st>>>((const T*)src, (T*)out, n_outer, len);
            };
            if (op == RED_SUM) go(std::integral_constant<int, RED_SUM>());
            else if (op == RED_MEAN) go(std::integral_constant<int, RED_MEAN>());
            else go(std::integral_constant<int, RED_MAX>());
        })) {
        MBR_CUDA(cudaGetLastError());
        return;
    }
    // leading dim of a contiguous [len][n_outer]: column partials over CTAs
    if (nd == 1 && s_outer[0] == 1 && rstride == n_outer && sdt == odt && n_outer < (int64_t)sm_count() * 1024 &&
        len >= 64 && n_outer % 8 == 0 && aligned16(src) &&
        with_float_type(sdt, [&](auto* t) {
            using T = std::remove_pointer_t<decltype(t)>;
            const int64_t bx = (n_outer + 32 * (16 / (int64_t)sizeof(T)) - 1) / (32 * (16 / (int64_t)sizeof(T)));
            // two CTAs per SM (each warp then has 16 rows' loads in flight per
            // step, enough to cover HBM latency) and at least 16 rows per warp,
            // so the second pass sums few partials
            const int splits = (int)std::max<int64_t>(1, std::min<int64_t>((len + 127) / 128,
                                                                            (sm_count() * 2 + bx - 1) / bx));
            float* part = (float*)CudaMemoryPool::instance().allocate(sizeof(float) * (size_t)splits * n_outer, st);
            const dim3 g1((unsigned)bx, (unsigned)splits);
            auto go = [&](auto opc) {
                constexpr int OP = decltype(opc)::value;
                reduce_cols_partial_kernel<T, OP><<<g1, 256, 0, st>>>((const T*)src, part, len, n_outer);
                reduce_cols_final_kernel<T, OP><<<(unsigned)((n_outer + 31) / 32), 256, 0, st>>>(part, (T*)out, splits,
                                                                                              len, n_outer);
            };
            if (op == RED_SUM) go(std::integral_constant<int, RED_SUM>());
            else if (op == RED_MEAN) go(std::integral_constant<int, RED_MEAN>());
            else go(std::integral_constant<int, RED_MAX>());
            CudaMemoryPool::instance().deallocate(part, st);  // reusable in stream order
        })) {
        MBR_CUDA(cudaGetLastError());
        return;
    }
    const Geo g = make_geo(nd, outer_shape, s_outer, so.data(), nullptr);
    if (fits32(n_outer, nd, outer_shape))
        reduce_kernel<uint32_t><<<grid(n_outer), 256, 0, st>>>(g, op, src, sdt, len, rstride, out, odt, n_outer);
    else
        reduce_kernel<uint64_t><<<grid(n_outer), 256, 0, st>>>(g, op, src, sdt, len, rstride, out, odt, n_outer);
    MBR_CUDA(cudaGetLastError());
}

void pad_reflect(const void* src, int dt, int64_t outer, int64_t L, int64_t left, int64_t right, void* dst,
                 cudaStream_t st) {
    const int64_t Lo = L + left + right, n = outer * Lo;
    if (n <= 0) return;
    pad_reflect_kernel<<<grid(n), 256, 0, st>>>(src, dt, L, left, Lo, dst, n);
    MBR_CUDA(cudaGetLastError());
}

void index_select(const void* src, int dt, int64_t outer, int64_t dsrc, int64_t inner, const int64_t* idx,
                  int64_t nidx, void* dst, int* d_bad, cudaStream_t st) {
    const int64_t n = outer * nidx * inner;
    if (n <= 0) return;
    index_select_kernel<<<grid(n), 256, 0, st>>>(src, dt, dsrc, inner, idx, nidx, dst, n, d_bad);
    MBR_CUDA(cudaGetLastError());
}

void arange(void* dst, int dt, int64_t start, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    arange_kernel<<<grid(n), 256, 0, st>>>(dst, dt, start, n);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace tk
}  // namespace cudasep
