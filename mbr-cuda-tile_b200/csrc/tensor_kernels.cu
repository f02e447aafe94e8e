// tensor_kernels.cu — generic strided kernels behind the Tensor API: copy /
// dtype conversion, fill, broadcast binary ops, scalar ops, reductions over
// one dim, reflect padding, index_select, arange.  Shapes and strides travel
// by value in the launch parameters (the reference uploads them with a
// blocking cudaMemcpy per call, src/tensor_cuda_glue.cu:47-55), so no op
// synchronises the host.
#include "common.cuh"
#include "tensor_kernels.h"

namespace cudasep {
namespace tk {

namespace {

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

__device__ __forceinline__ void offsets(const Geo& g, int64_t lin, int64_t& o0, int64_t& o1, int64_t& o2) {
    o0 = o1 = o2 = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
        const int64_t i = lin % g.shape[d];
        lin /= g.shape[d];
        o0 += i * g.s[0][d];
        o1 += i * g.s[1][d];
        o2 += i * g.s[2][d];
    }
}

__device__ __forceinline__ double ld(const void* p, int dt, int64_t off) {
    switch (dt) {
        case 0: return ((const float*)p)[off];
        case 1: return __half2float(((const __half*)p)[off]);
        case 2: return (double)((const int64_t*)p)[off];
        default: return __bfloat162float(((const __nv_bfloat16*)p)[off]);
    }
}

__device__ __forceinline__ void st(void* p, int dt, int64_t off, double v) {
    switch (dt) {
        case 0: ((float*)p)[off] = (float)v; break;
        case 1: ((__half*)p)[off] = __float2half_rn((float)v); break;
        case 2: ((int64_t*)p)[off] = (int64_t)v; break;
        default: ((__nv_bfloat16*)p)[off] = __float2bfloat16_rn((float)v); break;
    }
}

#define GRID_STRIDE(i, n) for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n); \
                               i += (int64_t)gridDim.x * blockDim.x)

__global__ void copy_kernel(Geo g, const void* src, int sdt, void* dst, int ddt, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t os, od, unused;
        offsets(g, i, os, od, unused);
        if (sdt == ddt) {
            switch (sdt) {
                case 0: ((float*)dst)[od] = ((const float*)src)[os]; break;
                case 2: ((int64_t*)dst)[od] = ((const int64_t*)src)[os]; break;
                default: ((uint16_t*)dst)[od] = ((const uint16_t*)src)[os]; break;
            }
        } else {
            st(dst, ddt, od, ld(src, sdt, os));
        }
    }
}

__global__ void fill_kernel(Geo g, void* dst, int dt, double v, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t od, u1, u2;
        offsets(g, i, od, u1, u2);
        st(dst, dt, od, v);
    }
}

__global__ void binary_kernel(Geo g, int op, const void* a, int adt, const void* b, int bdt, void* out, int odt,
                              int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t oa, ob, oo;
        offsets(g, i, oa, ob, oo);
        // fp32 arithmetic (the reference computes its elementwise ops in fp32)
        const float x = (float)ld(a, adt, oa), y = (float)ld(b, bdt, ob);
        float r;
        switch (op) {
            case BIN_ADD: r = x + y; break;
            case BIN_SUB: r = x - y; break;
            case BIN_MUL: r = x * y; break;
            default: r = x / y; break;
        }
        st(out, odt, oo, r);
    }
}

__global__ void unary_kernel(Geo g, int op, const void* a, int adt, void* out, int odt, float p0, float p1,
                             int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t oa, oo, u;
        offsets(g, i, oa, oo, u);
        const float x = (float)ld(a, adt, oa);
        float r;
        switch (op) {
            case UN_ADD_SCALAR: r = x + p0; break;
            case UN_MUL_SCALAR: r = x * p0; break;
            case UN_CLAMP: r = fminf(fmaxf(x, p0), p1); break;
            case UN_NEG: r = -x; break;
            default: r = x > p0 ? 1.0f : 0.0f; break;  // UN_GT
        }
        st(out, odt, oo, r);
    }
}

// One thread per output element; the reduced dim is walked with its stride.
__global__ void reduce_kernel(Geo g, int op, const void* src, int sdt, int64_t len, int64_t rstride, void* out,
                              int odt, int64_t n) {
    GRID_STRIDE(i, n) {
        int64_t os, oo, u;
        offsets(g, i, os, oo, u);
        float acc = op == RED_MAX ? -INFINITY : 0.f;
        for (int64_t k = 0; k < len; ++k) {
            const float v = (float)ld(src, sdt, os + k * rstride);
            acc = op == RED_MAX ? fmaxf(acc, v) : acc + v;
        }
        if (op == RED_MEAN) acc /= (float)len;
        st(out, odt, oo, acc);
    }
}

__global__ void pad_reflect_kernel(const void* src, int dt, int64_t L, int64_t left, int64_t Lo, void* dst,
                                   int64_t n) {
    GRID_STRIDE(i, n) {
        const int64_t r = i / Lo, q = i % Lo;
        const int64_t p = mbr::reflect_idx(q - left, L);
        if (dt == 0) ((float*)dst)[i] = ((const float*)src)[r * L + p];
        else if (dt == 2) ((int64_t*)dst)[i] = ((const int64_t*)src)[r * L + p];
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
        if (dt == 0) ((float*)dst)[i] = ((const float*)src)[s];
        else if (dt == 2) ((int64_t*)dst)[i] = ((const int64_t*)src)[s];
        else ((uint16_t*)dst)[i] = ((const uint16_t*)src)[s];
    }
}

__global__ void arange_kernel(void* dst, int dt, int64_t start, int64_t n) {
    GRID_STRIDE(i, n) st(dst, dt, i, (double)(start + i));
}

unsigned grid(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32)); }

}  // namespace

void copy(const void* src, int sdt, const int64_t* sstride, void* dst, int ddt, const int64_t* dstride, int nd,
          const int64_t* shape, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    copy_kernel<<<grid(n), 256, 0, st>>>(make_geo(nd, shape, sstride, dstride, nullptr), src, sdt, dst, ddt, n);
    MBR_CUDA(cudaGetLastError());
}

void fill(void* dst, int dt, const int64_t* stride, int nd, const int64_t* shape, int64_t n, double v,
          cudaStream_t st) {
    if (n <= 0) return;
    fill_kernel<<<grid(n), 256, 0, st>>>(make_geo(nd, shape, stride, nullptr, nullptr), dst, dt, v, n);
    MBR_CUDA(cudaGetLastError());
}

void binary(int op, const void* a, int adt, const int64_t* sa, const void* b, int bdt, const int64_t* sb, void* out,
            int odt, const int64_t* so, int nd, const int64_t* shape, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    binary_kernel<<<grid(n), 256, 0, st>>>(make_geo(nd, shape, sa, sb, so), op, a, adt, b, bdt, out, odt, n);
    MBR_CUDA(cudaGetLastError());
}

void unary(int op, const void* a, int adt, const int64_t* sa, void* out, int odt, const int64_t* so, int nd,
           const int64_t* shape, int64_t n, float p0, float p1, cudaStream_t st) {
    if (n <= 0) return;
    unary_kernel<<<grid(n), 256, 0, st>>>(make_geo(nd, shape, sa, so, nullptr), op, a, adt, out, odt, p0, p1, n);
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
    reduce_kernel<<<grid(n_outer), 256, 0, st>>>(make_geo(nd, outer_shape, s_outer, so.data(), nullptr), op, src,
                                                 sdt, len, rstride, out, odt, n_outer);
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
