// tensor_kernels.h — launchers of the generic strided Tensor kernels.
// dtype codes: 0 f32, 1 f16, 2 i64, 3 bf16 (cudasep::DType).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

namespace cudasep {
namespace tk {

constexpr int kMaxDims = 8;
enum BinOp { BIN_ADD = 0, BIN_SUB, BIN_MUL, BIN_DIV };
enum UnOp { UN_ADD_SCALAR = 0, UN_MUL_SCALAR, UN_CLAMP, UN_NEG, UN_GT };
enum RedOp { RED_SUM = 0, RED_MEAN, RED_MAX };

// Element-wise copy over `shape` from a strided source to a strided
// destination with dtype conversion (bit copy when the dtypes match).
void copy(const void* src, int sdt, const int64_t* sstride, void* dst, int ddt, const int64_t* dstride, int nd,
          const int64_t* shape, int64_t n, cudaStream_t st);
void fill(void* dst, int dt, const int64_t* stride, int nd, const int64_t* shape, int64_t n, double v,
          cudaStream_t st);
// out = a (op) b with broadcast strides (0 on broadcast dims).
void binary(int op, const void* a, int adt, const int64_t* sa, const void* b, int bdt, const int64_t* sb, void* out,
            int odt, const int64_t* so, int nd, const int64_t* shape, int64_t n, cudaStream_t st);
void unary(int op, const void* a, int adt, const int64_t* sa, void* out, int odt, const int64_t* so, int nd,
           const int64_t* shape, int64_t n, float p0, float p1, cudaStream_t st);
// out (contiguous over outer_shape) = reduce over `len` elements at `rstride`.
void reduce(int op, const void* src, int sdt, const int64_t* s_outer, int nd, const int64_t* outer_shape,
            int64_t n_outer, int64_t len, int64_t rstride, void* out, int odt, cudaStream_t st);
// contiguous [outer][L] -> [outer][left + L + right], reflect (no edge repeat).
void pad_reflect(const void* src, int dt, int64_t outer, int64_t L, int64_t left, int64_t right, void* dst,
                 cudaStream_t st);
// contiguous [outer][dsrc][inner] -> [outer][nidx][inner] (idx on the device; *d_bad set on a bad index).
void index_select(const void* src, int dt, int64_t outer, int64_t dsrc, int64_t inner, const int64_t* idx,
                  int64_t nidx, void* dst, int* d_bad, cudaStream_t st);
void arange(void* dst, int dt, int64_t start, int64_t n, cudaStream_t st);

}  // namespace tk
}  // namespace cudasep
