// gemm_simt.cu — grouped GEMM on the CUDA cores (fp32 FMA, fp32 accumulate)
// with the forward's fused epilogues.  It is the fp32 compute path (the fp32
// tolerance rules out TF32 tensor cores) and the reference implementation the
// tcgen05 kernel is checked against.
#include "common.cuh"
#include "ops.h"

namespace mbr {
namespace ops {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <typename T, int EPI>
__device__ __forceinline__ void epi_store(const GemmGroup& g, int m, int n, float acc) {
    if (g.bias) acc += g.bias[n];
    if constexpr (EPI == EPI_F32) {
        ((float*)g.C)[(int64_t)m * g.ldc + n] = acc;
    } else if constexpr (EPI == EPI_T) {
        ((T*)g.C)[(int64_t)m * g.ldc + n] = from_f32<T>(acc);
    } else if constexpr (EPI == EPI_ADD_F32) {
        float* c = (float*)g.C + (int64_t)m * g.ldc + n;
        *c += acc;
    } else if constexpr (EPI == EPI_GELU_T) {
        ((T*)g.C)[(int64_t)m * g.ldc + n] = from_f32<T>(gelu_erf(acc));
    } else if constexpr (EPI == EPI_TANH_T) {
        ((T*)g.C)[(int64_t)m * g.ldc + n] = from_f32<T>(tanhf(acc));
    }
}

template <typename T, int EPI>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const GemmGroup* __restrict__ groups) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const GemmGroup g = groups[blockIdx.z];
    int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (m0 >= g.M || n0 >= g.N) return;
    const T* A = (const T*)g.A;
    const T* B = (const T*)g.B;
    int tid = threadIdx.x;
    int ty = tid / 16, tx = tid % 16;
    float acc[4][4] = {};
    int lr = tid / 4, lk = (tid % 4) * 4;  // loader: 64 rows x 16 k, 4 per thread
    for (int k0 = 0; k0 < g.K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int kk = k0 + lk + i;
            int am = m0 + lr, bn = n0 + lr;
            As[lk + i][lr] = (am < g.M && kk < g.K) ? to_f32(A[(int64_t)am * g.lda + kk]) : 0.f;
            Bs[lk + i][lr] = (bn < g.N && kk < g.K) ? to_f32(B[(int64_t)bn * g.ldb + kk]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int m = m0 + ty * 4 + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int n = n0 + tx * 4 + j;
            if constexpr (EPI == EPI_GLU_F32) {
                if ((j & 1) == 0 && n + 1 < g.N) {
                    float a = acc[i][j] + (g.bias ? g.bias[n] : 0.f);
                    float b = acc[i][j + 1] + (g.bias ? g.bias[n + 1] : 0.f);
                    ((float*)g.C)[(int64_t)m * g.ldc + n / 2] = a / (1.0f + expf(-b));
                }
            } else {
                if (n < g.N) epi_store<T, EPI>(g, m, n, acc[i][j]);
            }
        }
    }
}

template <typename T>
void launch(const GemmGroup* d_groups, int ngroups, int maxM, int maxN, int epi, cudaStream_t st) {
    dim3 grid((unsigned)ceil_div(maxN, BN), (unsigned)ceil_div(maxM, BM), (unsigned)ngroups);
    switch (epi) {
        case EPI_F32: gemm_simt_kernel<T, EPI_F32><<<grid, 256, 0, st>>>(d_groups); break;
        case EPI_T: gemm_simt_kernel<T, EPI_T><<<grid, 256, 0, st>>>(d_groups); break;
        case EPI_ADD_F32: gemm_simt_kernel<T, EPI_ADD_F32><<<grid, 256, 0, st>>>(d_groups); break;
        case EPI_GELU_T: gemm_simt_kernel<T, EPI_GELU_T><<<grid, 256, 0, st>>>(d_groups); break;
        case EPI_TANH_T: gemm_simt_kernel<T, EPI_TANH_T><<<grid, 256, 0, st>>>(d_groups); break;
        case EPI_GLU_F32: gemm_simt_kernel<T, EPI_GLU_F32><<<grid, 256, 0, st>>>(d_groups); break;
        default: throw Error(ERR_INVALID, "gemm: bad epilogue");
    }
}

}  // namespace

void gemm_simt(const GemmGroup* d_groups, int ngroups, int maxM, int maxN, int dtype, int epi, cudaStream_t st) {
    if (ngroups <= 0 || maxM <= 0 || maxN <= 0) return;
    MBR_DISPATCH_DTYPE(dtype, T, { launch<T>(d_groups, ngroups, maxM, maxN, epi, st); });
    MBR_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace mbr
