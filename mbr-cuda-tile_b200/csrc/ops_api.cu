// ops_api.cu — stand-alone tensor ops of the reference op library (mbr_tile /
// stft_tile, reference layouts) for drop-in callers and the op sweep:
// RMSNorm+gamma, residual add, GELU, sigmoid-gate multiply, RoPE, band gather,
// mask scatter-average, STFT and iSTFT.  Memory-bound kernels: 16-byte
// vectorised, coalesced, one pass over HBM, reductions in registers.
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"
#include "ops_api.h"
#include "attention_tc.h"
#include "ffn_tc.h"
#include "gemm_tc.h"
#include "ops.h"

namespace mbr {
namespace opsapi {

namespace {

constexpr int kFft = 2048;
constexpr int kBins = kFft / 2 + 1;

inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        MBR_CUDA(cudaGetDevice(&dev));
        MBR_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    }
    return n;
}

// 8 elements of T in their storage form: one 16-byte word (16-bit T) or two
// (fp32), so a load in flight holds 4 or 8 registers until it is unpacked.
template <typename T>
struct Raw8 {
    static constexpr int N = sizeof(T) / 2;
    uint4 w[N];
    __device__ __forceinline__ void load(const T* p) {
#pragma unroll
        for (int i = 0; i < N; ++i) w[i] = reinterpret_cast<const uint4*>(p)[i];
    }
};

// 8 elements of T as floats through one 16-byte (16-bit T) or two (fp32) accesses.
template <typename T>
struct Vec8 {
    float v[8];
    __device__ __forceinline__ void set(const Raw8<T>& r) {
        if constexpr (sizeof(T) == 4) {
            const float4 a = *reinterpret_cast<const float4*>(&r.w[0]), b = *reinterpret_cast<const float4*>(&r.w[1]);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
            const uint32_t u[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = pair_to_f32<T>(u[i]);
                v[2 * i] = f.x, v[2 * i + 1] = f.y;
            }
        }
    }
    __device__ __forceinline__ void load(const T* p) {
        Raw8<T> r;
        r.load(p);
        set(r);
    }
    __device__ __forceinline__ void store(T* p) const {
        if constexpr (sizeof(T) == 4) {
            reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint4 u;
            T* e = reinterpret_cast<T*>(&u);
#pragma unroll
            for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
            *reinterpret_cast<uint4*>(p) = u;
        }
    }
};

// ---- residual add / GELU / gate (n % 8 == 0, grid-stride) ----
// Each thread keeps kEwU 8-element vectors in flight (64 bytes of loads per
// input), the vectors of one step spaced a whole grid apart so every warp
// access stays a contiguous 512-byte (16-bit) or 1024-byte (fp32) run.
template <typename T>
constexpr int ew_unroll() {
    return sizeof(T) == 4 ? 2 : 4;
}

template <typename T>
__global__ void __launch_bounds__(256) add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                                                  int64_t n8) {
    constexpr int U = ew_unroll<T>();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n8; i0 += U * stride) {
        Raw8<T> ra[U], rb[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < n8) {
                ra[u].load(a + 8 * (i0 + u * stride));
                rb[u].load(b + 8 * (i0 + u * stride));
            }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < n8) {
                Vec8<T> x, z;
                x.set(ra[u]);
                z.set(rb[u]);
#pragma unroll
                for (int k = 0; k < 8; ++k) x.v[k] += z.v[k];
                x.store(y + 8 * (i0 + u * stride));
            }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) gelu_kernel(const T* __restrict__ a, T* __restrict__ y, int64_t n8) {
    constexpr int U = ew_unroll<T>();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n8; i0 += U * stride) {
        Raw8<T> ra[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < n8) ra[u].load(a + 8 * (i0 + u * stride));
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < n8) {
                Vec8<T> x;
                x.set(ra[u]);
                gelu_tail(x.v);  // the reference's 0.5 x (1 + erf(x)), one exponential per element
                x.store(y + 8 * (i0 + u * stride));
            }
    }
}

// y[r][h*dh + d] = x[r][h*dh + d] * g[r][h]   (dh % 8 == 0)
template <typename T>
__global__ void __launch_bounds__(256) gate_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                                   T* __restrict__ y, int64_t rows, int H, int dh) {
    constexpr int U = ew_unroll<T>();
    const unsigned per_row = (unsigned)(H * dh / 8), dh8 = (unsigned)(dh / 8);
    const int64_t n8 = rows * per_row;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n8; i0 += U * stride) {
        Raw8<T> ra[U];
        float gv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < n8) {
                // 32-bit index arithmetic (n8 < 2^32 checked on the host)
                const unsigned r = (unsigned)i / per_row;
                const int h = (int)(((unsigned)i - r * per_row) / dh8);
                gv[u] = to_f32(g[(int64_t)r * H + h]);
                ra[u].load(x + 8 * i);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * stride < n8) {
                Vec8<T> a;
                a.set(ra[u]);
#pragma unroll
                for (int k = 0; k < 8; ++k) a.v[k] *= gv[u];
                a.store(y + 8 * (i0 + u * stride));
            }
    }
}

// RMSNorm over groups of R consecutive rows read as one flat run of R*D/8
// 8-element chunks (R*D/8 = 32*NC): lane l owns chunks l + 32 i (i < NC) of
// every group, so all 32 lanes carry data for any D the grouping fits, the
// lane's gamma chunks are the same for every group (loaded once), and a warp
// has NC 16-byte (16-bit) or 32-byte (fp32) loads in flight per group.
template <typename T, int R, int NC>
__global__ void __launch_bounds__(256) rms_group_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                        T* __restrict__ y, int64_t rows, int D, float scale) {
    __shared__ __align__(16) float gs[1024];
    const int lane = threadIdx.x & 31, D8 = D / 8;
    for (int k = threadIdx.x; k < D; k += blockDim.x) gs[k] = gamma[k];
    __syncthreads();
    int rq[NC], gc[NC];  // row within the group and gamma offset of the lane's chunks
#pragma unroll
    for (int i = 0; i < NC; ++i) {
        const int c = lane + 32 * i;
        rq[i] = c / D8;
        gc[i] = 8 * (c - rq[i] * D8);
    }
    const int64_t groups = (rows + R - 1) / R;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t grp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); grp < groups; grp += warps) {
        const int64_t r0 = grp * R;
        const int nrows = rows - r0 < R ? (int)(rows - r0) : R;
        const T* xg = x + r0 * D;
        Raw8<T> raw[NC];
#pragma unroll
        for (int i = 0; i < NC; ++i)
            if (rq[i] < nrows) raw[i].load(xg + 8 * (lane + 32 * i));
        float ss[R];
#pragma unroll
        for (int r = 0; r < R; ++r) ss[r] = 0.f;
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            float p = 0.f;
            if (rq[i] < nrows) {
                Vec8<T> v;
                v.set(raw[i]);
#pragma unroll
                for (int k = 0; k < 8; ++k) p += v.v[k] * v.v[k];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) ss[r] += rq[i] == r ? p : 0.f;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) ss[r] = rsqrtf(warp_sum(ss[r]) + 1e-12f) * scale;
        T* yg = y + r0 * D;
#pragma unroll
        for (int i = 0; i < NC; ++i)
            if (rq[i] < nrows) {
                float inv = ss[0];
#pragma unroll
                for (int r = 1; r < R; ++r) inv = rq[i] == r ? ss[r] : inv;
                Vec8<T> v;
                v.set(raw[i]);
                const float4 g0 = *reinterpret_cast<const float4*>(gs + gc[i]);
                const float4 g1 = *reinterpret_cast<const float4*>(gs + gc[i] + 4);
                const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) v.v[k] *= inv * g[k];
                v.store(yg + 8 * (lane + 32 * i));
            }
    }
}

// RMSNorm with gamma, dtype in / dtype out; D % 8 == 0, D <= 1024.  A warp
// normalises two rows at a time (both rows' loads in flight together).
template <typename T, int MAXC>
__global__ void __launch_bounds__(256) rms_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                  T* __restrict__ y, int64_t rows, int D, float scale) {
    const int lane = threadIdx.x & 31, D8 = D / 8;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r0 = 2 * ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); r0 < rows;
         r0 += 2 * warps) {
        const bool two = r0 + 1 < rows;
        Vec8<T> v[2][MAXC];
        float ss[2] = {0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int64_t r = two ? r0 + q : r0;
#pragma unroll
            for (int i = 0; i < MAXC; ++i) {
                const int c = lane + 32 * i;
                if (c < D8) {
                    v[q][i].load(x + r * D + 8 * c);
#pragma unroll
                    for (int k = 0; k < 8; ++k) ss[q] += v[q][i].v[k] * v[q][i].v[k];
                }
            }
        }
        ss[0] = warp_sum(ss[0]);
        ss[1] = warp_sum(ss[1]);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            if (q == 1 && !two) break;
            const float inv = rsqrtf(ss[q] + 1e-12f) * scale;
#pragma unroll
            for (int i = 0; i < MAXC; ++i) {
                const int c = lane + 32 * i;
                if (c < D8) {
                    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c);
                    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * c + 1);
                    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) v[q][i].v[k] *= inv * g[k];
                    v[q][i].store(y + (r0 + q) * D + 8 * c);
                }
            }
        }
    }
}

// RoPE over positions: x [seqs][L][H][64]; pair (2i, 2i+1) of every head at
// position p rotated by (cos, sin)[p][i].
template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const T* __restrict__ x, const float* __restrict__ cs,
                                                   const float* __restrict__ sn, T* __restrict__ y, int64_t seqs,
                                                   int L, int H) {
    constexpr int U = ew_unroll<T>();
    const int64_t n8 = seqs * L * H * 8;  // 8 chunks of 8 per 64-wide head
    const unsigned hh = (unsigned)(8 * H), ll = (unsigned)L;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n8; i0 += U * stride) {
        Raw8<T> ra[U];
        float4 c4[U], s4[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < n8) {
                const int chunk = (int)(i & 7);
                const int p = (int)(((unsigned)i / hh) % ll);  // 32-bit (n8 < 2^32 checked on the host)
                ra[u].load(x + 8 * i);
                // pairs 4*chunk .. 4*chunk+3 of position p: one 16-byte load of each table
                c4[u] = __ldg(reinterpret_cast<const float4*>(cs + p * 32) + chunk);
                s4[u] = __ldg(reinterpret_cast<const float4*>(sn + p * 32) + chunk);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (i0 + u * stride >= n8) continue;
            const float cc[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w}, ss[4] = {s4[u].x, s4[u].y, s4[u].z, s4[u].w};
            Vec8<T> a;
            a.set(ra[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float x0 = a.v[2 * k], x1 = a.v[2 * k + 1];
                a.v[2 * k] = x0 * cc[k] - x1 * ss[k];
                a.v[2 * k + 1] = x0 * ss[k] + x1 * cc[k];
            }
            a.store(y + 8 * (i0 + u * stride));
        }
    }
}

// Band gather (gather_freqs_fold_complex with the stereo merge folded in):
// spec [B][C][F][T] complex -> x[b][t][2j + r] = spec[b][fi_j % C][fi_j / C][t][r].
// One CTA per (frequency-range tile, 32 frames, b): the tile's spectrum rows
// come in as 256-byte runs of frames, and the tile's band-freq entries go out
// as runs of consecutive j per frame, so both sides are coalesced and every
// element moves once.  Each lane owns entries lane + 32 i of the tile (their
// j and tile row held in registers) and each warp writes whole frames, so the
// output loop is a shared-memory read and a store per element.  The tile's
// tables sit at fixed per-tile offsets, so every global load of the prologue
// is independent of the others.
constexpr int kTT = 32;      // frames per band-op CTA
constexpr int kBandEnt = 4;  // tile entries held per lane per pass (128 per warp)
constexpr int kBandWarps = 8;
constexpr int kBandRows = 2 * kBandTileBins / kBandWarps;  // tile rows per warp
constexpr int kBandFrames = kTT / kBandWarps;              // frames per warp

template <typename T>
__global__ void __launch_bounds__(kBandWarps * 32) gather_tiled_kernel(
    const float2* __restrict__ spec, int C, int F, int Tn, const int* __restrict__ jl, const int* __restrict__ jr,
    int stride, int64_t J, T* __restrict__ x) {
    __shared__ __align__(16) float2 tile[2 * kBandTileBins][kTT + 1];  // [c * nf + f - f0][tt], C <= 2
    const int f0 = blockIdx.x * kBandTileBins, nf = min(kBandTileBins, F - f0);
    const int b = blockIdx.z, t0 = blockIdx.y * kTT, nt = min(kTT, Tn - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int* jlt = jl + (int64_t)blockIdx.x * stride;
    const int* jrt = jr + (int64_t)blockIdx.x * stride;
    const float2* sp = spec + ((int64_t)b * C * F + f0) * Tn + t0 + lane;  // row (c, f0) of this lane's frame
#pragma unroll
    for (int i = 0; i < kBandRows; ++i) {
        const int row = warp + kBandWarps * i, c = row >= nf;  // C <= 2
        if (row < C * nf && lane < nt) cp_async<8>(&tile[row][lane], sp + (c * (F - nf) + row) * Tn);
    }
    const float2* tflat = &tile[0][0];
    for (int base = 0; base < stride; base += 32 * kBandEnt) {
        int jj[kBandEnt], rr[kBandEnt];
#pragma unroll
        for (int i = 0; i < kBandEnt; ++i) {
            const int k = base + lane + 32 * i;
            jj[i] = k < stride ? jlt[k] : -1;
            rr[i] = k < stride ? jrt[k] * (kTT + 1) : 0;  // flat offset of the entry's tile row
        }
        if (base == 0) {
            cp_async_wait_all();
            __syncthreads();
        }
#pragma unroll
        for (int u = 0; u < kBandFrames; ++u) {
            const int tt = warp + kBandWarps * u;
            if (tt >= nt) break;
            T* dst = x + ((int64_t)b * Tn + t0 + tt) * 2 * J;
#pragma unroll
            for (int i = 0; i < kBandEnt; ++i)
                if (jj[i] >= 0) store_pair(dst + 2 * jj[i], tflat[rr[i] + tt]);
        }
    }
}

// Mask scatter-average (apply_mask_and_scatter, gather form):
// out[b][s][c][f][t] = sum_{j: fi_j = f*C+c} spec[b][c][f][t] * mask[s][b*T+t][j] / nbpf[f*C+c]
// (each term scaled by 1 / nbpf before the sum; the reference divides each term before its atomic add).
// One CTA per (frequency-range tile, 32 frames, b, s).  Everything the CTA
// reads is copied into shared memory with asynchronous copies issued up front
// (the tile's spectrum rows, bin weights and entry tables, then the masks of
// the tile's entries as runs of consecutive j per frame), so a CTA waits for
// memory about twice; then each warp produces its (channel, bin) rows of the
// tile as 32-frame runs.
template <typename T>
__global__ void __launch_bounds__(kBandWarps * 32) scatter_tiled_kernel(
    const float2* __restrict__ spec, const T* __restrict__ masks, int B, int S, int C, int F, int Tn,
    const int* __restrict__ jl, const int* __restrict__ bk, const int* __restrict__ bo, int stride,
    const float* __restrict__ nbpf, int64_t J, float2* __restrict__ out) {
    using P = typename PairOf<T>::type;
    extern __shared__ __align__(16) uint8_t band_smem[];
    // [2 * kBandTileBins][kTT + 1] spectrum tile, [kTT][stride + 1] masks (odd pitch: conflict-free
    // frame-strided reads), row offsets, grouped entries, per-row bin weights
    auto xs = reinterpret_cast<float2 (*)[kTT + 1]>(band_smem);
    P* mk = reinterpret_cast<P*>(band_smem + sizeof(float2) * 2 * kBandTileBins * (kTT + 1));
    const int ld = stride + 1;
    int* bos = reinterpret_cast<int*>(mk + kTT * ld);  // [kBandRowOffs]
    int* bks = bos + kBandRowOffs;                     // [stride]
    float* nbs = reinterpret_cast<float*>(bks + stride);  // [2 * kBandTileBins]
    const int f0 = blockIdx.x * kBandTileBins, nf = min(kBandTileBins, F - f0);
    const int t0 = blockIdx.y * kTT, nt = min(kTT, Tn - t0);
    const int b = blockIdx.z % B, s = blockIdx.z / B;
    const int rows = C * nf;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float2* sp = spec + ((int64_t)b * C * F + f0) * Tn + t0 + lane;  // row (c, f0) of this lane's frame
#pragma unroll
    for (int i = 0; i < kBandRows; ++i) {
        const int row = warp + kBandWarps * i, c = row >= nf;  // C <= 2
        if (row < rows && lane < nt) cp_async<8>(&xs[row][lane], sp + (c * (F - nf) + row) * Tn);
    }
    for (int k = threadIdx.x; k < kBandRowOffs; k += blockDim.x)
        cp_async<4>(&bos[k], &bo[(int64_t)blockIdx.x * kBandRowOffs + k]);
    for (int k = threadIdx.x; k < stride; k += blockDim.x) cp_async<4>(&bks[k], &bk[(int64_t)blockIdx.x * stride + k]);
    for (int k = threadIdx.x; k < rows; k += blockDim.x) {
        const int c = k >= nf;
        cp_async<4>(&nbs[k], &nbpf[(f0 + k - c * nf) * C + c]);
    }
    const int* jlt = jl + (int64_t)blockIdx.x * stride;
    const T* mrow = masks + ((int64_t)s * B * Tn + (int64_t)b * Tn + t0) * 2 * J;
    const int jstride = (int)(2 * J);
    for (int base = 0; base < stride; base += 32 * kBandEnt) {
        int jj[kBandEnt];
#pragma unroll
        for (int i = 0; i < kBandEnt; ++i) {
            const int k = base + lane + 32 * i;
            jj[i] = k < stride ? jlt[k] : -1;
        }
#pragma unroll
        for (int u = 0; u < kBandFrames; ++u) {
            const int tt = warp + kBandWarps * u;
            if (tt >= nt) break;
#pragma unroll
            for (int i = 0; i < kBandEnt; ++i)
                if (jj[i] >= 0)
                    cp_async<sizeof(P)>(&mk[tt * ld + base + lane + 32 * i], mrow + tt * jstride + 2 * jj[i]);
        }
    }
    cp_async_wait_all();
    __syncthreads();
    if (lane >= nt) return;
    float2* op = out + (((int64_t)b * S + s) * C * F + f0) * Tn + t0 + lane;
    const P* mkl = mk + lane * ld;
#pragma unroll
    for (int i = 0; i < kBandRows; ++i) {
        const int row = warp + kBandWarps * i, c = row >= nf;
        if (row >= rows) break;
        const float2 xv = xs[row][lane];
        const float den = fmaxf(nbs[row], 1e-8f);
        float2 acc = make_float2(0.f, 0.f);
        const int q0 = bos[row], q1 = bos[row + 1];
        // each term times the row's correctly rounded reciprocal: exact for
        // power-of-two weights, within about one ulp of the quotient otherwise,
        // and one division per row instead of two per term
        const float inv = 1.f / den;
        for (int q = q0; q < q1; ++q) {
            const float2 mm = pair_to_f32<T>(mkl[bks[q]]);
            acc.x += (xv.x * mm.x - xv.y * mm.y) * inv;
            acc.y += (xv.x * mm.y + xv.y * mm.x) * inv;
        }
        op[(c * (F - nf) + row) * Tn] = acc;
    }
}

// ---- STFT / iSTFT in the reference layout ([n][F][T][2]) ----
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ int bitrev11(int n) { return (int)(__brev((unsigned)n) >> 21); }

__device__ void fft2048(float2* buf, const float2* tw, bool inverse) {
    for (int len = 2; len <= kFft; len <<= 1) {
        const int half = len >> 1, ts = kFft / len;
        __syncthreads();
        for (int bi = threadIdx.x; bi < kFft / 2; bi += blockDim.x) {
            const int grp = bi / half, k = bi % half;
            const int i0 = grp * len + k, i1 = i0 + half;
            float2 w = tw[k * ts];
            if (inverse) w.y = -w.y;
            const float2 a = buf[i0], b = cmul(buf[i1], w);
            buf[i0] = make_float2(a.x + b.x, a.y + b.y);
            buf[i1] = make_float2(a.x - b.x, a.y - b.y);
        }
    }
    __syncthreads();
}

// Periodic Hann window and FFT twiddles evaluated in the kernel (no tables).
__device__ __forceinline__ float hann(int n) { return 0.5f * (1.0f - cospif((float)n / (kFft / 2))); }
__device__ __forceinline__ void load_twiddles(float2* tw) {
    for (int k = threadIdx.x; k < kFft / 2; k += blockDim.x) {
        float s, c;
        sincospif(-(float)k / (kFft / 2), &s, &c);
        tw[k] = make_float2(c, s);
    }
}

__global__ void __launch_bounds__(512) stft_ref_kernel(const float* __restrict__ sig, int64_t L, int hop,
                                                       float2* __restrict__ out, int Tn) {
    __shared__ float2 tw[kFft / 2];
    __shared__ float2 buf[kFft];
    const int64_t n = blockIdx.y;
    const int t = blockIdx.x;
    load_twiddles(tw);
    for (int i = threadIdx.x; i < kFft; i += blockDim.x) {
        const int64_t p = reflect_idx((int64_t)t * hop + i - kFft / 2, L);
        buf[bitrev11(i)] = make_float2(sig[n * L + p] * hann(i), 0.f);
    }
    fft2048(buf, tw, false);
    for (int f = threadIdx.x; f < kBins; f += blockDim.x) out[(n * kBins + f) * Tn + t] = buf[f];
}

__global__ void __launch_bounds__(512) istft_frames_ref_kernel(const float2* __restrict__ spec, int Tn,
                                                               float* __restrict__ frames) {
    __shared__ float2 tw[kFft / 2];
    __shared__ float2 buf[kFft];
    const int64_t n = blockIdx.y;
    const int t = blockIdx.x;
    load_twiddles(tw);
    for (int i = threadIdx.x; i < kFft; i += blockDim.x) {
        float2 v;
        if (i < kBins) {
            v = spec[(n * kBins + i) * Tn + t];
        } else {
            v = spec[(n * kBins + (kFft - i)) * Tn + t];
            v.y = -v.y;
        }
        buf[bitrev11(i)] = v;
    }
    fft2048(buf, tw, true);
    float* o = frames + (n * Tn + t) * kFft;
    for (int i = threadIdx.x; i < kFft; i += blockDim.x) o[i] = buf[i].x * (1.0f / kFft) * hann(i);
}

__global__ void istft_ola_ref_kernel(const float* __restrict__ frames, int64_t nsig, int Tn, int hop, int64_t lout,
                                     float* __restrict__ out) {
    const int64_t total = nsig * lout;
    const int64_t full = (int64_t)(Tn - 1) * hop;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = idx / lout, q = idx % lout;
        float val = 0.f;
        if (q < full) {
            const int64_t p = q + kFft / 2;
            const int64_t tmin = p - (kFft - 1) <= 0 ? 0 : (p - (kFft - 1) + hop - 1) / hop;
            const int64_t tmax = min((int64_t)Tn - 1, p / hop);
            float acc = 0.f, ws = 0.f;
            for (int64_t t = tmin; t <= tmax; ++t) {
                const int k = (int)(p - t * hop);
                const float w = hann(k);
                acc += frames[(o * Tn + t) * kFft + k];
                ws += w * w;
            }
            val = ws > 1e-8f ? acc / ws : acc;
        }
        out[idx] = val;
    }
}

unsigned grid_for(int64_t work, int threads) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(nblk(work, threads), (int64_t)sm_count() * 16));
}

// CTAs of `kern` that fit on one SM at once (per device, cached).
int resident_ctas(const void* kern, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> cache;
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(kern, dev);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    MBR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem));
    n = std::max(1, n);
    cache[key] = n;
    return n;
}

// Grid of a grid-stride streaming kernel: at most one wave of resident CTAs,
// so every CTA starts at once and the loads of the whole grid are in flight
// together (a second wave would add its own ramp-up and tail).
unsigned grid_one_wave(const void* kern, int64_t work, int threads, size_t smem = 0) {
    const int64_t wave = (int64_t)sm_count() * resident_ctas(kern, threads, smem);
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(nblk(work, threads), wave));
}

// Frame scratch of the allocation-free iSTFT entry point: a fixed 16 MiB array
// that every device loading this library reserves for the life of the process.
__device__ __align__(256) float g_istft_frames[kIstftStaticFloats];

// Error word of the tensor-core kernels launched by the stand-alone ops.
__device__ int g_op_error;

int* op_error_word() {
    static std::mutex mu;
    static int* ptrs[kMaxDevices] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < kMaxDevices, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        MBR_CUDA(cudaGetSymbolAddress(&p, g_op_error));
        ptrs[dev] = (int*)p;
    }
    return ptrs[dev];
}

}  // namespace

float* istft_static_scratch() {
    // Host code cannot take the array's address directly (the symbol is a host
    // stand-in); ask the runtime once per device, with that device current.
    static std::mutex mu;
    static float* ptrs[kMaxDevices] = {};
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < kMaxDevices, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_istft_frames);
        if (e != cudaSuccess)
            throw Error(ERR_CUDA, std::string("cudaGetSymbolAddress(istft scratch) failed: ") + cudaGetErrorString(e));
        ptrs[dev] = (float*)p;
    }
    return ptrs[dev];
}

namespace {
// Launch descriptors of the stand-alone GEMM (one group + its tile list),
// grown on demand per device and reused by every call on that device.
struct LinearScratch {
    std::mutex mu;
    ops::GemmGroup* d_group = nullptr;
    int4* d_tiles = nullptr;
    size_t tile_cap = 0;
};
LinearScratch& linear_scratch(int dev) {
    static LinearScratch s[kMaxDevices];
    return s[dev];
}

void check_op_error(cudaStream_t st) {
    MBR_CUDA(cudaStreamSynchronize(st));
    int* err = op_error_word();
    int e = 0;
    MBR_CUDA(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e != 0) {
        const int zero = 0;
        MBR_CUDA(cudaMemcpy(err, &zero, sizeof(int), cudaMemcpyHostToDevice));
        throw Error(e == 2 ? ERR_CUDA : ERR_TIMEOUT, "tensor-core kernel error " + std::to_string(e));
    }
}
}  // namespace

void attention(const void* q, const void* k, const void* v, int64_t B, int H, int N, int D, float scale,
               const float* gates, void* out, int dtype, cudaStream_t st) {
    MBR_CHECK(B > 0 && H > 0 && N > 0 && (D == 32 || D == 64), "attention: bad shape (head dim 32 or 64)");
    if (scale == 0.0f) scale = 1.0f / std::sqrt((float)D);  // reference default
    // sequence s = b, position = token within it: the band-axis token map with NB = N
    if (dtype != DT_F32 && tc::attention_supported(D)) {
        int* err = op_error_word();
        tc::attention(q, k, v, tc::head_major_layout(B, H, N, D), B, H, N, D, scale, gates, ops::SEQ_FREQ, N, 1, out,
                      dtype, err, st);
        check_op_error(st);
    } else {
        ops::attention_simt(q, k, v, B, H, N, D, scale, gates, ops::SEQ_FREQ, N, 1, out, dtype, st);
    }
}


void linear(const void* x, const void* w, const float* bias, void* y, int64_t rows, int in, int out, int act,
            int dtype, cudaStream_t st) {
    MBR_CHECK(rows >= 0 && rows < (1ll << 31) && in > 0 && out > 0 && act >= 0 && act <= 2, "linear: bad argument");
    if (rows == 0) return;
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < kMaxDevices, "device index out of range");
    LinearScratch& S = linear_scratch(dev);
    std::lock_guard<std::mutex> lock(S.mu);
    if (!S.d_group) MBR_CUDA(cudaMalloc(&S.d_group, sizeof(ops::GemmGroup)));
    ops::GemmGroup g{};
    g.A = x;
    g.B = w;
    g.C = y;
    g.bias = bias;
    g.lda = in;
    g.ldb = in;
    g.ldc = out;
    g.M = (int)rows;
    g.N = out;
    g.K = in;
    const int epi = act == 1 ? ops::EPI_GELU_T : act == 2 ? ops::EPI_TANH_T : ops::EPI_T;
    MBR_CUDA(cudaMemcpyAsync(S.d_group, &g, sizeof(g), cudaMemcpyHostToDevice, st));
    auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    const bool tc_ok = dtype != DT_F32 && in % 16 == 0 && out % 8 == 0 && al16(x) && al16(w) && al16(y);
    if (tc_ok) {
        tc::GemmPlanTC p;
        p.groups = S.d_group;
        p.h_groups = &g;
        p.ngroups = 1;
        p.maxM = g.M;
        p.maxN = out;
        p.epi = epi;
        p.a_base = x, p.a_rows = rows, p.a_cols = in;
        p.b_base = w, p.b_rows = out, p.b_cols = in;
        p.c_base = y, p.c_rows = rows, p.c_cols = out, p.c_groups = 1;
        p.c_row_stride = out, p.c_group_stride = rows * out, p.c_dtype = dtype;
        std::vector<int4> tiles;
        tc::GemmLaunch L;
        size_t first = 0;
        tc::gemm_prepare(p, dtype, tiles, L, first);
        if (tiles.size() > S.tile_cap) {
            if (S.d_tiles) MBR_CUDA(cudaFree(S.d_tiles));
            S.d_tiles = nullptr;
            MBR_CUDA(cudaMalloc(&S.d_tiles, tiles.size() * sizeof(int4)));
            S.tile_cap = tiles.size();
        }
        MBR_CUDA(cudaMemcpyAsync(S.d_tiles, tiles.data(), tiles.size() * sizeof(int4), cudaMemcpyHostToDevice, st));
        L.tiles = S.d_tiles;
        tc::gemm_launch(L, dtype, op_error_word(), st);
    } else {
        ops::gemm_simt(S.d_group, 1, g.M, out, dtype, epi, st);
    }
    check_op_error(st);  // the scratch (and the pageable sources above) are reused next call
}

void ffn(const void* x, const void* w1, const float* b1, const void* w2, const float* b2, float* resid, int64_t rows,
         int dim, int hidden, int dtype, cudaStream_t st) {
    if (!tc::ffn_supported(dim, hidden, dtype))
        throw Error(ERR_UNSUPPORTED, "ffn: needs fp16/bf16, dim 256 or 384 and hidden a multiple of 64");
    if (rows == 0) return;
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    MBR_CHECK(dev >= 0 && dev < kMaxDevices, "device index out of range");
    LinearScratch& S = linear_scratch(dev);
    std::lock_guard<std::mutex> lock(S.mu);
    std::vector<int4> items;
    tc::FfnLaunch L;
    size_t first = 0;
    tc::ffn_prepare(x, w1, b1, w2, b2, resid, rows, dim, hidden, dtype, items, L, first);
    if (items.size() > S.tile_cap) {
        if (S.d_tiles) MBR_CUDA(cudaFree(S.d_tiles));
        S.d_tiles = nullptr;
        MBR_CUDA(cudaMalloc(&S.d_tiles, items.size() * sizeof(int4)));
        S.tile_cap = items.size();
    }
    MBR_CUDA(cudaMemcpyAsync(S.d_tiles, items.data(), items.size() * sizeof(int4), cudaMemcpyHostToDevice, st));
    L.items = S.d_tiles + first;
    tc::ffn_launch(L, dtype, op_error_word(), st);
    check_op_error(st);  // the scratch (and the pageable source above) are reused next call
}

void add(const void* a, const void* b, void* y, int64_t n, int dtype, cudaStream_t st) {
    MBR_CHECK(n % 8 == 0, "add: element count must be a multiple of 8");
    MBR_DISPATCH_DTYPE(dtype, T, {
        add_kernel<T><<<grid_for(n / 8, 256), 256, 0, st>>>((const T*)a, (const T*)b, (T*)y, n / 8);
    });
    MBR_CUDA(cudaGetLastError());
}

void gelu(const void* a, void* y, int64_t n, int dtype, cudaStream_t st) {
    MBR_CHECK(n % 8 == 0, "gelu: element count must be a multiple of 8");
    MBR_DISPATCH_DTYPE(dtype, T, { gelu_kernel<T><<<grid_for(n / 8, 256), 256, 0, st>>>((const T*)a, (T*)y, n / 8); });
    MBR_CUDA(cudaGetLastError());
}

void sigmoid_gate(const void* x, const void* g, void* y, int64_t rows, int H, int dh, int dtype, cudaStream_t st) {
    MBR_CHECK(dh % 8 == 0, "gate: head dim must be a multiple of 8");
    MBR_CHECK(rows * H * dh / 8 < (1ll << 32), "gate: tensor too large");
    MBR_DISPATCH_DTYPE(dtype, T, {
        gate_kernel<T><<<grid_one_wave((const void*)gate_kernel<T>, rows * H * dh / 8, 256), 256, 0, st>>>((const T*)x, (const T*)g, (T*)y, rows, H,
                                                                         dh);
    });
    MBR_CUDA(cudaGetLastError());
}

template <typename T>
bool launch_rms_group(int R, int NC, unsigned g, const void* x, const float* gamma, void* y, int64_t rows, int D,
                      float scale, cudaStream_t st) {
#define MBR_RMS_GROUP(r_, nc_)                                                              \
    if (R == r_ && NC == nc_) {                                                             \
        auto k = rms_group_kernel<T, r_, nc_>;                                              \
        const unsigned gg = std::min(g, grid_one_wave((const void*)k, (int64_t)g * 256, 256)); \
        k<<<gg, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);                    \
        MBR_CUDA(cudaGetLastError());                                                       \
        return true;                                                                        \
    }
    MBR_RMS_GROUP(1, 3) MBR_RMS_GROUP(1, 4) MBR_RMS_GROUP(2, 3) MBR_RMS_GROUP(2, 4) MBR_RMS_GROUP(3, 3)
    MBR_RMS_GROUP(4, 3) MBR_RMS_GROUP(4, 4) MBR_RMS_GROUP(6, 3) MBR_RMS_GROUP(8, 3) MBR_RMS_GROUP(8, 4)
#undef MBR_RMS_GROUP
    return false;
}

void rms_norm(const void* x, const float* gamma, void* y, int64_t rows, int D, float scale, int dtype,
              cudaStream_t st) {
    MBR_CHECK(D % 8 == 0 && D <= 1024, "rms_norm: dim must be a multiple of 8 and <= 1024");
    MBR_CHECK(((uintptr_t)gamma & 15) == 0, "rms_norm: gamma must be 16-byte aligned");
    // row groups with every lane busy: (R rows, NC chunks per lane) with R * D / 8 == 32 * NC
    const int D8 = D / 8;
    int R = 0, NC = 0;
    for (int r = 1; r <= 8 && !R; ++r)
        if ((r * D8) % 32 == 0 && (r * D8) / 32 >= 3 && (r * D8) / 32 <= 4) R = r, NC = r * D8 / 32;
    if (R) {
        // one warp per row group: as many CTAs as there are groups of 8, capped at one wave
        const unsigned g = (unsigned)ceil_div(ceil_div(rows, R), 8);
        bool done = false;
        MBR_DISPATCH_DTYPE(dtype, T, { done = launch_rms_group<T>(R, NC, g, x, gamma, y, rows, D, scale, st); });
        if (done) return;
    }
    unsigned grid = (unsigned)std::min<int64_t>(ceil_div(rows, 16), (int64_t)sm_count() * 8);
    MBR_DISPATCH_DTYPE(dtype, T, {
        if (D <= 256) rms_kernel<T, 1><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
        else if (D <= 512) rms_kernel<T, 2><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
        else rms_kernel<T, 4><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
    });
    MBR_CUDA(cudaGetLastError());
}

void rope(const void* x, const float* cs, const float* sn, void* y, int64_t seqs, int L, int H, int dtype,
          cudaStream_t st) {
    MBR_CHECK(seqs * L * H * 8 < (1ll << 32), "rope: tensor too large");
    MBR_CHECK(((uintptr_t)cs & 15) == 0 && ((uintptr_t)sn & 15) == 0, "rope: tables must be 16-byte aligned");
    MBR_DISPATCH_DTYPE(dtype, T, {
        rope_kernel<T><<<grid_one_wave((const void*)rope_kernel<T>, seqs * L * H * 8, 256), 256, 0, st>>>((const T*)x, cs, sn, (T*)y, seqs, L, H);
    });
    MBR_CUDA(cudaGetLastError());
}

BandTilesHost make_band_tiles(const std::vector<int>& fi, int C, int F) {
    BandTilesHost h;
    std::vector<std::vector<int>> ent;  // per tile: its j, ascending
    for (int f0 = 0; f0 < F; f0 += kBandTileBins) {
        std::vector<int> e;
        for (int j = 0; j < (int)fi.size(); ++j)
            if (fi[j] / C >= f0 && fi[j] / C < f0 + kBandTileBins) e.push_back(j);
        h.max_n = std::max(h.max_n, (int)e.size());
        ent.push_back(std::move(e));
    }
    h.stride = std::max(32, (h.max_n + 31) / 32 * 32);
    h.count = (int)ent.size();
    for (size_t t = 0; t < ent.size(); ++t) {
        const int f0 = (int)t * kBandTileBins, nf = std::min(kBandTileBins, F - f0), n = (int)ent[t].size();
        std::vector<int> row(n);
        for (int k = 0; k < n; ++k) row[k] = (fi[ent[t][k]] % C) * nf + fi[ent[t][k]] / C - f0;
        for (int k = 0; k < h.stride; ++k) {
            h.jl.push_back(k < n ? ent[t][k] : -1);
            h.jr.push_back(k < n ? row[k] : 0);
        }
        // entries grouped by row (counting sort), with the rows' start offsets
        std::vector<int> cnt(kBandRowOffs, 0);
        for (int k = 0; k < n; ++k) ++cnt[row[k] + 1];
        for (int r = 1; r < kBandRowOffs; ++r) cnt[r] += cnt[r - 1];
        h.bo.insert(h.bo.end(), cnt.begin(), cnt.end());
        std::vector<int> bk(h.stride, 0), cur(cnt.begin(), cnt.end() - 1);
        for (int k = 0; k < n; ++k) bk[cur[row[k]]++] = k;
        h.bk.insert(h.bk.end(), bk.begin(), bk.end());
    }
    return h;
}

void band_gather(const float2* spec, int B, int C, int F, int T, const int* fi, int64_t J, const BandTiles& bt,
                 void* x, int dtype, cudaStream_t st) {
    (void)fi;  // the tile tables carry the band map
    MBR_CHECK(C >= 1 && C <= 2 && bt.count == ceil_div(F, kBandTileBins) && bt.stride % 32 == 0,
              "band gather: one or two channels and a tile map of the spectrum");
    MBR_CHECK(((uintptr_t)spec & 7) == 0 && ((uintptr_t)x & (dtype == DT_F32 ? 7 : 3)) == 0,
              "band gather: misaligned buffers");
    MBR_CHECK((int64_t)C * F * T < (1ll << 31), "band gather: one batch entry of the spectrum exceeds 32-bit offsets");
    dim3 grid((unsigned)bt.count, (unsigned)ceil_div(T, kTT), (unsigned)B);
    MBR_DISPATCH_DTYPE(dtype, E, {
        gather_tiled_kernel<E><<<grid, kBandWarps * 32, 0, st>>>(spec, C, F, T, bt.jl, bt.jr, bt.stride, J, (E*)x);
    });
    MBR_CUDA(cudaGetLastError());
}

void mask_scatter(const float2* spec, const void* masks, int B, int S, int C, int F, int T, const float* nbpf,
                  int64_t J, const BandTiles& bt, float2* out, int dtype, cudaStream_t st) {
    MBR_CHECK(C >= 1 && C <= 2 && bt.count == ceil_div(F, kBandTileBins) && bt.stride % 32 == 0,
              "mask scatter: one or two channels and a tile map of the spectrum");
    MBR_CHECK(((uintptr_t)spec & 7) == 0 && ((uintptr_t)out & 7) == 0 &&
                  ((uintptr_t)masks & (dtype == DT_F32 ? 7 : 3)) == 0,
              "mask scatter: misaligned buffers");
    MBR_CHECK((int64_t)C * F * T < (1ll << 31) && 2 * J * (int64_t)kTT < (1ll << 31),
              "mask scatter: one batch entry of the spectrum or a frame block of masks exceeds 32-bit offsets");
    dim3 grid((unsigned)bt.count, (unsigned)ceil_div(T, kTT), (unsigned)(B * S));
    MBR_DISPATCH_DTYPE(dtype, E, {
        const size_t sm = sizeof(float2) * 2 * kBandTileBins * (kTT + 1) +
                          sizeof(typename PairOf<E>::type) * kTT * (size_t)(bt.stride + 1) +
                          sizeof(int) * (size_t)(kBandRowOffs + bt.stride) + sizeof(float) * 2 * kBandTileBins;
        MBR_CHECK(sm <= 200 * 1024, "mask scatter: band tile too wide");
        if (sm > 48 * 1024)
            MBR_CUDA(cudaFuncSetAttribute(scatter_tiled_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)sm));
        scatter_tiled_kernel<E><<<grid, kBandWarps * 32, sm, st>>>(spec, (const E*)masks, B, S, C, F, T, bt.jl,
                                                                    bt.bk, bt.bo, bt.stride, nbpf, J, out);
    });
    MBR_CUDA(cudaGetLastError());
}

int64_t stft_frames(int64_t L, int hop) { return L / hop + 1; }

void stft(const float* sig, int64_t nsig, int64_t L, int hop, float2* out, cudaStream_t st) {
    MBR_CHECK(L > kFft / 2 && hop > 0 && nsig > 0, "stft: signal shorter than the reflect padding");
    const int64_t T = stft_frames(L, hop);
    stft_ref_kernel<<<dim3((unsigned)T, (unsigned)nsig), 512, 0, st>>>(sig, L, hop, out, (int)T);
    MBR_CUDA(cudaGetLastError());
}

void istft(const float2* spec, int64_t nsig, int T, int hop, float* frames, int64_t lout, float* out,
           cudaStream_t st) {
    MBR_CHECK(T >= 1 && hop > 0 && nsig > 0 && lout > 0, "istft: bad shape");
    istft_frames_ref_kernel<<<dim3((unsigned)T, (unsigned)nsig), 512, 0, st>>>(spec, T, frames);
    MBR_CUDA(cudaGetLastError());
    istft_ola_ref_kernel<<<grid_for(nsig * lout, 256), 256, 0, st>>>(frames, nsig, T, hop, lout, out);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace opsapi
}  // namespace mbr
