// ops_api.cu — stand-alone tensor ops of the reference op library (mbr_tile /
// stft_tile, reference layouts) for drop-in callers and the op sweep:
// RMSNorm+gamma, residual add, GELU, sigmoid-gate multiply, RoPE, band gather,
// mask scatter-average, STFT and iSTFT.  Memory-bound kernels: 16-byte
// vectorised, coalesced, one pass over HBM, reductions in registers.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "common.cuh"
#include "ops_api.h"
#include "attention_tc.h"
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

// 8 elements of T as floats through one 16-byte (16-bit T) or two (fp32) accesses.
template <typename T>
struct Vec8 {
    float v[8];
    __device__ __forceinline__ void load(const T* p) {
        if constexpr (sizeof(T) == 4) {
            const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
            uint4 u = *reinterpret_cast<const uint4*>(p);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = to_f32(e[i]);
        }
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

// ---- residual add / GELU (n % 8 == 0, grid-stride) ----
template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, int64_t n8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        Vec8<T> x, z;
        x.load(a + 8 * i);
        z.load(b + 8 * i);
#pragma unroll
        for (int k = 0; k < 8; ++k) x.v[k] += z.v[k];
        x.store(y + 8 * i);
    }
}

template <typename T>
__global__ void gelu_kernel(const T* __restrict__ a, T* __restrict__ y, int64_t n8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        Vec8<T> x;
        x.load(a + 8 * i);
#pragma unroll
        for (int k = 0; k < 8; ++k) x.v[k] = gelu_erf(x.v[k]);
        x.store(y + 8 * i);
    }
}

// y[r][h*dh + d] = x[r][h*dh + d] * g[r][h]   (dh % 8 == 0)
template <typename T>
__global__ void gate_kernel(const T* __restrict__ x, const T* __restrict__ g, T* __restrict__ y, int64_t rows, int H,
                            int dh) {
    const int per_row = H * dh / 8;
    const int64_t n8 = rows * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / per_row;
        const int h = (int)(i % per_row) * 8 / dh;
        const float gv = to_f32(g[r * H + h]);
        Vec8<T> a;
        a.load(x + 8 * i);
#pragma unroll
        for (int k = 0; k < 8; ++k) a.v[k] *= gv;
        a.store(y + 8 * i);
    }
}

// RMSNorm with gamma, dtype in / dtype out; one warp per row, D % 8 == 0, D <= 1024.
template <typename T, int MAXC>
__global__ void __launch_bounds__(256) rms_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                  T* __restrict__ y, int64_t rows, int D, float scale) {
    const int lane = threadIdx.x & 31, D8 = D / 8;
    float g[MAXC][8];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
        const int c = lane + 32 * i;
#pragma unroll
        for (int k = 0; k < 8; ++k) g[i][k] = c < D8 ? gamma[8 * c + k] : 0.f;
    }
    const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += stride) {
        Vec8<T> v[MAXC];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            const int c = lane + 32 * i;
            if (c < D8) {
                v[i].load(x + r * D + 8 * c);
#pragma unroll
                for (int k = 0; k < 8; ++k) ss += v[i].v[k] * v[i].v[k];
            }
        }
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss + 1e-12f) * scale;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            const int c = lane + 32 * i;
            if (c < D8) {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[i].v[k] *= inv * g[i][k];
                v[i].store(y + r * D + 8 * c);
            }
        }
    }
}

// RoPE over positions: x [seqs][L][H][64]; pair (2i, 2i+1) of every head at
// position p rotated by (cos, sin)[p][i].
template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
                            T* __restrict__ y, int64_t seqs, int L, int H) {
    const int64_t n8 = seqs * L * H * 8;  // 8 chunks of 8 per 64-wide head
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int chunk = (int)(i & 7);
        const int p = (int)((i / (8 * H)) % L);
        Vec8<T> a;
        a.load(x + 8 * i);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int pi = chunk * 4 + k;
            const float c = cs[p * 32 + pi], s = sn[p * 32 + pi];
            const float x0 = a.v[2 * k], x1 = a.v[2 * k + 1];
            a.v[2 * k] = x0 * c - x1 * s;
            a.v[2 * k + 1] = x0 * s + x1 * c;
        }
        a.store(y + 8 * i);
    }
}

// Band gather (gather_freqs_fold_complex with the stereo merge folded in):
// spec [B][C][F][T] complex -> x[b][t][2j + r] = spec[b][fi_j % C][fi_j / C][t][r].
// One CTA per (b, 4-frame tile): the tile's frames of every bin pass through
// shared memory so each strided spectrum read is a full 32-byte sector.
constexpr int kGT = 4;  // frames per gather CTA

template <typename T>
__global__ void __launch_bounds__(256) gather_kernel(const float2* __restrict__ spec, int C, int F, int Tn,
                                                     const int* __restrict__ fi, int64_t J, T* __restrict__ x) {
    extern __shared__ float2 tile[];  // [C*F][kGT]
    const int b = blockIdx.y, t0 = blockIdx.x * kGT;
    const int nt = min(kGT, Tn - t0);
    const int FC = F * C;
    for (int i = threadIdx.x; i < FC * kGT; i += blockDim.x) {
        const int row = i / kGT, tt = i % kGT;  // row = c * F + f
        tile[i] = tt < nt ? spec[(((int64_t)b * FC + row) * Tn) + t0 + tt] : make_float2(0.f, 0.f);
    }
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt) {
        T* dst = x + ((int64_t)b * Tn + t0 + tt) * 2 * J;
        for (int64_t j = threadIdx.x; j < J; j += blockDim.x) {
            const int fs = fi[j];
            const float2 v = tile[((fs % C) * F + fs / C) * kGT + tt];
            dst[2 * j] = from_f32<T>(v.x);
            dst[2 * j + 1] = from_f32<T>(v.y);
        }
    }
}

// Mask scatter-average (apply_mask_and_scatter, gather form over the reverse
// band map): out[b][s][c][f][t] = sum_{j: fi_j = f*C+c} spec[b][c][f][t] * mask[s][b*T+t][j] / nbpf[f*C+c].
template <typename T>
__global__ void scatter_kernel(const float2* __restrict__ spec, const T* __restrict__ masks, int B, int S, int C,
                               int F, int Tn, const int* __restrict__ rev_off, const int* __restrict__ rev_idx,
                               const float* __restrict__ nbpf, int64_t J, float2* __restrict__ out) {
    const int64_t total = (int64_t)B * S * C * F * Tn;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i % Tn);
        int64_t r = i / Tn;
        const int f = (int)(r % F);
        r /= F;
        const int c = (int)(r % C);
        r /= C;
        const int s = (int)(r % S);
        const int b = (int)(r / S);
        const int fs = f * C + c;
        const float2 x = spec[(((int64_t)b * C + c) * F + f) * Tn + t];
        const float den = fmaxf(nbpf[fs], 1e-8f);
        const T* mk = masks + ((int64_t)s * B * Tn + (int64_t)b * Tn + t) * 2 * J;
        float2 acc = make_float2(0.f, 0.f);
        for (int q = rev_off[fs]; q < rev_off[fs + 1]; ++q) {
            const int j = rev_idx[q];
            const float mr = to_f32(mk[2 * j]), mi = to_f32(mk[2 * j + 1]);
            acc.x += (x.x * mr - x.y * mi) / den;
            acc.y += (x.x * mi + x.y * mr) / den;
        }
        out[i] = acc;
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
    MBR_DISPATCH_DTYPE(dtype, T, {
        gate_kernel<T><<<grid_for(rows * H * dh / 8, 256), 256, 0, st>>>((const T*)x, (const T*)g, (T*)y, rows, H,
                                                                         dh);
    });
    MBR_CUDA(cudaGetLastError());
}

void rms_norm(const void* x, const float* gamma, void* y, int64_t rows, int D, float scale, int dtype,
              cudaStream_t st) {
    MBR_CHECK(D % 8 == 0 && D <= 1024, "rms_norm: dim must be a multiple of 8 and <= 1024");
    unsigned grid = (unsigned)std::min<int64_t>(ceil_div(rows, 8), (int64_t)sm_count() * 8);
    MBR_DISPATCH_DTYPE(dtype, T, {
        if (D <= 256) rms_kernel<T, 1><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
        else if (D <= 512) rms_kernel<T, 2><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
        else rms_kernel<T, 4><<<grid, 256, 0, st>>>((const T*)x, gamma, (T*)y, rows, D, scale);
    });
    MBR_CUDA(cudaGetLastError());
}

void rope(const void* x, const float* cs, const float* sn, void* y, int64_t seqs, int L, int H, int dtype,
          cudaStream_t st) {
    MBR_DISPATCH_DTYPE(dtype, T, {
        rope_kernel<T><<<grid_for(seqs * L * H * 8, 256), 256, 0, st>>>((const T*)x, cs, sn, (T*)y, seqs, L, H);
    });
    MBR_CUDA(cudaGetLastError());
}

void band_gather(const float2* spec, int B, int C, int F, int T, const int* fi, int64_t J, void* x, int dtype,
                 cudaStream_t st) {
    size_t sm = sizeof(float2) * (size_t)C * F * kGT;
    dim3 grid((unsigned)ceil_div(T, kGT), (unsigned)B);
    MBR_DISPATCH_DTYPE(dtype, E, {
        if (sm > 48 * 1024)
            MBR_CUDA(cudaFuncSetAttribute(gather_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        gather_kernel<E><<<grid, 256, sm, st>>>(spec, C, F, T, fi, J, (E*)x);
    });
    MBR_CUDA(cudaGetLastError());
}

void mask_scatter(const float2* spec, const void* masks, int B, int S, int C, int F, int T, const int* rev_off,
                  const int* rev_idx, const float* nbpf, int64_t J, float2* out, int dtype, cudaStream_t st) {
    const int64_t total = (int64_t)B * S * C * F * T;
    MBR_DISPATCH_DTYPE(dtype, E, {
        scatter_kernel<E><<<grid_for(total, 256), 256, 0, st>>>(spec, (const E*)masks, B, S, C, F, T, rev_off,
                                                                 rev_idx, nbpf, J, out);
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
