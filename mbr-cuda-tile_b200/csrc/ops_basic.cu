// ops_basic.cu — memory-bound kernels of the forward: STFT, band gather + band
// RMSNorm, RMSNorm (+gates), RoPE scatter, mask scatter-average, iSTFT and the
// chunk overlap-add.  Every kernel reads and writes HBM once per element with
// coalesced (mostly 128-bit) accesses and keeps reductions in registers /
// warp shuffles.
#include <algorithm>

#include "common.cuh"
#include "ops.h"

namespace mbr {
namespace ops {

namespace {

constexpr int kFft = 2048;
constexpr int kLog2Fft = 11;
constexpr int kBins = kFft / 2 + 1;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// In-place radix-2 DIT FFT over `nch` 2048-point buffers in shared memory whose
// inputs were stored in bit-reversed order.  tw[k] = exp(-2*pi*i*k/2048).
__device__ void fft2048_smem(float2* buf, int nch, const float2* tw, bool inverse) {
    for (int len = 2; len <= kFft; len <<= 1) {
        int half = len >> 1;
        int tstride = kFft / len;
        __syncthreads();
        for (int bi = threadIdx.x; bi < nch * (kFft / 2); bi += blockDim.x) {
            int ch = bi / (kFft / 2);
            int kk = bi % (kFft / 2);
            int grp = kk / half, k = kk % half;
            int i0 = ch * kFft + grp * len + k, i1 = i0 + half;
            float2 w = tw[k * tstride];
            if (inverse) w.y = -w.y;
            float2 a = buf[i0], b = cmul(buf[i1], w);
            buf[i0] = make_float2(a.x + b.x, a.y + b.y);
            buf[i1] = make_float2(a.x - b.x, a.y - b.y);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ int bitrev11(int n) { return (int)(__brev((unsigned)n) >> (32 - kLog2Fft)); }

// One CTA per (b, t): the C channel frames of that time step.
__global__ void __launch_bounds__(512) stft_kernel(const float* __restrict__ sig, int C, int64_t L, int hop,
                                                   const float* __restrict__ window,
                                                   const float2* __restrict__ twiddle, float norm,
                                                   float2* __restrict__ spec, int T) {
    extern __shared__ float2 smem[];
    float2* tw = smem;            // [1024]
    float2* buf = smem + kFft / 2;  // [C][2048]
    int bt = blockIdx.x;
    int b = bt / T, t = bt % T;
    for (int i = threadIdx.x; i < kFft / 2; i += blockDim.x) tw[i] = twiddle[i];
    for (int i = threadIdx.x; i < C * kFft; i += blockDim.x) {
        int ch = i / kFft, n = i % kFft;
        int64_t p = reflect_idx((int64_t)t * hop + n - kFft / 2, L);
        float x = sig[((int64_t)b * C + ch) * L + p] * window[n];
        buf[ch * kFft + bitrev11(n)] = make_float2(x, 0.f);
    }
    fft2048_smem(buf, C, tw, false);
    float2* out = spec + (int64_t)bt * kBins * C;
    for (int i = threadIdx.x; i < kBins * C; i += blockDim.x) {
        int f = i / C, ch = i % C;
        float2 v = buf[ch * kFft + f];
        out[i] = make_float2(v.x * norm, v.y * norm);
    }
}

// One CTA per token row (b, t): stage the spectrum row, then one warp per band
// gathers the band's (re, im) values, RMS-normalises them and writes the padded
// band slot of xb.
template <typename T>
__global__ void __launch_bounds__(256) band_gather_norm_kernel(const float2* __restrict__ spec, int FC,
                                                               const int* __restrict__ fi,
                                                               const int* __restrict__ band_jofs,
                                                               const int* __restrict__ band_kofs,
                                                               const float* __restrict__ gamma, int NB,
                                                               T* __restrict__ xb, int64_t KP) {
    extern __shared__ float2 row[];
    int64_t mt = blockIdx.x;
    const float2* src = spec + mt * FC;
    for (int i = threadIdx.x; i < FC; i += blockDim.x) row[i] = src[i];
    __syncthreads();
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    T* dst = xb + mt * KP;
    for (int b = warp; b < NB; b += nw) {
        int j0 = band_jofs[b], j1 = band_jofs[b + 1];
        int nv = 2 * (j1 - j0);
        float ss = 0.f;
        for (int q = lane; q < nv; q += 32) {
            float2 v = row[fi[j0 + (q >> 1)]];
            float x = (q & 1) ? v.y : v.x;
            ss += x * x;
        }
        ss = warp_sum(ss);
        float inv = rsqrtf(ss + 1e-12f);
        float scale = sqrtf((float)nv);
        int k0 = band_kofs[b], k1 = band_kofs[b + 1];
        for (int q = lane; q < k1 - k0; q += 32) {
            float y = 0.f;
            if (q < nv) {
                float2 v = row[fi[j0 + (q >> 1)]];
                float x = (q & 1) ? v.y : v.x;
                y = x * inv * gamma[2 * j0 + q] * scale;
            }
            dst[k0 + q] = from_f32<T>(y);
        }
    }
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 y) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(p) = y;
    } else {
        T e[4] = {from_f32<T>(y.x), from_f32<T>(y.y), from_f32<T>(y.z), from_f32<T>(y.w)};
        *reinterpret_cast<uint2*>(p) = *reinterpret_cast<uint2*>(e);
    }
}

// Packed f32x2 helpers of the row kernels: q + (v.x, v.y)^2 + (v.z, v.w)^2
// as two pair sums, v * s * g (the product rounded in that order), and
// q + (v.x w.x, v.y w.y) + (v.z w.z, v.w w.w).
__device__ __forceinline__ float2 sq_acc2(float4 v, float2 q) {
    q = __ffma2_rn(make_float2(v.x, v.y), make_float2(v.x, v.y), q);
    return __ffma2_rn(make_float2(v.z, v.w), make_float2(v.z, v.w), q);
}
__device__ __forceinline__ float4 scale_mul2(float4 v, float s, float4 g) {
    const float2 a = __fmul2_rn(__fmul2_rn(make_float2(v.x, v.y), make_float2(s, s)), make_float2(g.x, g.y));
    const float2 b = __fmul2_rn(__fmul2_rn(make_float2(v.z, v.w), make_float2(s, s)), make_float2(g.z, g.w));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float2 dot_acc2(float4 v, float4 w, float2 q) {
    q = __ffma2_rn(make_float2(v.x, v.y), make_float2(w.x, w.y), q);
    return __ffma2_rn(make_float2(v.z, v.w), make_float2(w.z, w.w), q);
}

// One warp per row, rows strided over a persistent grid (the gate weights are
// staged in shared memory once per CTA).  Each lane holds up to MAXC float4
// chunks of the row in registers.  D % 4 == 0, D <= 128 * MAXC, H <= 32.
template <typename T, int MAXC>
__global__ void __launch_bounds__(256, 2) rms_norm_kernel(const float* __restrict__ R, int64_t M, int D,
                                                          const float* __restrict__ gamma, float scale,
                                                          T* __restrict__ xn, int64_t band_major_mt, int NB,
                                                          float* r_out, const float* __restrict__ wg,
                                                          const float* __restrict__ bg, int H,
                                                          float* __restrict__ gates,
                                                          const float* __restrict__ gamma2) {
    // One warp normalises two rows at a time (lane c holds columns 4c + 128i):
    // the gate weights read from shared memory then feed both rows.
    extern __shared__ float4 swg4[];  // [H][D/4]
    const int D4 = D / 4;
    if (wg) {
        const float4* w4 = reinterpret_cast<const float4*>(wg);
        for (int i = threadIdx.x; i < H * D4; i += blockDim.x) swg4[i] = w4[i];
        __syncthreads();
    }
    const int lane = threadIdx.x & 31;
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* h4 = reinterpret_cast<const float4*>(gamma2);
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    // software pipeline: the loads of the next PF row pairs are in flight while
    // this pair is reduced, normalised and stored (PF = 2 while the buffers fit
    // the register budget, for D <= 384)
    constexpr int PF = MAXC <= 3 ? 2 : 1;
    float4 nx[PF][2][MAXC];
    auto load_pair = [&](int64_t mp, float4 (&dst)[2][MAXC]) {
        const bool two_p = mp + 1 < M;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float4* x4 = reinterpret_cast<const float4*>(R + (mp + (r && two_p ? 1 : 0)) * D);
#pragma unroll
            for (int i = 0; i < MAXC; ++i) {
                const int c = lane + 32 * i;
                dst[r][i] = c < D4 ? __ldcs(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
#pragma unroll
    for (int k = 0; k < PF; ++k)
        if (2 * wid + 2 * warps * k < M) load_pair(2 * wid + 2 * warps * k, nx[k]);
    for (int64_t m0 = 2 * wid; m0 < M; m0 += 2 * warps) {
        const bool two = m0 + 1 < M;
        float4 v[2][MAXC];
        float ss[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float2 q = make_float2(0.f, 0.f);  // packed partial sums of squares
#pragma unroll
            for (int i = 0; i < MAXC; ++i) {
                v[r][i] = nx[0][r][i];
                q = sq_acc2(v[r][i], q);
            }
            ss[r] = q.x + q.y;
        }
#pragma unroll
        for (int k = 0; k + 1 < PF; ++k)
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int i = 0; i < MAXC; ++i) nx[k][r][i] = nx[k + 1][r][i];
        if (m0 + 2 * warps * PF < M) load_pair(m0 + 2 * warps * PF, nx[PF - 1]);
        ss[0] = warp_sum(ss[0]);
        ss[1] = warp_sum(ss[1]);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int64_t m = m0 + r;
            const float inv = rsqrtf(ss[r] + 1e-12f) * scale;
#pragma unroll
            for (int i = 0; i < MAXC; ++i) {
                const int c = lane + 32 * i;
                const float4 g = c < D4 ? __ldg(g4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[r][i] = scale_mul2(v[r][i], inv, g);
                if (c < D4 && r_out && (r == 0 || two)) reinterpret_cast<float4*>(r_out + m * D)[c] = v[r][i];
            }
        }
        if (gamma2) {
            // a second RMSNorm of the (stored) first result: the next block's
            // pre-norm, so the residual stream is read once for both
            float s2[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float2 q = make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < MAXC; ++i) q = sq_acc2(v[r][i], q);
                s2[r] = q.x + q.y;
            }
            s2[0] = warp_sum(s2[0]);
            s2[1] = warp_sum(s2[1]);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const float inv2 = rsqrtf(s2[r] + 1e-12f) * scale;
#pragma unroll
                for (int i = 0; i < MAXC; ++i) {
                    const int c = lane + 32 * i;
                    const float4 g2 = c < D4 ? __ldg(h4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    v[r][i] = scale_mul2(v[r][i], inv2, g2);
                }
            }
        }
        if (xn) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && !two) break;
                const int64_t m = m0 + r;
                const int64_t orow = band_major_mt > 0 ? (m % NB) * band_major_mt + m / NB : m;
#pragma unroll
                for (int i = 0; i < MAXC; ++i) {
                    const int c = lane + 32 * i;
                    if (c < D4) store4<T>(xn + orow * D + 4 * c, v[r][i]);
                }
            }
        }
        if (wg && H == 8) {
            // eight dot products per row at once: per-lane partial sums for all
            // heads, then a transposing butterfly (each xor step halves the
            // heads a lane carries) so lane 4h ends with head h
            float a[2][8];
#pragma unroll
            for (int h = 0; h < 8; ++h) {
                float2 q[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // packed partial dots
#pragma unroll
                for (int i = 0; i < MAXC; ++i) {
                    const int c = lane + 32 * i;
                    if (c < D4) {
                        const float4 w = swg4[h * D4 + c];
#pragma unroll
                        for (int r = 0; r < 2; ++r) q[r] = dot_acc2(v[r][i], w, q[r]);
                    }
                }
                a[0][h] = q[0].x + q[0].y;
                a[1][h] = q[1].x + q[1].y;
            }
            const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float send = b4 ? a[r][k] : a[r][k + 4];
                    const float keep = b4 ? a[r][k + 4] : a[r][k];
                    a[r][k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const float send = b3 ? a[r][k] : a[r][k + 2];
                    const float keep = b3 ? a[r][k + 2] : a[r][k];
                    a[r][k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                const float send = b2 ? a[r][0] : a[r][1];
                const float keep = b2 ? a[r][1] : a[r][0];
                float t = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                t += __shfl_xor_sync(0xffffffffu, t, 1);
                if ((lane & 3) == 0 && (r == 0 || two)) {
                    const int h = lane >> 2;
                    gates[(m0 + r) * H + h] = 1.0f / (1.0f + expf(-(t + bg[h])));
                }
            }
        } else if (wg) {
            for (int r = 0; r < 2; ++r) {
                float mine = 0.f;  // lane h ends up holding the dot product of gate h
                for (int h = 0; h < H; ++h) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < MAXC; ++i) {
                        const int c = lane + 32 * i;
                        if (c < D4) {
                            const float4 w = swg4[h * D4 + c];
                            acc += v[r][i].x * w.x + v[r][i].y * w.y + v[r][i].z * w.z + v[r][i].w * w.w;
                        }
                    }
                    acc = warp_sum(acc);
                    if (lane == h) mine = acc;
                }
                if (lane < H && (r == 0 || two)) gates[(m0 + r) * H + lane] = 1.0f / (1.0f + expf(-(mine + bg[lane])));
            }
        }
    }
}

__device__ __forceinline__ void seq_of_token(int64_t m, int mode, int NB, int T, int64_t& s, int& pos) {
    if (mode == SEQ_TIME) {
        int k = (int)(m % NB);
        int64_t bt = m / NB;
        int64_t b = bt / T;
        pos = (int)(bt % T);
        s = b * NB + k;
    } else {
        s = m / NB;
        pos = (int)(m % NB);
    }
}
__device__ __forceinline__ int64_t token_of(int64_t s, int pos, int mode, int NB, int T) {
    return mode == SEQ_TIME ? (((s / NB) * T + pos) * NB + (s % NB)) : (s * NB + pos);
}

template <typename T>
__global__ void rope_scatter_kernel(const T* __restrict__ qkv, int64_t M, int H, int dh,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int mode,
                                    int NB, int Tn, T* __restrict__ q, T* __restrict__ k, T* __restrict__ v) {
    int half = dh / 2;
    int64_t total = M * H * half;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    int i = (int)(idx % half);
    int h = (int)((idx / half) % H);
    int64_t m = idx / ((int64_t)half * H);
    int64_t s;
    int pos;
    seq_of_token(m, mode, NB, Tn, s, pos);
    int L = mode == SEQ_TIME ? Tn : NB;
    int DI = H * dh;
    const T* row = qkv + m * 3 * DI + h * dh + 2 * i;
    float c = cos_t[pos * half + i], sn = sin_t[pos * half + i];
    float q0 = to_f32(row[0]), q1 = to_f32(row[1]);
    float k0 = to_f32(row[DI]), k1 = to_f32(row[DI + 1]);
    int64_t o = ((s * H + h) * L + pos) * dh + 2 * i;
    q[o] = from_f32<T>(q0 * c - q1 * sn);
    q[o + 1] = from_f32<T>(q0 * sn + q1 * c);
    k[o] = from_f32<T>(k0 * c - k1 * sn);
    k[o + 1] = from_f32<T>(k0 * sn + k1 * c);
    if (v) {
        v[o] = row[2 * DI];
        v[o + 1] = row[2 * DI + 1];
    }
}

// Simple online-softmax attention: one thread per query row, K/V tiles of 64
// keys staged in shared memory.  Used for fp32 compute and as the first
// correct path; the tensor-core kernel replaces it for 16-bit dtypes.
template <typename T, int DH>
__global__ void __launch_bounds__(128) attention_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                             const T* __restrict__ v, int H, int L, float scale,
                                                             const float* __restrict__ gates, int mode, int NB,
                                                             int Tn, T* __restrict__ merged) {
    __shared__ float Ks[64][DH + 1];
    __shared__ float Vs[64][DH + 1];
    int64_t sh = blockIdx.y;
    int64_t s = sh / H;
    int h = (int)(sh % H);
    int qi = blockIdx.x * blockDim.x + threadIdx.x;
    const T* qb = q + sh * (int64_t)L * DH;
    const T* kb = k + sh * (int64_t)L * DH;
    const T* vb = v + sh * (int64_t)L * DH;
    const float kLog2e = 1.4426950408889634f;
    float qr[DH], o[DH];
    bool valid = qi < L;
#pragma unroll
    for (int d = 0; d < DH; ++d) {
        qr[d] = valid ? to_f32(qb[(int64_t)qi * DH + d]) * scale * kLog2e : 0.f;
        o[d] = 0.f;
    }
    float mx = -INFINITY, l = 0.f;
    for (int k0 = 0; k0 < L; k0 += 64) {
        __syncthreads();
        for (int i = threadIdx.x; i < 64 * DH; i += blockDim.x) {
            int r = i / DH, d = i % DH;
            bool ok = k0 + r < L;
            Ks[r][d] = ok ? to_f32(kb[(int64_t)(k0 + r) * DH + d]) : 0.f;
            Vs[r][d] = ok ? to_f32(vb[(int64_t)(k0 + r) * DH + d]) : 0.f;
        }
        __syncthreads();
        int nk = min(64, L - k0);
        for (int j0 = 0; j0 < nk; j0 += 16) {
            float sc[16];
            float cmax = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                float a = 0.f;
#pragma unroll
                for (int d = 0; d < DH; ++d) a += qr[d] * Ks[j0 + jj][d];
                sc[jj] = (j0 + jj < nk) ? a : -INFINITY;
                cmax = fmaxf(cmax, sc[jj]);
            }
            float nm = fmaxf(mx, cmax);
            float corr = exp2f(mx - nm);
            l *= corr;
#pragma unroll
            for (int d = 0; d < DH; ++d) o[d] *= corr;
            mx = nm;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                float p = exp2f(sc[jj] - mx);
                l += p;
#pragma unroll
                for (int d = 0; d < DH; ++d) o[d] += p * Vs[j0 + jj][d];
            }
        }
    }
    if (!valid) return;
    int64_t tok = token_of(s, qi, mode, NB, Tn);
    float g = (gates ? gates[tok * H + h] : 1.0f) / l;
    T* dst = merged + tok * (int64_t)H * DH + h * DH;
#pragma unroll
    for (int d = 0; d < DH; ++d) dst[d] = from_f32<T>(o[d] * g);
}

// Gather-form mask application: one thread per (b, s, t, fs).
__global__ void mask_scatter_kernel(const float2* __restrict__ spec, const float* __restrict__ masks, int B, int S,
                                    int T, int C, int F, const int* __restrict__ rev_off,
                                    const int* __restrict__ rev_idx, const float* __restrict__ nbpf, int64_t J,
                                    bool zero_dc, float2* __restrict__ y) {
    int FC = F * C;
    int64_t total = (int64_t)B * S * T * FC;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    int fs = (int)(idx % FC);
    int64_t r = idx / FC;
    int t = (int)(r % T);
    r /= T;
    int s = (int)(r % S);
    int b = (int)(r / S);
    int f = fs / C, c = fs % C;
    float2 acc = make_float2(0.f, 0.f);
    if (!(zero_dc && f == 0)) {
        int64_t mt = (int64_t)b * T + t;
        float2 x = spec[mt * FC + fs];
        float den = fmaxf(nbpf[fs], 1e-8f);
        const float* mk = masks + ((int64_t)s * B * T + mt) * 2 * J;
        for (int q = rev_off[fs]; q < rev_off[fs + 1]; ++q) {
            int j = rev_idx[q];
            float2 m = make_float2(mk[2 * j], mk[2 * j + 1]);
            acc.x += (x.x * m.x - x.y * m.y) / den;
            acc.y += (x.x * m.y + x.y * m.x) / den;
        }
    }
    y[((((int64_t)b * S + s) * C + c) * T + t) * F + f] = acc;
}

// One CTA per frame: Hermitian completion, bit-reversed load, inverse FFT,
// frames[n] = Re(x[n]) / 2048 * w[n].
__global__ void __launch_bounds__(512) istft_frames_kernel(const float2* __restrict__ y, int T,
                                                           const float* __restrict__ window,
                                                           const float2* __restrict__ twiddle, float spec_scale,
                                                           float* __restrict__ frames) {
    extern __shared__ float2 smem[];
    float2* tw = smem;
    float2* buf = smem + kFft / 2;
    int64_t fr = blockIdx.x;  // o * T + t
    const float2* row = y + fr * kBins;
    for (int i = threadIdx.x; i < kFft / 2; i += blockDim.x) tw[i] = twiddle[i];
    for (int n = threadIdx.x; n < kFft; n += blockDim.x) {
        float2 v;
        if (n < kBins) {
            v = row[n];
        } else {
            v = row[kFft - n];
            v.y = -v.y;
        }
        buf[bitrev11(n)] = make_float2(v.x * spec_scale, v.y * spec_scale);
    }
    fft2048_smem(buf, 1, tw, true);
    float* out = frames + fr * kFft;
    const float inv = 1.0f / (float)kFft;
    for (int n = threadIdx.x; n < kFft; n += blockDim.x) out[n] = buf[n].x * inv * window[n];
}

__global__ void istft_ola_kernel(const float* __restrict__ frames, int64_t nsig, int T, int hop,
                                 const float* __restrict__ window, int64_t lout, float* __restrict__ out) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nsig * lout) return;
    int64_t o = idx / lout, q = idx % lout;
    int64_t full = (int64_t)(T - 1) * hop;  // centre-cropped length
    float val = 0.f;
    if (q < full) {
        int64_t p = q + kFft / 2;
        int64_t tmin = p - (kFft - 1) <= 0 ? 0 : (p - (kFft - 1) + hop - 1) / hop;
        int64_t tmax = min((int64_t)T - 1, p / hop);
        float acc = 0.f, ws = 0.f;
        for (int64_t t = tmin; t <= tmax; ++t) {
            int n = (int)(p - t * hop);
            float w = window[n];
            acc += frames[(o * T + t) * kFft + n];
            ws += w * w;
        }
        val = ws > 1e-8f ? acc / ws : acc;
    }
    out[idx] = val;
}

__device__ __forceinline__ float fade_weight(int64_t q, int chunk, int fade, bool first, bool last) {
    if (fade <= 0) return 1.0f;
    if (first && q < fade) return 1.0f;
    if (last && q >= chunk - fade) return 1.0f;
    if (fade == 1) return (q == 0 || q == chunk - 1) ? 0.0f : 1.0f;
    if (q < fade) return (float)q / (float)(fade - 1);
    if (q >= chunk - fade) return 1.0f - (float)(q - (chunk - fade)) / (float)(fade - 1);
    return 1.0f;
}

__global__ void prepare_chunks_kernel(const float* __restrict__ track, int C, int64_t N, int64_t track_lo,
                                      int64_t track_ld, int64_t border, bool padded,
                                      const int64_t* __restrict__ starts, int nchunks, int64_t total, int chunk,
                                      float* __restrict__ in) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)nchunks * C * chunk) return;
    int64_t q = idx % chunk;
    int ch = (int)((idx / chunk) % C);
    int ci = (int)(idx / ((int64_t)chunk * C));
    int64_t st = starts[ci];
    int64_t al = min((int64_t)chunk, total - st);
    float v = 0.f;
    int64_t pp = -1;
    if (q < al) pp = st + q;
    else if (al > chunk / 2) pp = st + reflect_idx(q, al);
    if (pp >= 0) v = track[(int64_t)ch * track_ld + (padded ? reflect_idx(pp - border, N) : pp) - track_lo];
    in[idx] = v;
}

// Adds the chunks of one batch in chunk order per sample (no atomics; the
// per-sample order equals the reference's sequential chunk order).  acc and
// wsum hold the padded-sample window [acc_lo, acc_lo + acc_stride).
__global__ void accumulate_chunks_kernel(const float* __restrict__ y, int nchunks, int SC, int64_t lout,
                                         const int64_t* __restrict__ starts, int64_t total, int chunk, int fade,
                                         float* __restrict__ acc, float* __restrict__ wsum, int64_t acc_lo,
                                         int64_t acc_stride) {
    int64_t lo = starts[0];
    int64_t hi = min(total, starts[nchunks - 1] + chunk);
    int64_t span = hi - lo;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)(SC + 1) * span) return;
    int o = (int)(idx / span);
    int64_t p = lo + idx % span;
    int64_t pl = p - acc_lo;
    float a = o < SC ? acc[(int64_t)o * acc_stride + pl] : wsum[pl];
    for (int ci = 0; ci < nchunks; ++ci) {
        int64_t st = starts[ci];
        int64_t en = min(st + chunk, total);
        if (p < st || p >= en) continue;
        int64_t q = p - st;
        float w = fade_weight(q, chunk, fade, st == 0, en >= total);
        if (o < SC) a += y[((int64_t)ci * SC + o) * lout + q] * w;
        else a += w;
    }
    if (o < SC) acc[(int64_t)o * acc_stride + pl] = a;
    else wsum[pl] = a;
}

// out[o][p - border] = acc / wsum (where wsum > 1e-8) for padded samples p in [p0, p1).
__global__ void normalize_crop_kernel(const float* __restrict__ acc, const float* __restrict__ wsum, int SC,
                                      int64_t acc_lo, int64_t acc_stride, int64_t p0, int64_t p1, int64_t border,
                                      int64_t out_stride, float* __restrict__ out) {
    int64_t n = p1 - p0;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)SC * n) return;
    int o = (int)(idx / n);
    int64_t p = p0 + idx % n;
    float w = wsum[p - acc_lo], v = acc[(int64_t)o * acc_stride + p - acc_lo];
    out[(int64_t)o * out_stride + p - border] = w > 1e-8f ? v / w : v;
}

// dst window gets src added (the previous shard's overlap-add boundary).
__global__ void add_window_kernel(float* __restrict__ acc, float* __restrict__ wsum, int64_t acc_stride,
                                  const float* __restrict__ racc, const float* __restrict__ rwsum, int64_t rlen,
                                  int SC) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)(SC + 1) * rlen) return;
    int o = (int)(idx / rlen);
    int64_t q = idx % rlen;
    if (o < SC) acc[(int64_t)o * acc_stride + q] += racc[(int64_t)o * rlen + q];
    else wsum[q] += rwsum[q];
}

__global__ void add_inplace_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] += src[i];
}

inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

void stft(const float* sig, int B, int C, int64_t L, int hop, const float* window, const float2* twiddle,
          float norm, float2* spec, int T, cudaStream_t st) {
    size_t sm = sizeof(float2) * (kFft / 2 + C * kFft);
    stft_kernel<<<B * T, 512, sm, st>>>(sig, C, L, hop, window, twiddle, norm, spec, T);
    MBR_CUDA(cudaGetLastError());
}

void band_gather_norm(const float2* spec, int64_t MT, int FC, const int* fi, const int* band_jofs,
                      const int* band_kofs, const float* gamma, int NB, void* xb, int64_t KP, int dtype,
                      cudaStream_t st) {
    MBR_DISPATCH_DTYPE(dtype, T, {
        band_gather_norm_kernel<T><<<(unsigned)MT, 256, sizeof(float2) * FC, st>>>(
            spec, FC, fi, band_jofs, band_kofs, gamma, NB, (T*)xb, KP);
    });
    MBR_CUDA(cudaGetLastError());
}

void rms_norm(const float* R, int64_t M, int D, const float* gamma, float scale, void* xn, int dtype,
              int64_t band_major_mt, int NB, float* r_out, const float* wg, const float* bg, int H, float* gates,
              cudaStream_t st, const float* gamma2) {
    MBR_CHECK(D % 4 == 0 && D <= 1024, "rms_norm: dim must be a multiple of 4 and <= 1024");
    MBR_CHECK(!wg || H <= 32, "rms_norm: at most 32 gates");
    size_t sm = wg ? sizeof(float) * H * D : 0;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        MBR_CUDA(cudaGetDevice(&dev));
        MBR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    }
    unsigned grid = (unsigned)std::min<int64_t>(ceil_div(M, 16), (int64_t)sms * 2);  // 2 rows per warp, 2 resident CTAs per SM
    MBR_DISPATCH_DTYPE(dtype, T, {
        auto run = [&](auto kern) {
            if (sm > 48 * 1024)
                MBR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
            kern<<<grid, 256, sm, st>>>(R, M, D, gamma, scale, (T*)xn, band_major_mt, NB, r_out, wg, bg, H, gates,
                                        gamma2);
        };
        if (D <= 128) run(rms_norm_kernel<T, 1>);
        else if (D <= 256) run(rms_norm_kernel<T, 2>);
        else if (D <= 384) run(rms_norm_kernel<T, 3>);
        else if (D <= 512) run(rms_norm_kernel<T, 4>);
        else run(rms_norm_kernel<T, 8>);
    });
    MBR_CUDA(cudaGetLastError());
}

void rope_scatter(const void* qkv, int64_t M, int H, int dh, const float* cos_t, const float* sin_t, int mode,
                  int NB, int T, void* q, void* k, void* v, int dtype, cudaStream_t st) {
    int64_t total = M * H * (dh / 2);
    MBR_DISPATCH_DTYPE(dtype, E, {
        rope_scatter_kernel<E><<<nblk(total, 256), 256, 0, st>>>((const E*)qkv, M, H, dh, cos_t, sin_t, mode, NB,
                                                                 T, (E*)q, (E*)k, (E*)v);
    });
    MBR_CUDA(cudaGetLastError());
}


void attention_simt(const void* q, const void* k, const void* v, int64_t nseq, int H, int L, int dh, float scale,
                    const float* gates, int mode, int NB, int T, void* merged, int dtype, cudaStream_t st) {
    dim3 grid(nblk(L, 128), (unsigned)(nseq * H));
    MBR_DISPATCH_DTYPE(dtype, E, {
        if (dh == 64)
            attention_simt_kernel<E, 64><<<grid, 128, 0, st>>>((const E*)q, (const E*)k, (const E*)v, H, L, scale,
                                                               gates, mode, NB, T, (E*)merged);
        else if (dh == 32)
            attention_simt_kernel<E, 32><<<grid, 128, 0, st>>>((const E*)q, (const E*)k, (const E*)v, H, L, scale,
                                                               gates, mode, NB, T, (E*)merged);
        else
            throw Error(ERR_UNSUPPORTED, "attention: dim_head must be 32 or 64");
    });
    MBR_CUDA(cudaGetLastError());
}

void mask_scatter(const float2* spec, const float* masks, int B, int S, int T, int C, int F, const int* rev_off,
                  const int* rev_idx, const float* nbpf, int64_t J, bool zero_dc, float2* y, cudaStream_t st) {
    int64_t total = (int64_t)B * S * T * F * C;
    mask_scatter_kernel<<<nblk(total, 256), 256, 0, st>>>(spec, masks, B, S, T, C, F, rev_off, rev_idx, nbpf, J,
                                                          zero_dc, y);
    MBR_CUDA(cudaGetLastError());
}

void istft_frames(const float2* y, int64_t nsig, int T, const float* window, const float2* twiddle, float spec_scale,
                  float* frames, cudaStream_t st) {
    size_t sm = sizeof(float2) * (kFft / 2 + kFft);
    istft_frames_kernel<<<(unsigned)(nsig * T), 512, sm, st>>>(y, T, window, twiddle, spec_scale, frames);
    MBR_CUDA(cudaGetLastError());
}

void istft_ola(const float* frames, int64_t nsig, int T, int hop, const float* window, int64_t lout, float* out,
               cudaStream_t st) {
    istft_ola_kernel<<<nblk(nsig * lout, 256), 256, 0, st>>>(frames, nsig, T, hop, window, lout, out);
    MBR_CUDA(cudaGetLastError());
}

void prepare_chunks(const float* track, int C, int64_t N, int64_t track_lo, int64_t track_ld, int64_t border,
                    bool padded, const int64_t* starts, int nchunks, int64_t total, int chunk, float* in,
                    cudaStream_t st) {
    int64_t n = (int64_t)nchunks * C * chunk;
    prepare_chunks_kernel<<<nblk(n, 256), 256, 0, st>>>(track, C, N, track_lo, track_ld, border, padded, starts,
                                                        nchunks, total, chunk, in);
    MBR_CUDA(cudaGetLastError());
}

void accumulate_chunks(const float* y, int nchunks, int SC, int64_t lout, const int64_t* starts, int64_t total,
                       int chunk, int fade, float* acc, float* wsum, int64_t acc_lo, int64_t acc_stride,
                       cudaStream_t st) {
    // span bound: the batch covers at most nchunks*chunk samples
    int64_t n = (int64_t)(SC + 1) * ((int64_t)nchunks * chunk);
    accumulate_chunks_kernel<<<nblk(n, 256), 256, 0, st>>>(y, nchunks, SC, lout, starts, total, chunk, fade, acc,
                                                           wsum, acc_lo, acc_stride);
    MBR_CUDA(cudaGetLastError());
}

void add_window(float* acc, float* wsum, int64_t acc_stride, const float* racc, const float* rwsum, int64_t rlen,
                int SC, cudaStream_t st) {
    if (rlen <= 0) return;
    add_window_kernel<<<nblk((int64_t)(SC + 1) * rlen, 256), 256, 0, st>>>(acc, wsum, acc_stride, racc, rwsum, rlen,
                                                                         SC);
    MBR_CUDA(cudaGetLastError());
}

void add_inplace_f32(float* dst, const float* src, int64_t n, cudaStream_t st) {
    add_inplace_kernel<<<nblk(n, 256), 256, 0, st>>>(dst, src, n);
    MBR_CUDA(cudaGetLastError());
}

void normalize_crop(const float* acc, const float* wsum, int SC, int64_t acc_lo, int64_t acc_stride, int64_t p0,
                    int64_t p1, int64_t border, int64_t out_stride, float* out, cudaStream_t st) {
    if (p1 <= p0) return;
    normalize_crop_kernel<<<nblk((int64_t)SC * (p1 - p0), 256), 256, 0, st>>>(acc, wsum, SC, acc_lo, acc_stride, p0,
                                                                              p1, border, out_stride, out);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace mbr
