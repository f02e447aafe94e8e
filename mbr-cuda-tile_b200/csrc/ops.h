// ops.h — host launchers of the B200 kernels used by the MelBandRoformer forward.
//
// Layouts (B chunk batch, C audio channels, T frames, F = n_fft/2+1 bins,
// FC = F*C stereo-interleaved bins (f-major, channel-minor), NB bands,
// D model dim, H heads, dh head dim, DI = H*dh, J band-freqs, MT = B*T,
// M = MT*NB tokens):
//   spec   [B][T][FC]             float2  (STFT output, time-major)
//   xb     [MT][KP]               T       (band-gathered, band-normed; band b at
//                                          columns kofs[b].., zero padded to kofs[b+1])
//   R      [B][T][NB][D]          fp32    residual stream; token m = (b*T+t)*NB+k
//   q,k,v  [nseq][H][L][dh]       T       per-sequence head-major
//   masks  [S][MT][2J]            fp32    (band-freq j at 2j, 2j+1 = re, im)
//   y      [B][S][C][T][F]        float2  masked spectrum, frame rows for the iSTFT
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mbr {
namespace ops {

// Token mapping of a sequence position (attention / RoPE):
//   SEQ_TIME: sequence s = b*NB + k runs over t;  SEQ_FREQ: s = b*T + t runs over k.
enum SeqMode { SEQ_TIME = 0, SEQ_FREQ = 1 };

void stft(const float* sig, int B, int C, int64_t L, int hop, const float* window, const float2* twiddle,
          float norm, float2* spec, int T, cudaStream_t st);

void band_gather_norm(const float2* spec, int64_t MT, int FC, const int* fi, const int* band_jofs,
                      const int* band_kofs, const float* gamma, int NB, void* xb, int64_t KP, int dtype,
                      cudaStream_t st);

// y = x * rsqrt(sum x^2 + 1e-12) * gamma * scale, row-wise over D.
//  xn (dtype) receives y (row map: identity, or band-major k*MT + bt when band_major_mt > 0);
//  r_out (fp32, may alias R) receives y too when non-null;
//  gates[m][h] = sigmoid(y . wg[h] + bg[h]) when wg is non-null.
//  With gamma2, r_out still receives y but xn and the gates are taken from
//  y2 = RMSNorm(y) * gamma2 * scale (a block's final norm fused with the next
//  block's pre-norm).
void rms_norm(const float* R, int64_t M, int D, const float* gamma, float scale, void* xn, int dtype,
              int64_t band_major_mt, int NB, float* r_out, const float* wg, const float* bg, int H, float* gates,
              cudaStream_t st, const float* gamma2 = nullptr);

// q, k (rotated) and, if v is non-null, v -> [nseq][H][L][dh].
void rope_scatter(const void* qkv, int64_t M, int H, int dh, const float* cos_t, const float* sin_t, int mode,
                  int NB, int T, void* q, void* k, void* v, int dtype, cudaStream_t st);

void attention_simt(const void* q, const void* k, const void* v, int64_t nseq, int H, int L, int dh, float scale,
                    const float* gates, int mode, int NB, int T, void* merged, int dtype, cudaStream_t st);

// Grouped GEMM: C_g[m][n] = epi( sum_k A_g[m*lda+k] * B_g[n*ldb+k] + bias_g[n] ).
struct GemmGroup {
    const void* A;
    const void* B;
    void* C;
    const float* bias;
    int64_t lda, ldb, ldc;
    int M, N, K;
    int a_row0, b_row0;  // row offsets of this group inside the A / B tensor maps
    int k_col0;          // column offset of this group's K range inside A and B
    int c_group;         // index of this group's C block in a [groups][rows][cols] output map
};
enum Epilogue {
    EPI_F32 = 0,      // C (fp32) = acc + bias
    EPI_T = 1,        // C (dtype) = acc + bias
    EPI_ADD_F32 = 2,  // C (fp32) += acc + bias
    EPI_GELU_T = 3,   // C (dtype) = gelu(acc + bias)
    EPI_TANH_T = 4,   // C (dtype) = tanh(acc + bias)
    EPI_GLU_F32 = 5,  // C[m][n/2] (fp32) = (acc_n + b_n) * sigmoid(acc_{n+1} + b_{n+1}), n even
    EPI_QKV = 6,      // RoPE(q, k) + scatter of q, k, v into [seq][H][L][64] (tensor-core path only)
    EPI_ROPE_T = 7,   // C (dtype) = acc with RoPE on the q and k sections, token-major (tensor-core path only)
};
void gemm_simt(const GemmGroup* d_groups, int ngroups, int maxM, int maxN, int dtype, int epi, cudaStream_t st);

void mask_scatter(const float2* spec, const float* masks, int B, int S, int T, int C, int F, const int* rev_off,
                  const int* rev_idx, const float* nbpf, int64_t J, bool zero_dc, float2* y, cudaStream_t st);

void istft_frames(const float2* y, int64_t nsig, int T, const float* window, const float2* twiddle, float spec_scale,
                  float* frames, cudaStream_t st);
// Overlap-add in gather form, division by the window-square sum, centre crop and
// the length rule.  out [nsig][lout].
void istft_ola(const float* frames, int64_t nsig, int T, int hop, const float* window, int64_t lout, float* out,
               cudaStream_t st);

// Chunk driver kernels (process_chunked restated on the device).
// prepare_chunks reads track samples [track_lo, track_lo + track_ld) of each
// channel from `track` (row stride track_ld): the whole track (0, N) or a
// shard's input window.
void prepare_chunks(const float* track, int C, int64_t N, int64_t track_lo, int64_t track_ld, int64_t border,
                    bool padded, const int64_t* starts, int nchunks, int64_t total, int chunk, float* in,
                    cudaStream_t st);
// acc [SC][acc_stride] / wsum [acc_stride] hold padded samples [acc_lo, acc_lo + acc_stride).
void accumulate_chunks(const float* y, int nchunks, int SC, int64_t lout, const int64_t* starts, int64_t total,
                       int chunk, int fade, float* acc, float* wsum, int64_t acc_lo, int64_t acc_stride,
                       cudaStream_t st);
// acc[o][q] += racc[o][q], wsum[q] += rwsum[q] for q < rlen.
void add_window(float* acc, float* wsum, int64_t acc_stride, const float* racc, const float* rwsum, int64_t rlen,
                int SC, cudaStream_t st);
// dst[i] += src[i] (fp32), used for the optional skip connections.
void add_inplace_f32(float* dst, const float* src, int64_t n, cudaStream_t st);

// out[o][p - border] = acc[o][p - acc_lo] / wsum[p - acc_lo] (where > 1e-8) for p in [p0, p1).
void normalize_crop(const float* acc, const float* wsum, int SC, int64_t acc_lo, int64_t acc_stride, int64_t p0,
                    int64_t p1, int64_t border, int64_t out_stride, float* out, cudaStream_t st);

}  // namespace ops
}  // namespace mbr
