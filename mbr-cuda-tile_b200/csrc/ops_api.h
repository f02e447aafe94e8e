// ops_api.h — stand-alone ops in the reference op library's layouts
// (mbr_tile / stft_tile, src/mbr_cuda_tile.h:6-257, src/stft_cuda_tile.h:5-26).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace mbr {
namespace opsapi {

// y = a + b (n % 8 == 0)
void add(const void* a, const void* b, void* y, int64_t n, int dtype, cudaStream_t st);
// y = gelu(x) with the exact erf form (n % 8 == 0)
void gelu(const void* x, void* y, int64_t n, int dtype, cudaStream_t st);
// y[r][h*dh + d] = x[r][h*dh + d] * g[r][h]
void sigmoid_gate(const void* x, const void* g, void* y, int64_t rows, int H, int dh, int dtype, cudaStream_t st);
// y = x * rsqrt(sum x^2 + 1e-12) * gamma * scale per row of D
void rms_norm(const void* x, const float* gamma, void* y, int64_t rows, int D, float scale, int dtype,
              cudaStream_t st);
// x [seqs][L][H][64] rotated by cos/sin [L][32] (interleaved pairs)
void rope(const void* x, const float* cs, const float* sn, void* y, int64_t seqs, int L, int H, int dtype,
          cudaStream_t st);
// Frequency-range tiles of a band map for the transposing band ops: tile i
// covers bins [32 i, 32 i + 32) of all channels and the band-freq entries j
// whose bin lies there.  The per-tile tables sit at fixed offsets (tile i at
// i * stride, i * kBandRowOffs) so a kernel reads them without first reading
// where they are.
constexpr int kBandTileBins = 32;
constexpr int kBandRowOffs = 2 * kBandTileBins + 1;  // row offsets per tile (two channels)
struct BandTiles {
    // per tile, padded to `stride` entries (pads: j = -1, row 0, k 0)
    const int* jl = nullptr;  // band-freq indices j of the tile's entries, ascending
    const int* jr = nullptr;  // tile row of each entry (channel * nf + bin - f0)
    const int* bk = nullptr;  // entries grouped by tile row: tile-local entry positions
    const int* bo = nullptr;  // [kBandRowOffs] per tile: start of each row's group in bk (last = n)
    int count = 0, max_n = 0, stride = 0;
};
// Host construction from the band map (fi: bin*C + channel per entry j).
struct BandTilesHost {
    int count = 0, max_n = 0, stride = 0;
    std::vector<int> jl, jr, bk, bo;
};
BandTilesHost make_band_tiles(const std::vector<int>& fi, int C, int F);

// spec [B][C][F][T] complex -> x [B][T][2J]
void band_gather(const float2* spec, int B, int C, int F, int T, const int* fi, int64_t J, const BandTiles& bt,
                 void* x, int dtype, cudaStream_t st);
// masks [S][B*T][2J] (dtype), spec [B][C][F][T] complex -> out [B][S][C][F][T] complex
void mask_scatter(const float2* spec, const void* masks, int B, int S, int C, int F, int T, const float* nbpf,
                  int64_t J, const BandTiles& bt, float2* out, int dtype, cudaStream_t st);
// q, k, v [B][H][N][D] -> out [B][N][H*D] = softmax(q k^T * scale) v, times
// gates [B][N][H] when non-null (scaled_dot_product_attention followed by
// apply_gates_and_merge_heads).  16-bit dtypes with D = 64 run the tcgen05
// kernel and return after the stream drains (a pipeline timeout throws).
void attention(const void* q, const void* k, const void* v, int64_t B, int H, int N, int D, float scale,
               const float* gates, void* out, int dtype, cudaStream_t st);
// y [rows][out] = act(x [rows][in] . w[out][in]^T + bias[out]), act 0 none,
// 1 exact GELU, 2 tanh; y has the input dtype.  16-bit inputs whose shapes
// meet the TMA rules (in % 16 == 0, out % 8 == 0, 16-byte aligned rows) run
// the tcgen05 GEMM, everything else the CUDA-core GEMM; both return after the
// stream drains (the launch descriptors live in per-device scratch).
void linear(const void* x, const void* w, const float* bias, void* y, int64_t rows, int in, int out, int act,
            int dtype, cudaStream_t st);
// resid += GELU(x w1^T + b1) w2^T + b2 through the fused tcgen05 FFN kernel
// (dim 256 / 384, hidden % 64 == 0, fp16 / bf16); returns after the stream drains.
void ffn(const void* x, const void* w1, const float* b1, const void* w2, const float* b2, float* resid, int64_t rows,
         int dim, int hidden, int dtype, cudaStream_t st);
// STFT frames of an L-sample signal (center, reflect pad n_fft/2)
int64_t stft_frames(int64_t L, int hop);
// sig [n][L] -> out [n][1025][T] complex (n_fft 2048, periodic Hann, onesided)
void stft(const float* sig, int64_t nsig, int64_t L, int hop, float2* out, cudaStream_t st);
// spec [n][1025][T] complex -> out [n][lout]; frames is scratch of n*T*2048 floats
void istft(const float2* spec, int64_t nsig, int T, int hop, float* frames, int64_t lout, float* out,
           cudaStream_t st);

// Size of the file-scope frame scratch of the allocation-free iSTFT: 16 MiB,
// i.e. n * T <= 2048 frames of 2048 samples per call.
constexpr int64_t kIstftStaticFloats = (int64_t)4 << 20;
constexpr int kMaxDevices = 64;
// Device address of that scratch on the current device (looked up once per
// device with cudaGetSymbolAddress).
float* istft_static_scratch();

}  // namespace opsapi
}  // namespace mbr
