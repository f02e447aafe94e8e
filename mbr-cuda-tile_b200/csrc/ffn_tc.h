// ffn_tc.h — the feed-forward block of a transformer layer as one tcgen05
// kernel (sm_100a):
//
//   R[m] += GELU(X[m] W1^T + b1) W2^T + b2       (X: M x D, W1: Hd x D, W2: D x Hd)
//
// the reference's fused FFN1 + GELU + FFN2 with the residual add
// (mbr_tile::try_feedforward_fused_residual, src/mbr_cuda_tile.cu:6840, over
// the kernels of src/mbr_ffn12_cutile.cu:226-387; called for every layer at
// src/model_mel_band_roformer.cu:481).  The hidden activations never reach HBM: each 128-row
// tile walks the hidden dimension in 64-wide chunks, H_c = X W1_c^T lands in
// TMEM, eight epilogue warps turn it into GELU(H_c + b1) as 16-bit values in
// shared memory, and the tensor core accumulates O += P_c W2_c^T in TMEM
// (D fp32 columns) while the next chunk's H is computed.  The tile's O is
// reduce-added into the fp32 residual R by TMA.
//
// Work is balanced stream-K style: the tiles' (tile, chunk) units are dealt to
// the CTAs in equal contiguous shares, so a tile may be split between two
// CTAs; both halves reduce-add into R (b2 is added by the half holding chunk 0).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace mbr {
namespace tc {

struct FfnLaunch {
    CUtensorMap tmX, tmW1, tmW2, tmR;
    const float* b1 = nullptr;
    const float* b2 = nullptr;
    // device: per CTA a header {first item, end item, 0, 0}, then the items
    // {row m0, first chunk, end chunk, add b2}
    const int4* items = nullptr;
    int grid = 0;
    int D = 0;
    int64_t M = 0;
    bool ok = false;
};

// True when the fused kernel covers this shape: 16-bit compute, D = 256 or
// 384 (the D fp32 output columns plus two 64-column hidden chunks fit TMEM's
// 512 columns), Hd a multiple of 64, 16-byte aligned operands.
bool ffn_supported(int D, int Hd, int dtype);
// Builds the tensor maps and appends the work list to `items` (host); the
// caller uploads it and points L.items at element `first`.
void ffn_prepare(const void* x, const void* w1, const float* b1, const void* w2, const float* b2, float* R,
                 int64_t M, int D, int Hd, int dtype, std::vector<int4>& items, FfnLaunch& L, size_t& first);
void ffn_launch(const FfnLaunch& L, int dtype, int* d_err, cudaStream_t st);

}  // namespace tc
}  // namespace mbr
