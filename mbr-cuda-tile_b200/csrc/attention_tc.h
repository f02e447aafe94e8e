// attention_tc.h — tcgen05 flash attention (time axis and band axis) for sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mbr {
namespace tc {

bool attention_supported(int dim_head);
// q, k, v [nseq][H][L][dh] (fp16/bf16) -> merged[token][h*dh + d] = softmax(q k^T * scale) v * gate[token][h]
void attention(const void* q, const void* k, const void* v, int64_t nseq, int H, int L, int dh, float scale,
               const float* gates, int mode, int NB, int T, void* merged, int dtype, int* d_err, cudaStream_t st);

}  // namespace tc
}  // namespace mbr
