// attention_tc.h — tcgen05 flash attention (time axis and band axis) for sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mbr {
namespace tc {

bool attention_supported(int dim_head);

// Where element d of head h at position p of sequence s lives, in elements
// from q / k / v: d + h*head + p*pos + (s % n_lo)*lo + (s / n_lo)*hi.  It
// covers head-major [nseq][H][L][dh] tensors (head = L*dh, pos = dh, lo =
// H*L*dh, n_lo = nseq, hi = 0) and the token-major output of the fused q|k|v
// projection read in place along either axis.
struct AttnLayout {
    int64_t head, pos, lo, hi;
    int n_lo, n_hi;
};
// Head-major [nseq][H][L][dh].
AttnLayout head_major_layout(int64_t nseq, int H, int L, int dh);

// merged[token][h*dh + d] = softmax(q k^T * scale) v * gate[token][h] (fp16/bf16);
// the token of (sequence, position) follows `mode` (SEQ_TIME / SEQ_FREQ) with NB, T.
void attention(const void* q, const void* k, const void* v, const AttnLayout& lay, int64_t nseq, int H, int L,
               int dh, float scale, const float* gates, int mode, int NB, int T, void* merged, int dtype, int* d_err,
               cudaStream_t st);

}  // namespace tc
}  // namespace mbr
