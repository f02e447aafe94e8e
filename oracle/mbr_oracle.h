/*
 * mbr_oracle.h — C interface of the CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a scalar/threaded CPU restatement of the
 * reference MelBandRoformer forward (baicai-1145/MBR-CUDA-Tile,
 * src/model_mel_band_roformer.cu:682-845) and of its chunk driver
 * (src/inference_app.cpp:46-232).  It is the parity checker for the CUDA
 * product and the CPU baseline timed by bench.py.  The product never links,
 * loads or calls it.
 *
 * Precision: activations are stored as fp32, every reduction (dot products,
 * norms, softmax sums, FFT butterflies) is carried in fp64.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Last error message of the calling thread ("" when none). */
const char* orc_last_error(void);

/* Number of worker threads used by the oracle (0 = hardware concurrency). */
void orc_set_threads(int n);
int orc_get_threads(void);

/* Mel band map (published MelBandRoformer construction over a slaney mel
 * filterbank, see mbr_oracle.cpp).  freq_indices has capacity `cap`;
 * *n_out receives its length.  nfpb: [num_bands], nbpf: [n_fft/2+1].
 * Returns 0 on success. */
int orc_band_map(int sample_rate, int n_fft, int num_bands, int stereo,
                 int64_t* freq_indices, int64_t cap, int64_t* n_out,
                 int64_t* nfpb, int64_t* nbpf);

/* STFT of `n_sig` signals of length L (center=True, reflect pad n_fft/2,
 * periodic Hann, onesided, unnormalised).  out: [n_sig, n_fft/2+1, T, 2]
 * with T = L/hop + 1.  Returns 0 on success. */
int orc_stft(const float* sig, int64_t n_sig, int64_t L, int n_fft, int hop,
             float* out, int64_t* T_out);

/* Inverse of orc_stft: spec [n_sig, n_fft/2+1, T, 2] -> out [n_sig, (T-1)*hop]
 * (or `length` samples when length > 0).  Returns 0 on success. */
int orc_istft(const float* spec, int64_t n_sig, int64_t T, int n_fft, int hop,
              int64_t length, float* out, int64_t* len_out);

/* Scaled dot-product attention of nsh independent (sequence, head) slices:
 * q, k, v, out [nsh][L][dh]; out = softmax(q k^T * scale) v with fp64 sums and
 * an exact softmax (the attention inside orc_forward, exposed alone so it can
 * be checked against the reference's own attention validators). */
int orc_attention(const float* q, const float* k, const float* v, int64_t nsh, int64_t L, int dh, float scale,
                  float* out);

/* Model handle: loads a .csm file.  weight_dtype: 0 = use weights as stored,
 * 1 = round every 2-D fp32 tensor to fp16, 3 = round to bf16 (this restates
 * ModelWeights::convert_linear_weights_to_{fp16,bf16}, src/weights.cu:511-540),
 * 4 = the reference's default --bf16 path: weights, biases, norm gammas and
 * rotary tables in bf16, and every activation rounded to bf16 where that path
 * stores it (GEMM accumulators stay fp32 / fp64). */
void* orc_model_load(const char* csm_path, int weight_dtype);
void orc_model_free(void* model);
/* Query: 0 dim, 1 depth, 2 num_stems, 3 audio_channels, 4 num_bands,
 * 5 sample_rate, 6 chunk_size, 7 num_overlap, 8 n_fft, 9 hop, 10 heads,
 * 11 dim_head, 12 total band-freqs (J), 13 zero_dc, 14 match_input_audio_length */
int64_t orc_model_info(void* model, int what);

/* One forward over a chunk batch: audio [B, C, L] -> out [B, S, C, Lout]
 * (Lout written to *lout; the caller sizes out for Lout <= L).  */
int orc_forward(void* model, const float* audio, int B, int64_t L, float* out,
                int64_t* lout);

/* Intermediate taps of one forward (for per-stage parity):
 *  0 band-split output [B,T,NB,D]; 1 after depth block 0 [B,T,NB,D];
 *  2 final residual stream [B,T,NB,D]; 3 stem-0 mask [B,T,2J];
 *  4 masked spectrum before iSTFT [B*S*C, F, T, 2].
 * `buf` receives the tap; *n receives its element count (call once with
 * buf == NULL to size it). */
int orc_forward_tap(void* model, const float* audio, int B, int64_t L, int tap,
                    float* buf, int64_t* n);

/* Full track separation (restates process_chunked / run_inference):
 * track [C, N] -> out [S, C, N].  overlap: <=0 uses the config's num_overlap,
 * (0,1) = overlap ratio, >=1 = num_overlap.  chunk_batch >= 1. */
int orc_separate(void* model, const float* track, int64_t N, float overlap,
                 int chunk_batch, float* out);

/* Chunk plan of process_chunked: writes up to cap chunk starts; returns the
 * count (or -1).  border and total receive the reflect border and the padded
 * length.  step from resolve_step (src/inference_app.cpp:46-57). */
int64_t orc_chunk_plan(int64_t N, int chunk_size, float overlap, int default_overlap,
                       int64_t* starts, int64_t cap, int64_t* step, int64_t* border,
                       int64_t* total);

#ifdef __cplusplus
}
#endif
