/*
 * mbr_b200.h — C ABI of the B200-native MelBandRoformer separator.
 *
 * The reference (baicai-1145/MBR-CUDA-Tile) exposes its hot path only as C++
 * (cudasep::app::load_model / run_inference, MelBandRoformer::load / forward,
 * the mbr_tile / stft_tile / chunk_tile op namespaces).  This header is the
 * drop-in boundary a maintainer binds from any FFI: plain pointers, sizes and
 * status codes, no C++ or CUDA types.  Each entry point names the reference
 * interface (file:line) it replaces.
 *
 * Conventions
 *  - Every function returns MBR_OK (0) or an MBR_ERR_* code; the message of
 *    the last failure on the calling thread is mbr_last_error().
 *  - "d_" pointers are device memory on the handle's device, "h_" pointers are
 *    host memory.  All buffers are caller owned; the library owns only its
 *    weights and workspaces (one set per handle).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *    device entry points enqueue work and return without synchronising.
 *  - One handle per host thread at a time; handles on different devices run
 *    concurrently.
 */
#ifndef MBR_B200_H
#define MBR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MBR_API __attribute__((visibility("default")))

/* status codes */
#define MBR_OK 0
#define MBR_ERR_INVALID 1     /* bad argument / shape */
#define MBR_ERR_CUDA 2        /* CUDA runtime failure */
#define MBR_ERR_IO 3          /* file missing or malformed (.csm) */
#define MBR_ERR_UNSUPPORTED 4 /* configuration the kernels do not cover */
#define MBR_ERR_OOM 5         /* device allocation failed */
#define MBR_ERR_TIMEOUT 6     /* a bounded wait gave up */

/* compute dtypes (the .csm dtype codes) */
#define MBR_FP32 0
#define MBR_FP16 1
#define MBR_BF16 3

/* mbr_get_info keys */
#define MBR_INFO_DIM 0
#define MBR_INFO_DEPTH 1
#define MBR_INFO_NUM_STEMS 2
#define MBR_INFO_CHANNELS 3
#define MBR_INFO_NUM_BANDS 4
#define MBR_INFO_SAMPLE_RATE 5
#define MBR_INFO_CHUNK_SIZE 6
#define MBR_INFO_NUM_OVERLAP 7
#define MBR_INFO_HEADS 8
#define MBR_INFO_DIM_HEAD 9
#define MBR_INFO_BAND_FREQS 10
#define MBR_INFO_DTYPE 11
#define MBR_INFO_DEVICE 12
#define MBR_INFO_HOP 13

/* kernel backends for mbr_set_backend */
#define MBR_BACKEND_SIMT 0 /* CUDA-core kernels (fp32 path, cross-check) */
#define MBR_BACKEND_TC 1   /* tcgen05 tensor-core kernels (fp16 / bf16) */
#define MBR_BACKEND_TC_DIRECT 2 /* GEMMs only: tensor cores, epilogue stores from registers */

typedef struct mbr_handle mbr_handle;

/* Message of the last failed call on this thread ("" if none). */
MBR_API const char* mbr_last_error(void);

/* Library ABI version (major * 100 + minor). */
MBR_API int mbr_version(void);

/* Load a .csm checkpoint onto `device` with compute dtype MBR_FP32 / MBR_FP16 /
 * MBR_BF16 (2-D fp32 weights are rounded to the dtype, as --fp16/--bf16 do).
 * Replaces cudasep::app::load_model (src/inference_app.cpp:258-311) and
 * MelBandRoformer::load (src/model_mel_band_roformer.cu:75-264). */
MBR_API int mbr_create(const char* csm_path, int device, int dtype, mbr_handle** out);

/* Release the handle, its weights and workspaces. */
MBR_API void mbr_destroy(mbr_handle* h);

/* Config / handle queries (MBR_INFO_*).  Replaces MelBandRoformer::config()
 * (src/model_mel_band_roformer.h:46) and LoadedModel fields
 * (src/inference_app.h:16-30). */
MBR_API int mbr_get_info(mbr_handle* h, int what, int64_t* value);

/* Output samples per channel of a forward over `L` input samples. */
MBR_API int mbr_output_length(mbr_handle* h, int64_t L, int64_t* lout);

/* One forward over a chunk batch: d_audio [B][C][L] -> d_out [B][S][C][lout]
 * (S = num_stems; lout from mbr_output_length).  Replaces
 * MelBandRoformer::forward (src/model_mel_band_roformer.cu:682-845). */
MBR_API int mbr_forward_chunk(mbr_handle* h, const float* d_audio, int B, int64_t L, float* d_out, void* stream);

/* Per-stage tap of one forward, for parity checks (fp32 copy into d_tap):
 * 0 band-split output [B][T][NB][D], 1 residual stream after depth block 0,
 * 2 final residual stream, 3 stem-0 mask [B*T][2J], 4 masked spectrum
 * [B][S][C][T][F][2].  With d_tap == NULL only *n is set. */
MBR_API int mbr_forward_tap(mbr_handle* h, const float* d_audio, int B, int64_t L, int tap, float* d_tap,
                            int64_t* n, void* stream);

/* Whole-track separation with inputs and outputs in device memory:
 * d_track [C][N] -> d_out [S][C][N].  overlap <= 0 uses the checkpoint's
 * num_overlap, (0,1) is an overlap ratio, >= 1 a num_overlap; chunk_batch >= 1.
 * Replaces process_chunked (src/inference_app.cpp:72-232) and the timed part
 * of run_inference (:313-357). */
MBR_API int mbr_separate_device(mbr_handle* h, const float* d_track, int64_t N, float overlap, int chunk_batch,
                                float* d_out, void* stream);

/* Whole-track separation from host memory (copies in, separates, copies out,
 * synchronises): h_track [C][N] -> h_out [S][C][N].  On one GPU the copies
 * overlap the chunks: each chunk batch's new input samples are uploaded on a
 * copy stream ahead of it, and every output range that no later chunk
 * touches is normalised and downloaded while later batches run (pinned host
 * buffers make these copies asynchronous).  With n_gpus > 1 the chunk list is
 * split into contiguous ranges run on devices device .. device+n_gpus-1 in
 * parallel; each device receives only its input window and holds only its
 * own output range, and only the overlap-add boundaries are exchanged (peer
 * copies, all at once when every range holds enough chunks that no boundary
 * depends on another).  Replaces run_inference
 * (src/inference_app.cpp:313-357; its chunk-batch loop :92-128) without the
 * WAV file I/O. */
MBR_API int mbr_separate(mbr_handle* h, const float* h_track, int64_t N, float overlap, int chunk_batch, int n_gpus,
                         float* h_out);

/* Sharded separation for one-process-per-GPU callers (e.g. torch.distributed).
 * mbr_shard_info: for track length N and (rank, world) gives the chunk range
 * [c0, c1), the padded-sample window [lo, hi) the shard accumulates, the
 * part [send_lo, hi) it must send to rank+1, and the track range
 * [out_lo, out_hi) it finalises.  Values are written to info[0..7] as
 * c0, c1, lo, hi, send_lo, out_lo, out_hi, n_chunks. */
MBR_API int mbr_shard_info(mbr_handle* h, int64_t N, float overlap, int rank, int world, int64_t* info);
/* The same shard plan without a handle or GPU (host arithmetic only), for a
 * track of N samples, the checkpoint's chunk_size and default num_overlap:
 * info[0..7] as in mbr_shard_info, info[8..10] = step, border, padded length. */
MBR_API int mbr_plan_shard(int64_t N, int chunk_size, float overlap, int default_overlap, int rank, int world,
                           int64_t* info);
/* Runs the shard's chunks: d_acc [S*C][hi-lo], d_wsum [hi-lo] (overwritten). */
MBR_API int mbr_shard_run(mbr_handle* h, const float* d_track, int64_t N, float overlap, int chunk_batch, int rank,
                          int world, float* d_acc, float* d_wsum, void* stream);
/* The track samples [*in_lo, *in_hi) a shard reads (its chunks through the
 * reflect padding), so that a rank uploads only that window.  The
 * reference's process_chunked reads the whole padded track
 * (src/inference_app.cpp:78-89); this is its per-rank restriction. */
MBR_API int mbr_shard_window(mbr_handle* h, int64_t N, float overlap, int rank, int world, int64_t* in_lo,
                             int64_t* in_hi);
/* mbr_shard_window without a handle or GPU (host arithmetic only), for the
 * checkpoint's chunk_size and default num_overlap. */
MBR_API int mbr_plan_shard_window(int64_t N, int chunk_size, float overlap, int default_overlap, int rank, int world,
                                  int64_t* in_lo, int64_t* in_hi);
/* mbr_shard_run over a track window: d_window [C][win_len] holds track
 * samples [win_lo, win_lo + win_len) of each channel and must cover the
 * shard's mbr_shard_window. */
MBR_API int mbr_shard_run_window(mbr_handle* h, const float* d_window, int64_t win_lo, int64_t win_len, int64_t N,
                                 float overlap, int chunk_batch, int rank, int world, float* d_acc, float* d_wsum,
                                 void* stream);
/* Adds the previous rank's boundary (d_recv_acc [S*C][recv_len],
 * d_recv_wsum [recv_len], recv_len = previous hi - this lo) into the
 * shard's accumulators (call before sending this shard's own boundary). */
MBR_API int mbr_shard_add_boundary(mbr_handle* h, int64_t N, float overlap, int rank, int world, float* d_acc,
                                   float* d_wsum, const float* d_recv_acc, const float* d_recv_wsum,
                                   int64_t recv_len, void* stream);
/* Normalises the shard's own range into d_out [S*C][out_stride] at columns
 * [out_lo, out_hi) (track coordinates); only those columns are written, so a
 * caller holding just its own range passes its buffer's address minus out_lo
 * columns with out_stride = out_hi - out_lo. */
MBR_API int mbr_shard_finalize(mbr_handle* h, int64_t N, float overlap, int rank, int world, float* d_acc,
                               float* d_wsum, float* d_out, int64_t out_stride, void* stream);

/* CUDA-graph replay of the chunk forward (on by default): the first forward
 * with a given input shape and input/output buffer pair runs eagerly and is
 * captured; later ones replay the graph.  Streams that cannot be captured (the
 * legacy default stream, a stream the caller is capturing) always run eagerly.
 * This is the "graph capture per (B, T)" step of the chunk-batched pipeline
 * (src/inference_app.cpp:92-128 runs every chunk op by op). */
MBR_API int mbr_set_graphs(mbr_handle* h, int enable);

/* Kernel backend selection (MBR_BACKEND_*) for the GEMMs and the attention. */
MBR_API int mbr_set_backend(mbr_handle* h, int gemm, int attention);

/* Kernel launches issued by the last forward / separation on this handle. */
MBR_API int mbr_last_launches(mbr_handle* h, int64_t* n);

/* Waits for the handle's device and reports a kernel-side failure: the
 * tensor-core kernels bound every pipeline wait and, instead of hanging, set an
 * error word that this call turns into MBR_ERR_TIMEOUT.  No reference
 * counterpart (the reference's kernels have no device-side waits). */
MBR_API int mbr_sync_check(mbr_handle* h);

/* Per-kernel-class profiler (CUDA events on the launching stream).
 * Classes: 0 stft, 1 band gather+norm, 2 band-split GEMM, 3 rms norms,
 * 4 QKV GEMM, 5 rope scatter, 6 time attention, 7 band attention,
 * 8 out-proj GEMM, 9 FFN1 GEMM, 10 FFN2 GEMM, 11 mask hidden GEMMs,
 * 12 mask output GEMM, 13 mask scatter, 14 iSTFT.  Replaces the out-of-band
 * nsys summaries of the reference (bench/nsys_kernel_summary.sh). */
MBR_API int mbr_profile_enable(mbr_handle* h, int on);
MBR_API int mbr_profile_read(mbr_handle* h, int kind, double* ms, int64_t* count);

/* ---- WAV I/O (host only) -------------------------------------------------
 * Replaces load_wav / save_wav (src/audio_io.h:14-18, src/audio_io.cpp:59-334):
 * PCM 16/24/32-bit and float32 input (WAVE_FORMAT_EXTENSIBLE included),
 * integer PCM scaled by 1/2^(bits-1); output is float32 WAV.  Samples are
 * planar [channels][frames]. */
MBR_API int mbr_wav_info(const char* path, int* sample_rate, int* channels, int64_t* frames);
MBR_API int mbr_wav_read(const char* path, float* h_planar, int64_t capacity);
MBR_API int mbr_wav_write(const char* path, const float* h_planar, int channels, int64_t frames, int sample_rate);

/* ---- WAV I/O with the sample conversion on the GPU ------------------------
 * The reference converts samples on the host (src/audio_io.cpp:200-334).
 * mbr_pcm_to_planar: interleaved PCM bytes already in device memory
 * ([frames][channels], 16 / 24 / 32-bit integer or, with is_float, 32-bit
 * float) -> planar fp32 d_planar [channels][frames], integer PCM scaled by
 * 1/2^(bits-1): the same values the host reader gives.
 * mbr_wav_read_device: parses the file on the host, uploads its data chunk
 * as raw bytes and converts it on the device into d_planar (capacity in
 * floats); with d_planar == NULL it only reports the format.  Synchronises
 * `stream` before returning.
 * mbr_wav_write_device: interleaves d_planar [channels][frames] on the device
 * and writes a float32 WAV (synchronises `stream`). */
MBR_API int mbr_pcm_to_planar(const void* d_pcm, int64_t frames, int channels, int bits, int is_float,
                              float* d_planar, void* stream);
MBR_API int mbr_wav_read_device(const char* path, float* d_planar, int64_t capacity, int* sample_rate, int* channels,
                                int64_t* frames, void* stream);
MBR_API int mbr_wav_write_device(const char* path, const float* d_planar, int channels, int64_t frames,
                                 int sample_rate, void* stream);

/* ---- stand-alone ops in the reference op library's layouts ------------
 * All buffers are device memory; dtype is MBR_FP32 / MBR_FP16 / MBR_BF16;
 * element counts of the elementwise ops are multiples of 8. */

/* y = x * rsqrt(sum_d x^2 + 1e-12) * gamma * scale over rows of `dim`
 * (x, y: dtype; gamma: fp32).  Replaces mbr_tile::rms_norm
 * (src/mbr_cuda_tile.h:34; kernels src/mbr_cuda_tile.cu:4791-5091). */
MBR_API int mbr_op_rms_norm(const void* d_x, const float* d_gamma, void* d_y, int64_t rows, int dim, float scale,
                            int dtype, void* stream);

/* y = a + b (residual add).  Replaces Tensor::add_ (src/tensor.h:117) and
 * try_residual_add_bf16_cutile (src/mbr_residual_cutile.cu:71-94). */
MBR_API int mbr_op_add(const void* d_a, const void* d_b, void* d_y, int64_t n, int dtype, void* stream);

/* y = 0.5 x (1 + erf(x / sqrt 2)).  The activation of mbr_tile::linear_gelu
 * (src/mbr_cuda_tile.h:78; the reference evaluates erf with polynomial fits,
 * src/mbr_cuda_tile.cu:566-690). */
MBR_API int mbr_op_gelu(const void* d_x, void* d_y, int64_t n, int dtype, void* stream);

/* y[r][h*dh + d] = x[r][h*dh + d] * gate[r][h] (gate already sigmoid'ed).
 * Replaces apply_gates_and_merge_heads (src/mbr_cuda_tile.h:29-30). */
MBR_API int mbr_op_sigmoid_gate(const void* d_x, const void* d_gate, void* d_y, int64_t rows, int heads,
                                int dim_head, int dtype, void* stream);

/* RoPE over positions: x [seqs][L][heads][64], interleaved pairs (2i, 2i+1) of
 * position p rotated by (d_cos, d_sin)[p][i] ([L][32] fp32).  Replaces the
 * rotary part of split_qkv_heads_rotary (src/mbr_cuda_tile.h:8-10). */
MBR_API int mbr_op_rope(const void* d_x, const float* d_cos, const float* d_sin, void* d_y, int64_t seqs, int L,
                        int heads, int dtype, void* stream);

/* Linear layer: y [rows][out] = act(x [rows][in] . w[out][in]^T + bias[out])
 * with act MBR_ACT_NONE / MBR_ACT_GELU (exact erf form) / MBR_ACT_TANH; d_bias
 * (fp32) may be null; x, w, y have the given dtype.  Replaces linear and
 * linear_gelu (src/mbr_cuda_tile.h:63,68; src/mbr_cuda_tile.cu:6851,6926).
 * fp16/bf16 with in % 16 == 0, out % 8 == 0 and 16-byte aligned pointers run
 * the tcgen05 GEMM, other shapes and fp32 the CUDA-core GEMM; the call returns
 * after the stream drains. */
#define MBR_ACT_NONE 0
#define MBR_ACT_GELU 1
#define MBR_ACT_TANH 2
MBR_API int mbr_op_linear(const void* d_x, const void* d_w, const float* d_bias, void* d_y, int64_t rows, int in,
                          int out, int act, int dtype, void* stream);

/* Feed-forward block with its residual add, as one tcgen05 kernel:
 * resid [rows][dim] (fp32) += GELU(x . w1^T + b1) . w2^T + b2, with x
 * [rows][dim], w1 [hidden][dim], w2 [dim][hidden] in dtype (fp16 / bf16), b1
 * [hidden] and b2 [dim] fp32, GELU the exact erf form, the hidden activations
 * rounded to dtype (they never reach device memory).  Replaces
 * try_feedforward_fused_residual (src/mbr_cuda_tile.cu:6840) over the fused
 * FFN kernels of src/mbr_ffn12_cutile.cu.  Needs dim 256 or 384, hidden a
 * multiple of 64 and 16-byte aligned pointers (else MBR_ERR_UNSUPPORTED);
 * the call returns after the stream drains. */
MBR_API int mbr_op_ffn(const void* d_x, const void* d_w1, const float* d_b1, const void* d_w2, const float* d_b2,
                       float* d_resid, int64_t rows, int dim, int hidden, int dtype, void* stream);

/* Multi-head attention with the head merge: q, k, v [B][heads][N][dim_head]
 * (dtype), out [B][N][heads*dim_head] = softmax(q k^T * scale) v, multiplied
 * by gates [B][N][heads] (fp32, already sigmoid'ed) when d_gates is non-null.
 * scale 0 means 1/sqrt(dim_head).  Replaces scaled_dot_product_attention
 * (src/mbr_cuda_tile.h:42-45, src/mbr_cuda_tile.cu:6530) followed by
 * apply_gates_and_merge_heads (src/mbr_cuda_tile.h:28-29).  fp16/bf16 with
 * dim_head 64 run the tcgen05 flash-attention kernel and return after the
 * stream drains (a pipeline timeout is MBR_ERR_TIMEOUT); fp32 or dim_head 32
 * run the CUDA-core kernel asynchronously. */
MBR_API int mbr_op_attention(const void* d_q, const void* d_k, const void* d_v, int64_t B, int heads, int N,
                             int dim_head, float scale, const float* d_gates, void* d_out, int dtype, void* stream);

/* Host tables of MelBandRoformer::compute_rotary_cos_sin
 * (src/model_mel_band_roformer.cu:270-300): h_cos, h_sin [L][dim_head/2]. */
MBR_API int mbr_rope_tables(int L, int dim_head, float* h_cos, float* h_sin);

/* Band gather with the handle's band map: d_spec [B][C][1025][T] complex ->
 * d_x [B][T][2J] (the stereo merge of src/model_mel_band_roformer.cu:714-725
 * folded in).  Replaces gather_freqs_fold_complex (src/mbr_cuda_tile.h:12). */
MBR_API int mbr_op_band_gather(mbr_handle* h, const float* d_spec, int B, int T, void* d_x, int dtype,
                               void* stream);

/* Mask scatter-average with the handle's band map: d_masks [S][B*T][2J]
 * (dtype), d_spec [B][C][1025][T] complex -> d_out [B][S][C][1025][T]
 * complex (fp32).  Replaces apply_mask_and_scatter (src/mbr_cuda_tile.h:230-242). */
MBR_API int mbr_op_mask_scatter(mbr_handle* h, const float* d_spec, const void* d_masks, int B, int S, int T,
                                float* d_out, int dtype, void* stream);

/* STFT (n_fft 2048, periodic Hann, center reflect pad, onesided):
 * d_sig [n][L] -> d_spec [n][1025][T][2], T = L / hop + 1.  Replaces
 * stft_tile::stft (src/stft_cuda_tile.h:9-15). */
MBR_API int mbr_op_stft(const float* d_sig, int64_t n, int64_t L, int hop, float* d_spec, void* stream);

/* iSTFT: d_spec [n][1025][T][2] -> d_out [n][lout], lout = length > 0 ? length
 * : (T - 1) * hop.  Its n*T*2048-float frame scratch comes from the
 * stream-ordered allocator.  Replaces stft_tile::istft (src/stft_cuda_tile.h:17-24). */
MBR_API int mbr_op_istft(const float* d_spec, int64_t n, int T, int hop, int64_t length, float* d_out,
                         void* stream);

/* iSTFT that allocates no device memory; same arguments and result as
 * mbr_op_istft.  No counterpart in the reference: it is for callers that may
 * not call cudaMalloc or the stream-ordered allocator at run time, such as a
 * real-time audio host whose processing thread must not block on an allocator
 * (cudaMalloc can synchronise the device) or a service that reserves all GPU
 * memory up front and forbids later allocations.
 * Limits and rules:
 *  - the frame scratch is a fixed 16 MiB array inside the library, so
 *    n * T <= 2048 (e.g. one stereo 8 s chunk, 2 x 801 frames); larger calls
 *    fail with MBR_ERR_INVALID.  Every GPU that loads the library holds this
 *    array until the process exits.
 *  - the device that is current when the call is made must own d_spec,
 *    d_out and the stream: the array used is the current device's copy.
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current, and with CUDA's lazy
 *    module loading it may also load the library's module and reserve the
 *    16 MiB array there, which can allocate and block.  So make that first
 *    call in set-up code, before any real-time work and before any stream
 *    capture.
 *  - all calls share the one array: calls whose work overlaps on the GPU
 *    (different streams without ordering, or different host threads) race.
 *    Every frame the call reads is written by the same call first, so nothing
 *    needs clearing between calls. */
MBR_API int mbr_op_istft_noalloc(const float* d_spec, int64_t n, int T, int hop, int64_t length, float* d_out,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MBR_B200_H */
