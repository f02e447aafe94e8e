// separator.h — long-track separation by overlapped chunks (device resident).
//
// Restates the reference chunk driver (src/inference_app.cpp:46-232,
// resolve_step + process_chunked, and the single-chunk branch of run_inference
// :330-344) with the chunk gather, the fade-weighted overlap-add and the final
// normalisation done by kernels on one stream; no host round trips between
// chunks.  The chunk list can be split into contiguous ranges (shards) so that
// several GPUs each run a range and exchange only the overlap-add boundary.
#pragma once

#include <stdint.h>

#include <vector>

#include "model.h"

namespace mbr {

int resolve_step(int chunk_size, float overlap, int default_overlap);

struct ChunkPlan {
    int64_t N = 0;       // input samples per channel
    int chunk = 0, step = 0, fade = 0;
    int64_t border = 0;  // reflect padding on each side (0 when not padded)
    bool padded = false;
    int64_t total = 0;   // padded length
    bool single = false; // N <= chunk: one forward over the whole input
    std::vector<int64_t> starts;
};
ChunkPlan make_chunk_plan(int64_t N, int chunk_size, float overlap, int default_overlap);

// A contiguous chunk range [c0, c1) and the padded-sample windows it touches.
struct Shard {
    int c0 = 0, c1 = 0;
    int64_t lo = 0, hi = 0;          // samples the range writes: [lo, hi)
    int64_t own_lo = 0, own_hi = 0;  // samples this shard finalises (disjoint across shards)
    int64_t send_lo = 0;             // [send_lo, hi) is added into the next shard
    int64_t out_lo = 0, out_hi = 0;  // own range in output (track) coordinates
    int64_t in_lo = 0, in_hi = 0;    // input (track) samples the range reads: [in_lo, in_hi)
};
Shard make_shard(const ChunkPlan& p, int rank, int world);

class Separator {
public:
    explicit Separator(MelBandRoformer& m) : m_(m) {}
    ~Separator();
    // d_track [C][N] -> d_out [S][C][N] (device, fp32).
    void separate(const float* d_track, int64_t N, float overlap, int chunk_batch, float* d_out, cudaStream_t st);
    // Runs the chunks of `sh` and accumulates into d_acc [S*C][hi-lo] and
    // d_wsum [hi-lo] (zeroed here first).  d_track holds track samples
    // [track_lo, track_lo + track_ld) of each channel, rows track_ld apart
    // (the whole track: 0, N; or at least the shard's [in_lo, in_hi)).
    void run_shard(const ChunkPlan& p, const Shard& sh, const float* d_track, int64_t track_lo, int64_t track_ld,
                   int chunk_batch, float* d_acc, float* d_wsum, cudaStream_t st);
    // Host track in, host stems out, with the copies overlapped with the
    // chunks: each chunk batch's new input samples go up on `copy_st` ahead of
    // it, and every output range that no later chunk touches is normalised
    // and copied down while the next batches run.  h_track [C][N], h_out
    // [S][C][N] (pinned host memory lets the copies run asynchronously).
    void separate_host(const float* h_track, int64_t N, float overlap, int chunk_batch, float* h_out,
                       cudaStream_t st, cudaStream_t copy_st);
    // Adds the previous shard's boundary (its [send_lo, hi) = this shard's
    // [lo, lo + recv_len)): d_recv_acc [S*C][recv_len], d_recv_wsum [recv_len].
    void add_boundary(const Shard& sh, float* d_acc, float* d_wsum, const float* d_recv_acc,
                      const float* d_recv_wsum, int64_t recv_len, cudaStream_t st);
    // Writes the normalised, cropped own range into d_out [S*C][out_stride]
    // at track columns [out_lo, out_hi).
    void finalize_shard(const ChunkPlan& p, const Shard& sh, const float* d_acc, const float* d_wsum, float* d_out,
                        int64_t out_stride, cudaStream_t st);
    int64_t last_launches() const { return launches_; }

private:
    float* buf(int i, size_t bytes);
    MelBandRoformer& m_;
    void* bufs_[8] = {};
    size_t caps_[8] = {};
    cudaEvent_t ev_[3] = {};  // separate_host: input batch uploaded, output range ready, last download done
    int64_t launches_ = 0;
};

}  // namespace mbr
