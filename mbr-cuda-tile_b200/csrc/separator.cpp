// separator.cpp — chunked separation driver (reference: src/inference_app.cpp:46-357).
#include "separator.h"

#include <algorithm>
#include <cmath>

#include "common.h"

namespace mbr {

// resolve_step (src/inference_app.cpp:46-57)
int resolve_step(int chunk, float overlap, int def) {
    if (overlap > 0.0f && overlap < 1.0f) {
        int step = (int)std::lround(chunk * (1.0f - overlap));
        return std::max(1, step);
    }
    int no = def;
    if (overlap >= 1.0f) no = std::max(1, (int)std::lround(overlap));
    return std::max(1, chunk / std::max(1, no));
}

// Chunk boundaries of process_chunked (src/inference_app.cpp:72-89) and the
// single-chunk branch of run_inference (:330).
ChunkPlan make_chunk_plan(int64_t N, int chunk, float overlap, int def) {
    ChunkPlan p;
    p.N = N;
    p.chunk = chunk;
    if (!(chunk > 0 && N > chunk)) {
        p.single = true;
        p.total = N;
        return p;
    }
    p.step = resolve_step(chunk, overlap, def);
    p.fade = chunk / 10;
    int64_t border = chunk - p.step;
    p.padded = N > 2 * border && border > 0;
    p.border = p.padded ? border : 0;
    p.total = p.padded ? N + 2 * border : N;
    for (int64_t s = 0; s < p.total; s += p.step) p.starts.push_back(s);
    return p;
}

// Track samples [*in_lo, *in_hi) that padded positions [lo, hi) read.  The
// reflect padding is a single fold on each side (border < N) and the map is
// monotone between the fold points 0 and N - 1, so its extremes over the
// range lie at the range's ends or at those fold points.
static void input_window(const ChunkPlan& p, int64_t lo, int64_t hi, int64_t* in_lo, int64_t* in_hi) {
    if (!p.padded) {
        *in_lo = std::min<int64_t>(lo, p.N);
        *in_hi = std::min<int64_t>(hi, p.N);
        return;
    }
    const int64_t a = lo - p.border, b = hi - 1 - p.border;
    auto fold = [&](int64_t x) { return x < 0 ? -x : (x >= p.N ? 2 * (p.N - 1) - x : x); };
    int64_t mn = std::min(fold(a), fold(b)), mx = std::max(fold(a), fold(b));
    for (int64_t brk : {(int64_t)0, p.N - 1})
        if (a <= brk && brk <= b) {
            mn = std::min(mn, fold(brk));
            mx = std::max(mx, fold(brk));
        }
    *in_lo = mn;
    *in_hi = mx + 1;
}

Shard make_shard(const ChunkPlan& p, int rank, int world) {
    Shard s;
    int n = (int)p.starts.size();
    MBR_CHECK(world >= 1 && rank >= 0 && rank < world, "bad rank/world");
    MBR_CHECK(n >= world, "track has fewer chunks than ranks");
    s.c0 = (int)((int64_t)rank * n / world);
    s.c1 = (int)((int64_t)(rank + 1) * n / world);
    s.lo = p.starts[s.c0];
    s.hi = std::min<int64_t>(p.starts[s.c1 - 1] + p.chunk, p.total);
    s.own_lo = s.lo;
    s.own_hi = s.c1 < n ? p.starts[s.c1] : p.total;
    s.send_lo = s.c1 < n ? p.starts[s.c1] : s.hi;
    s.out_lo = std::max<int64_t>(s.own_lo, p.border) - p.border;
    s.out_hi = std::min<int64_t>(s.own_hi, p.border + p.N) - p.border;
    if (s.out_hi < s.out_lo) s.out_hi = s.out_lo;
    input_window(p, s.lo, s.hi, &s.in_lo, &s.in_hi);
    return s;
}

Separator::~Separator() {
    for (void* b : bufs_)
        if (b) cudaFree(b);
    for (cudaEvent_t e : ev_)
        if (e) cudaEventDestroy(e);
}

float* Separator::buf(int i, size_t bytes) {
    if (caps_[i] < bytes) {
        if (bufs_[i]) MBR_CUDA(cudaFree(bufs_[i]));
        bufs_[i] = nullptr;
        MBR_CUDA(cudaMalloc(&bufs_[i], bytes));
        caps_[i] = bytes;
    }
    return (float*)bufs_[i];
}

void Separator::run_shard(const ChunkPlan& p, const Shard& sh, const float* d_track, int64_t track_lo,
                          int64_t track_ld, int chunk_batch, float* d_acc, float* d_wsum, cudaStream_t st) {
    MBR_CHECK(track_lo <= sh.in_lo && sh.in_hi <= track_lo + track_ld, "track window does not cover the shard");
    const int C = m_.channels(), S = m_.config().num_stems, SC = S * C;
    const int64_t lout = m_.out_length(p.chunk);
    const int64_t span = sh.hi - sh.lo;
    MBR_CHECK(chunk_batch >= 1, "chunk_batch must be >= 1");
    MBR_CUDA(cudaMemsetAsync(d_acc, 0, sizeof(float) * SC * span, st));
    MBR_CUDA(cudaMemsetAsync(d_wsum, 0, sizeof(float) * span, st));
    launches_ += 2;
    // every chunk's actual length must fit the model output (the reference
    // reshapes the output to the actual length, src/inference_app.cpp:194-197)
    for (int c = sh.c0; c < sh.c1; ++c) {
        int64_t al = std::min<int64_t>(p.chunk, p.total - p.starts[c]);
        MBR_CHECK(lout >= al, "model output shorter than the chunk (chunk_size not a multiple of the hop)");
    }
    int cb = std::min(chunk_batch, sh.c1 - sh.c0);
    float* d_in = buf(0, sizeof(float) * (size_t)cb * C * p.chunk);
    float* d_y = buf(1, sizeof(float) * (size_t)cb * SC * lout);
    int64_t* d_starts = (int64_t*)buf(2, sizeof(int64_t) * (sh.c1 - sh.c0));
    MBR_CUDA(cudaMemcpyAsync(d_starts, p.starts.data() + sh.c0, sizeof(int64_t) * (sh.c1 - sh.c0),
                             cudaMemcpyHostToDevice, st));
    for (int g0 = sh.c0; g0 < sh.c1; g0 += cb) {
        int n = std::min(cb, sh.c1 - g0);
        const int64_t* gs = d_starts + (g0 - sh.c0);
        ops::prepare_chunks(d_track, C, p.N, track_lo, track_ld, p.border, p.padded, gs, n, p.total, p.chunk, d_in,
                            st);
        m_.forward(d_in, n, p.chunk, d_y, st);
        ops::accumulate_chunks(d_y, n, SC, lout, gs, p.total, p.chunk, p.fade, d_acc, d_wsum, sh.lo, span, st);
        launches_ += 2 + m_.last_launches();
    }
}

void Separator::add_boundary(const Shard& sh, float* d_acc, float* d_wsum, const float* d_recv_acc,
                             const float* d_recv_wsum, int64_t recv_len, cudaStream_t st) {
    const int SC = m_.config().num_stems * m_.channels();
    MBR_CHECK(recv_len >= 0 && recv_len <= sh.hi - sh.lo, "boundary longer than the shard window");
    if (recv_len > 0) {
        ops::add_window(d_acc, d_wsum, sh.hi - sh.lo, d_recv_acc, d_recv_wsum, recv_len, SC, st);
        ++launches_;
    }
}

void Separator::finalize_shard(const ChunkPlan& p, const Shard& sh, const float* d_acc, const float* d_wsum,
                               float* d_out, int64_t out_stride, cudaStream_t st) {
    const int SC = m_.config().num_stems * m_.channels();
    const int64_t span = sh.hi - sh.lo;
    int64_t p0 = std::max<int64_t>(sh.own_lo, p.border), p1 = std::min<int64_t>(sh.own_hi, p.border + p.N);
    ops::normalize_crop(d_acc, d_wsum, SC, sh.lo, span, p0, p1, p.border, out_stride, d_out, st);
    ++launches_;
}

void Separator::separate(const float* d_track, int64_t N, float overlap, int chunk_batch, float* d_out,
                         cudaStream_t st) {
    const MBRConfig& c = m_.config();
    const int C = m_.channels(), SC = c.num_stems * C;
    launches_ = 0;
    ChunkPlan p = make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
    if (p.single) {
        // run_inference single-chunk branch: forward over the whole input
        int64_t lout = m_.out_length(N);
        float* d_y = buf(1, sizeof(float) * (size_t)SC * lout);
        m_.forward(d_track, 1, N, d_y, st);
        launches_ += m_.last_launches();
        int64_t w = std::min(lout, N);
        if (w < N) MBR_CUDA(cudaMemsetAsync(d_out, 0, sizeof(float) * SC * N, st));
        MBR_CUDA(cudaMemcpy2DAsync(d_out, sizeof(float) * N, d_y, sizeof(float) * lout, sizeof(float) * w, SC,
                                   cudaMemcpyDeviceToDevice, st));
        return;
    }
    Shard sh = make_shard(p, 0, 1);
    int64_t span = sh.hi - sh.lo;
    float* d_acc = buf(3, sizeof(float) * (size_t)SC * span);
    float* d_wsum = buf(4, sizeof(float) * (size_t)span);
    run_shard(p, sh, d_track, 0, N, chunk_batch, d_acc, d_wsum, st);
    finalize_shard(p, sh, d_acc, d_wsum, d_out, N, st);
}

void Separator::separate_host(const float* h_track, int64_t N, float overlap, int chunk_batch, float* h_out,
                              cudaStream_t st, cudaStream_t cst) {
    const MBRConfig& c = m_.config();
    const int C = m_.channels(), S = c.num_stems, SC = S * C;
    launches_ = 0;
    ChunkPlan p = make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
    float* d_track = buf(5, sizeof(float) * (size_t)C * N);
    float* d_out = buf(6, sizeof(float) * (size_t)SC * N);
    if (p.single) {
        MBR_CUDA(cudaMemcpyAsync(d_track, h_track, sizeof(float) * C * N, cudaMemcpyHostToDevice, st));
        separate(d_track, N, overlap, chunk_batch, d_out, st);
        MBR_CUDA(cudaMemcpyAsync(h_out, d_out, sizeof(float) * SC * N, cudaMemcpyDeviceToHost, st));
        return;
    }
    for (auto& e : ev_)
        if (!e) MBR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    MBR_CHECK(chunk_batch >= 1, "chunk_batch must be >= 1");
    const int64_t lout = m_.out_length(p.chunk);
    const int n = (int)p.starts.size();
    const int cb = std::min(chunk_batch, n);
    const Shard sh = make_shard(p, 0, 1);
    const int64_t span = sh.hi - sh.lo;
    float* d_acc = buf(3, sizeof(float) * (size_t)SC * span);
    float* d_wsum = buf(4, sizeof(float) * (size_t)span);
    float* d_in = buf(0, sizeof(float) * (size_t)cb * C * p.chunk);
    float* d_y = buf(1, sizeof(float) * (size_t)cb * SC * lout);
    int64_t* d_starts = (int64_t*)buf(2, sizeof(int64_t) * n);
    for (int i = 0; i < n; ++i) {
        int64_t al = std::min<int64_t>(p.chunk, p.total - p.starts[i]);
        MBR_CHECK(lout >= al, "model output shorter than the chunk (chunk_size not a multiple of the hop)");
    }
    MBR_CUDA(cudaMemcpyAsync(d_starts, p.starts.data(), sizeof(int64_t) * n, cudaMemcpyHostToDevice, st));
    MBR_CUDA(cudaMemsetAsync(d_acc, 0, sizeof(float) * SC * span, st));
    MBR_CUDA(cudaMemsetAsync(d_wsum, 0, sizeof(float) * span, st));
    launches_ += 2;
    int64_t up = 0;       // track samples [0, up) uploaded
    int64_t done = 0;     // padded positions [0, done) normalised and downloaded
    for (int g0 = 0; g0 < n; g0 += cb) {
        const int nb = std::min(cb, n - g0);
        // upload the prefix of the track this batch reads (batches move left
        // to right, so every later batch reads at least as far)
        int64_t in_lo, in_hi;
        input_window(p, p.starts[g0], std::min<int64_t>(p.starts[g0 + nb - 1] + p.chunk, p.total), &in_lo, &in_hi);
        const int64_t need = std::max(up, in_hi);
        if (need > up) {
            MBR_CUDA(cudaMemcpy2DAsync(d_track + up, sizeof(float) * N, h_track + up, sizeof(float) * N,
                                       sizeof(float) * (need - up), C, cudaMemcpyHostToDevice, cst));
            MBR_CUDA(cudaEventRecord(ev_[0], cst));
            MBR_CUDA(cudaStreamWaitEvent(st, ev_[0], 0));
            up = need;
        }
        const int64_t* gs = d_starts + g0;
        ops::prepare_chunks(d_track, C, p.N, 0, N, p.border, p.padded, gs, nb, p.total, p.chunk, d_in, st);
        m_.forward(d_in, nb, p.chunk, d_y, st);
        ops::accumulate_chunks(d_y, nb, SC, lout, gs, p.total, p.chunk, p.fade, d_acc, d_wsum, sh.lo, span, st);
        launches_ += 2 + m_.last_launches();
        // positions before the next batch's first chunk are final
        const int64_t fin = g0 + nb < n ? p.starts[g0 + nb] : p.total;
        const int64_t p0 = std::max<int64_t>(done, p.border), p1 = std::min<int64_t>(fin, p.border + N);
        if (p1 > p0) {
            ops::normalize_crop(d_acc, d_wsum, SC, sh.lo, span, p0, p1, p.border, N, d_out, st);
            ++launches_;
            MBR_CUDA(cudaEventRecord(ev_[1], st));
            MBR_CUDA(cudaStreamWaitEvent(cst, ev_[1], 0));
            const int64_t o0 = p0 - p.border, w = p1 - p0;
            MBR_CUDA(cudaMemcpy2DAsync(h_out + o0, sizeof(float) * N, d_out + o0, sizeof(float) * N,
                                       sizeof(float) * w, SC, cudaMemcpyDeviceToHost, cst));
        }
        done = std::max(done, fin);
    }
    // the caller's stream completes only after the last download
    MBR_CUDA(cudaEventRecord(ev_[2], cst));
    MBR_CUDA(cudaStreamWaitEvent(st, ev_[2], 0));
}

}  // namespace mbr
