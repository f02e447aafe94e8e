// capi.cpp — extern "C" boundary (include/mbr_b200.h).  No C++ exception crosses it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/mbr_b200.h"
#include "common.h"
#include "model.h"
#include "audio_device.h"
#include "audio_io.h"
#include "ops_api.h"
#include "separator.h"
#include "weights.h"

struct mbr_handle {
    std::string path;
    int device = 0;
    int dtype = 1;
    std::unique_ptr<mbr::MelBandRoformer> model;
    std::unique_ptr<mbr::Separator> sep;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;  // host <-> device copies of mbr_separate
    // host-path buffers
    float* d_track = nullptr;
    float* d_out = nullptr;
    size_t track_cap = 0, out_cap = 0;
    // per-extra-GPU handles for multi-GPU mbr_separate
    std::vector<std::unique_ptr<mbr_handle>> peers;
    int64_t launches = 0;
    ~mbr_handle() {
        peers.clear();
        if (model) cudaSetDevice(device);
        if (d_track) cudaFree(d_track);
        if (d_out) cudaFree(d_out);
        if (stream) cudaStreamDestroy(stream);
        if (copy_stream) cudaStreamDestroy(copy_stream);
        sep.reset();
        model.reset();
    }
};

namespace {

thread_local std::string g_err;

template <class F>
int guard(F&& f) {
    try {
        g_err.clear();
        f();
        return MBR_OK;
    } catch (const mbr::Error& e) {
        g_err = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_err = "host out of memory";
        return MBR_ERR_OOM;
    } catch (const std::exception& e) {
        g_err = e.what();
        return MBR_ERR_INVALID;
    }
}

void need(bool c, const char* m) {
    if (!c) throw mbr::Error(MBR_ERR_INVALID, m);
}

std::unique_ptr<mbr_handle> make_handle(const char* path, int device, int dtype) {
    auto h = std::make_unique<mbr_handle>();
    h->path = path;
    h->device = device;
    h->dtype = dtype;
    int ndev = 0;
    MBR_CUDA(cudaGetDeviceCount(&ndev));
    need(device >= 0 && device < ndev, "device index out of range");
    MBR_CUDA(cudaSetDevice(device));
    mbr::ModelWeights w = mbr::ModelWeights::load(path);
    h->model = std::make_unique<mbr::MelBandRoformer>(w, device, dtype);
    h->sep = std::make_unique<mbr::Separator>(*h->model);
    MBR_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    MBR_CUDA(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
    return h;
}

float* ensure(float*& p, size_t& cap, size_t bytes) {
    if (cap < bytes) {
        if (p) MBR_CUDA(cudaFree(p));
        p = nullptr;
        MBR_CUDA(cudaMalloc(&p, bytes));
        cap = bytes;
    }
    return p;
}

}  // namespace

extern "C" {

MBR_API const char* mbr_last_error(void) { return g_err.c_str(); }
MBR_API int mbr_version(void) { return 100; }

MBR_API int mbr_create(const char* csm_path, int device, int dtype, mbr_handle** out) {
    return guard([&] {
        need(csm_path && out, "null argument");
        *out = nullptr;
        *out = make_handle(csm_path, device, dtype).release();
    });
}

MBR_API void mbr_destroy(mbr_handle* h) { delete h; }

MBR_API int mbr_get_info(mbr_handle* h, int what, int64_t* value) {
    return guard([&] {
        need(h && value, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        switch (what) {
            case MBR_INFO_DIM: *value = c.dim; break;
            case MBR_INFO_DEPTH: *value = c.depth; break;
            case MBR_INFO_NUM_STEMS: *value = c.num_stems; break;
            case MBR_INFO_CHANNELS: *value = h->model->channels(); break;
            case MBR_INFO_NUM_BANDS: *value = c.num_bands; break;
            case MBR_INFO_SAMPLE_RATE: *value = c.sample_rate; break;
            case MBR_INFO_CHUNK_SIZE: *value = c.chunk_size; break;
            case MBR_INFO_NUM_OVERLAP: *value = c.num_overlap; break;
            case MBR_INFO_HEADS: *value = c.heads; break;
            case MBR_INFO_DIM_HEAD: *value = c.dim_head; break;
            case MBR_INFO_BAND_FREQS: *value = h->model->band_freqs(); break;
            case MBR_INFO_DTYPE: *value = h->dtype; break;
            case MBR_INFO_DEVICE: *value = h->device; break;
            case MBR_INFO_HOP: *value = c.stft_hop_length; break;
            default: throw mbr::Error(MBR_ERR_INVALID, "unknown info key");
        }
    });
}

MBR_API int mbr_output_length(mbr_handle* h, int64_t L, int64_t* lout) {
    return guard([&] {
        need(h && lout, "null argument");
        *lout = h->model->out_length(L);
    });
}

MBR_API int mbr_forward_chunk(mbr_handle* h, const float* d_audio, int B, int64_t L, float* d_out, void* stream) {
    return guard([&] {
        need(h && d_audio && d_out, "null argument");
        h->model->forward(d_audio, B, L, d_out, (cudaStream_t)stream);
        h->launches = h->model->last_launches();
    });
}

MBR_API int mbr_forward_tap(mbr_handle* h, const float* d_audio, int B, int64_t L, int tap, float* d_tap, int64_t* n,
                            void* stream) {
    return guard([&] {
        need(h && n, "null argument");
        *n = h->model->forward_tap(d_audio, B, L, tap, d_tap, (cudaStream_t)stream);
    });
}

MBR_API int mbr_separate_device(mbr_handle* h, const float* d_track, int64_t N, float overlap, int chunk_batch,
                                float* d_out, void* stream) {
    return guard([&] {
        need(h && d_track && d_out, "null argument");
        need(N > 0, "empty track");
        MBR_CUDA(cudaSetDevice(h->device));
        h->sep->separate(d_track, N, overlap, chunk_batch, d_out, (cudaStream_t)stream);
        h->launches = h->sep->last_launches();
    });
}

MBR_API int mbr_separate(mbr_handle* h, const float* h_track, int64_t N, float overlap, int chunk_batch, int n_gpus,
                         float* h_out) {
    return guard([&] {
        need(h && h_track && h_out, "null argument");
        need(N > 0, "empty track");
        need(n_gpus >= 1, "n_gpus must be >= 1");
        const int C = h->model->channels(), S = h->model->config().num_stems, SC = S * C;
        const mbr::MBRConfig& cfg = h->model->config();
        mbr::ChunkPlan plan = mbr::make_chunk_plan(N, cfg.chunk_size, overlap, cfg.num_overlap);
        int world = (plan.single || (int)plan.starts.size() < n_gpus) ? 1 : n_gpus;
        if (world == 1) {
            // copies overlapped with the chunks (Separator::separate_host)
            MBR_CUDA(cudaSetDevice(h->device));
            h->sep->separate_host(h_track, N, overlap, chunk_batch, h_out, h->stream, h->copy_stream);
            MBR_CUDA(cudaStreamSynchronize(h->stream));
            h->launches = h->sep->last_launches();
            h->model->check_device_error();
            return;
        }
        // one handle per GPU (device, device+1, ...)
        while ((int)h->peers.size() < world - 1)
            h->peers.push_back(make_handle(h->path.c_str(), h->device + 1 + (int)h->peers.size(), h->dtype));
        std::vector<mbr_handle*> hs{h};
        for (auto& p : h->peers) hs.push_back(p.get());
        std::vector<mbr::Shard> sh(world);
        std::vector<int64_t> rlen(world, 0);
        for (int r = 0; r < world; ++r) {
            sh[r] = mbr::make_shard(plan, r, world);
            if (r > 0) rlen[r] = sh[r - 1].hi - sh[r - 1].send_lo;
        }
        // per-rank device layout: accumulators [SC][span], weight sum [span],
        // received boundary [SC + 1][rlen], own output range [SC][out width];
        // the track buffer holds only the rank's input window
        std::vector<float*> acc(world), ws(world), racc(world), dout(world);
        std::vector<std::string> errs(world);
        auto run = [&](int r) {
            try {
                mbr_handle* x = hs[r];
                MBR_CUDA(cudaSetDevice(x->device));
                const int64_t span = sh[r].hi - sh[r].lo, win = sh[r].in_hi - sh[r].in_lo;
                const int64_t wout = sh[r].out_hi - sh[r].out_lo;
                float* dt = ensure(x->d_track, x->track_cap, sizeof(float) * C * win);
                float* buf = ensure(x->d_out, x->out_cap,
                                    sizeof(float) * ((size_t)(SC + 1) * span + (size_t)(SC + 1) * rlen[r] +
                                                     (size_t)SC * wout));
                acc[r] = buf;
                ws[r] = buf + (size_t)SC * span;
                racc[r] = ws[r] + span;
                dout[r] = racc[r] + (size_t)(SC + 1) * rlen[r];
                MBR_CUDA(cudaMemcpy2DAsync(dt, sizeof(float) * win, h_track + sh[r].in_lo, sizeof(float) * N,
                                           sizeof(float) * win, C, cudaMemcpyHostToDevice, x->stream));
                x->sep->run_shard(plan, sh[r], dt, sh[r].in_lo, win, chunk_batch, acc[r], ws[r], x->stream);
                MBR_CUDA(cudaStreamSynchronize(x->stream));
            } catch (const std::exception& e) {
                errs[r] = e.what();
            }
        };
        std::vector<std::thread> th;
        for (int r = 0; r < world; ++r) th.emplace_back(run, r);
        for (auto& t : th) t.join();
        for (auto& e : errs)
            if (!e.empty()) throw mbr::Error(MBR_ERR_CUDA, e);
        // Boundary exchange: rank r-1's tail [send_lo, hi) is added into rank
        // r's head.  When no rank's tail overlaps the head it receives (every
        // rank holds enough chunks), the tails are final after run_shard and all
        // exchanges go at once; otherwise they run as a chain in rank order.
        bool independent = true;
        for (int r = 1; r + 1 < world; ++r) independent = independent && sh[r - 1].hi <= sh[r].send_lo;
        for (int r = 1; r < world; ++r) {
            mbr_handle* x = hs[r];
            const int64_t off = sh[r - 1].send_lo - sh[r - 1].lo, span_prev = sh[r - 1].hi - sh[r - 1].lo;
            float* rws = racc[r] + (size_t)SC * rlen[r];
            MBR_CUDA(cudaSetDevice(x->device));
            for (int o = 0; o < SC; ++o)
                MBR_CUDA(cudaMemcpyPeerAsync(racc[r] + (size_t)o * rlen[r], x->device,
                                             acc[r - 1] + (size_t)o * span_prev + off, hs[r - 1]->device,
                                             sizeof(float) * rlen[r], x->stream));
            MBR_CUDA(cudaMemcpyPeerAsync(rws, x->device, ws[r - 1] + off, hs[r - 1]->device, sizeof(float) * rlen[r],
                                         x->stream));
            x->sep->add_boundary(sh[r], acc[r], ws[r], racc[r], rws, rlen[r], x->stream);
            if (!independent) MBR_CUDA(cudaStreamSynchronize(x->stream));
        }
        // normalise each own range into the rank's output buffer and copy it out
        for (int r = 0; r < world; ++r) {
            mbr_handle* x = hs[r];
            MBR_CUDA(cudaSetDevice(x->device));
            const int64_t wout = sh[r].out_hi - sh[r].out_lo;
            if (wout <= 0) continue;
            // finalize_shard writes track column t at dout[o * wout + t - out_lo]
            x->sep->finalize_shard(plan, sh[r], acc[r], ws[r], dout[r] - sh[r].out_lo, wout, x->stream);
            MBR_CUDA(cudaMemcpy2DAsync(h_out + sh[r].out_lo, sizeof(float) * N, dout[r], sizeof(float) * wout,
                                       sizeof(float) * wout, SC, cudaMemcpyDeviceToHost, x->stream));
        }
        for (int r = 0; r < world; ++r) {
            MBR_CUDA(cudaSetDevice(hs[r]->device));
            MBR_CUDA(cudaStreamSynchronize(hs[r]->stream));
        }
        MBR_CUDA(cudaSetDevice(h->device));
    });
}

MBR_API int mbr_shard_info(mbr_handle* h, int64_t N, float overlap, int rank, int world, int64_t* info) {
    return guard([&] {
        need(h && info, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        mbr::Shard s = mbr::make_shard(p, rank, world);
        int64_t v[8] = {s.c0, s.c1, s.lo, s.hi, s.send_lo, s.out_lo, s.out_hi, (int64_t)p.starts.size()};
        for (int i = 0; i < 8; ++i) info[i] = v[i];
    });
}

MBR_API int mbr_plan_shard(int64_t N, int chunk_size, float overlap, int default_overlap, int rank, int world,
                           int64_t* info) {
    return guard([&] {
        need(info && N > 0 && chunk_size > 0, "bad argument");
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, chunk_size, overlap, default_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        mbr::Shard s = mbr::make_shard(p, rank, world);
        int64_t v[11] = {s.c0,     s.c1,     s.lo,     s.hi,     s.send_lo,
                         s.out_lo, s.out_hi, (int64_t)p.starts.size(), p.step, p.border, p.total};
        for (int i = 0; i < 11; ++i) info[i] = v[i];
    });
}

MBR_API int mbr_shard_run(mbr_handle* h, const float* d_track, int64_t N, float overlap, int chunk_batch, int rank,
                          int world, float* d_acc, float* d_wsum, void* stream) {
    return guard([&] {
        need(h && d_track && d_acc && d_wsum, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        MBR_CUDA(cudaSetDevice(h->device));
        h->sep->run_shard(p, mbr::make_shard(p, rank, world), d_track, 0, N, chunk_batch, d_acc, d_wsum,
                          (cudaStream_t)stream);
        h->launches = h->sep->last_launches();
    });
}

MBR_API int mbr_shard_window(mbr_handle* h, int64_t N, float overlap, int rank, int world, int64_t* in_lo,
                             int64_t* in_hi) {
    return guard([&] {
        need(h && in_lo && in_hi, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        mbr::Shard s = mbr::make_shard(p, rank, world);
        *in_lo = s.in_lo;
        *in_hi = s.in_hi;
    });
}

MBR_API int mbr_plan_shard_window(int64_t N, int chunk_size, float overlap, int default_overlap, int rank, int world,
                                  int64_t* in_lo, int64_t* in_hi) {
    return guard([&] {
        need(in_lo && in_hi && N > 0 && chunk_size > 0, "bad argument");
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, chunk_size, overlap, default_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        mbr::Shard s = mbr::make_shard(p, rank, world);
        *in_lo = s.in_lo;
        *in_hi = s.in_hi;
    });
}

MBR_API int mbr_shard_run_window(mbr_handle* h, const float* d_window, int64_t win_lo, int64_t win_len, int64_t N,
                                 float overlap, int chunk_batch, int rank, int world, float* d_acc, float* d_wsum,
                                 void* stream) {
    return guard([&] {
        need(h && d_window && d_acc && d_wsum, "null argument");
        need(win_lo >= 0 && win_len > 0 && win_lo + win_len <= N, "bad track window");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        need(!p.single, "track fits one chunk: nothing to shard");
        MBR_CUDA(cudaSetDevice(h->device));
        h->sep->run_shard(p, mbr::make_shard(p, rank, world), d_window, win_lo, win_len, chunk_batch, d_acc, d_wsum,
                          (cudaStream_t)stream);
        h->launches = h->sep->last_launches();
    });
}

MBR_API int mbr_shard_add_boundary(mbr_handle* h, int64_t N, float overlap, int rank, int world, float* d_acc,
                                   float* d_wsum, const float* d_recv_acc, const float* d_recv_wsum,
                                   int64_t recv_len, void* stream) {
    return guard([&] {
        need(h && d_acc && d_wsum, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        mbr::Shard s = mbr::make_shard(p, rank, world);
        MBR_CUDA(cudaSetDevice(h->device));
        h->sep->add_boundary(s, d_acc, d_wsum, d_recv_acc, d_recv_wsum, recv_len, (cudaStream_t)stream);
    });
}

MBR_API int mbr_shard_finalize(mbr_handle* h, int64_t N, float overlap, int rank, int world, float* d_acc,
                               float* d_wsum, float* d_out, int64_t out_stride, void* stream) {
    return guard([&] {
        need(h && d_acc && d_wsum && d_out, "null argument");
        const mbr::MBRConfig& c = h->model->config();
        mbr::ChunkPlan p = mbr::make_chunk_plan(N, c.chunk_size, overlap, c.num_overlap);
        mbr::Shard s = mbr::make_shard(p, rank, world);
        MBR_CUDA(cudaSetDevice(h->device));
        h->sep->finalize_shard(p, s, d_acc, d_wsum, d_out, out_stride, (cudaStream_t)stream);
    });
}

MBR_API int mbr_set_graphs(mbr_handle* h, int enable) {
    return guard([&] {
        need(h, "null argument");
        MBR_CUDA(cudaSetDevice(h->device));
        h->model->set_graphs(enable != 0);
        for (auto& p : h->peers) {
            MBR_CUDA(cudaSetDevice(p->device));
            p->model->set_graphs(enable != 0);
        }
        MBR_CUDA(cudaSetDevice(h->device));
    });
}

MBR_API int mbr_set_backend(mbr_handle* h, int gemm, int attention) {
    return guard([&] {
        need(h, "null argument");
        need(gemm >= 0 && gemm <= 2 && (attention == 0 || attention == 1),
             "gemm backend must be 0, 1 or 2 and attention backend 0 or 1");
        h->model->set_backend(gemm, attention);
    });
}

MBR_API int mbr_last_launches(mbr_handle* h, int64_t* n) {
    return guard([&] {
        need(h && n, "null argument");
        *n = h->launches;
    });
}

MBR_API int mbr_sync_check(mbr_handle* h) {
    return guard([&] {
        need(h, "null argument");
        MBR_CUDA(cudaSetDevice(h->device));
        MBR_CUDA(cudaDeviceSynchronize());
        h->model->check_device_error();
    });
}

MBR_API int mbr_profile_enable(mbr_handle* h, int on) {
    return guard([&] {
        need(h, "null argument");
        h->model->profile_enable(on != 0);
    });
}

MBR_API int mbr_profile_read(mbr_handle* h, int kind, double* ms, int64_t* count) {
    return guard([&] {
        need(h && ms && count, "null argument");
        h->model->profile_read(kind, ms, count);
    });
}

// ---- WAV I/O ----
MBR_API int mbr_wav_info(const char* path, int* sample_rate, int* channels, int64_t* frames) {
    return guard([&] {
        need(path && sample_rate && channels && frames, "null argument");
        cudasep::HostAudio a = cudasep::read_wav_host(path);
        *sample_rate = a.sample_rate;
        *channels = a.channels;
        *frames = a.frames;
    });
}

MBR_API int mbr_wav_read(const char* path, float* h_planar, int64_t capacity) {
    return guard([&] {
        need(path && h_planar, "null argument");
        cudasep::HostAudio a = cudasep::read_wav_host(path);
        need((int64_t)a.planar.size() <= capacity, "mbr_wav_read: buffer too small");
        std::copy(a.planar.begin(), a.planar.end(), h_planar);
    });
}

MBR_API int mbr_wav_write(const char* path, const float* h_planar, int channels, int64_t frames, int sample_rate) {
    return guard([&] {
        need(path && h_planar && channels > 0 && frames >= 0 && sample_rate > 0, "bad argument");
        cudasep::write_wav_host(path, h_planar, channels, frames, sample_rate);
    });
}

MBR_API int mbr_pcm_to_planar(const void* d_pcm, int64_t frames, int channels, int bits, int is_float,
                              float* d_planar, void* stream) {
    return guard([&] {
        need(d_pcm && d_planar && frames >= 0 && channels > 0, "bad argument");
        mbr::audio::pcm_to_planar(d_pcm, frames, channels, bits, is_float != 0, d_planar, (cudaStream_t)stream);
    });
}

MBR_API int mbr_wav_read_device(const char* path, float* d_planar, int64_t capacity, int* sample_rate, int* channels,
                                int64_t* frames, void* stream) {
    return guard([&] {
        need(path && sample_rate && channels && frames, "null argument");
        std::vector<uint8_t> bytes = cudasep::read_file(path);
        const cudasep::WavLayout w = cudasep::parse_wav(bytes.data(), bytes.size(), path);
        *sample_rate = w.sample_rate;
        *channels = w.channels;
        *frames = w.frames;
        if (!d_planar) return;  // size query
        need(w.frames * w.channels <= capacity, "mbr_wav_read_device: buffer too small");
        if (w.frames == 0) return;
        cudaStream_t st = (cudaStream_t)stream;
        // the data chunk's raw bytes go up once; conversion happens on the device
        void* d_pcm = nullptr;
        MBR_CUDA(cudaMallocAsync(&d_pcm, w.data_bytes, st));
        try {
            MBR_CUDA(cudaMemcpyAsync(d_pcm, bytes.data() + w.data_off, w.data_bytes, cudaMemcpyHostToDevice, st));
            mbr::audio::pcm_to_planar(d_pcm, w.frames, w.channels, w.bits, w.format == 3, d_planar, st);
        } catch (...) {
            cudaFreeAsync(d_pcm, st);
            throw;
        }
        MBR_CUDA(cudaFreeAsync(d_pcm, st));
        MBR_CUDA(cudaStreamSynchronize(st));  // `bytes` is released on return
    });
}

MBR_API int mbr_wav_write_device(const char* path, const float* d_planar, int channels, int64_t frames,
                                 int sample_rate, void* stream) {
    return guard([&] {
        need(path && d_planar && channels > 0 && frames >= 0 && sample_rate > 0, "bad argument");
        cudaStream_t st = (cudaStream_t)stream;
        std::vector<float> inter((size_t)frames * channels);
        if (frames > 0) {
            float* d_inter = nullptr;
            MBR_CUDA(cudaMallocAsync((void**)&d_inter, sizeof(float) * inter.size(), st));
            try {
                mbr::audio::planar_to_interleaved(d_planar, frames, channels, d_inter, st);
                MBR_CUDA(cudaMemcpyAsync(inter.data(), d_inter, sizeof(float) * inter.size(), cudaMemcpyDeviceToHost,
                                         st));
            } catch (...) {
                cudaFreeAsync(d_inter, st);
                throw;
            }
            MBR_CUDA(cudaFreeAsync(d_inter, st));
            MBR_CUDA(cudaStreamSynchronize(st));
        }
        cudasep::write_wav_interleaved(path, inter.data(), channels, frames, sample_rate);
    });
}

// ---- stand-alone ops ----
MBR_API int mbr_op_rms_norm(const void* d_x, const float* d_gamma, void* d_y, int64_t rows, int dim, float scale,
                            int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_gamma && d_y && rows >= 0, "bad argument");
        if (rows > 0) mbr::opsapi::rms_norm(d_x, d_gamma, d_y, rows, dim, scale, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_add(const void* d_a, const void* d_b, void* d_y, int64_t n, int dtype, void* stream) {
    return guard([&] {
        need(d_a && d_b && d_y && n >= 0, "bad argument");
        if (n > 0) mbr::opsapi::add(d_a, d_b, d_y, n, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_gelu(const void* d_x, void* d_y, int64_t n, int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_y && n >= 0, "bad argument");
        if (n > 0) mbr::opsapi::gelu(d_x, d_y, n, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_sigmoid_gate(const void* d_x, const void* d_gate, void* d_y, int64_t rows, int heads,
                                int dim_head, int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_gate && d_y && rows >= 0 && heads > 0 && dim_head > 0, "bad argument");
        if (rows > 0) mbr::opsapi::sigmoid_gate(d_x, d_gate, d_y, rows, heads, dim_head, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_rope(const void* d_x, const float* d_cos, const float* d_sin, void* d_y, int64_t seqs, int L,
                        int heads, int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_cos && d_sin && d_y && seqs >= 0 && L > 0 && heads > 0, "bad argument");
        if (seqs > 0) mbr::opsapi::rope(d_x, d_cos, d_sin, d_y, seqs, L, heads, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_linear(const void* d_x, const void* d_w, const float* d_bias, void* d_y, int64_t rows, int in,
                          int out, int act, int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_w && d_y && rows >= 0 && in > 0 && out > 0 && act >= 0 && act <= 2, "bad argument");
        mbr::opsapi::linear(d_x, d_w, d_bias, d_y, rows, in, out, act, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_ffn(const void* d_x, const void* d_w1, const float* d_b1, const void* d_w2, const float* d_b2,
                       float* d_resid, int64_t rows, int dim, int hidden, int dtype, void* stream) {
    return guard([&] {
        need(d_x && d_w1 && d_b1 && d_w2 && d_b2 && d_resid && rows >= 0 && dim > 0 && hidden > 0, "bad argument");
        mbr::opsapi::ffn(d_x, d_w1, d_b1, d_w2, d_b2, d_resid, rows, dim, hidden, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_attention(const void* d_q, const void* d_k, const void* d_v, int64_t B, int heads, int N,
                             int dim_head, float scale, const float* d_gates, void* d_out, int dtype, void* stream) {
    return guard([&] {
        need(d_q && d_k && d_v && d_out && B >= 0 && heads > 0 && N > 0 && (dim_head == 32 || dim_head == 64),
             "bad argument");
        if (B > 0)
            mbr::opsapi::attention(d_q, d_k, d_v, B, heads, N, dim_head, scale, d_gates, d_out, dtype,
                                   (cudaStream_t)stream);
    });
}

MBR_API int mbr_rope_tables(int L, int dim_head, float* h_cos, float* h_sin) {
    return guard([&] {
        need(h_cos && h_sin && L > 0 && dim_head > 0 && dim_head % 2 == 0, "bad argument");
        std::vector<float> cs, sn;
        mbr::rotary_tables(L, dim_head, cs, sn);
        std::copy(cs.begin(), cs.end(), h_cos);
        std::copy(sn.begin(), sn.end(), h_sin);
    });
}

MBR_API int mbr_op_band_gather(mbr_handle* h, const float* d_spec, int B, int T, void* d_x, int dtype,
                               void* stream) {
    return guard([&] {
        need(h && d_spec && d_x && B > 0 && T > 0, "bad argument");
        MBR_CUDA(cudaSetDevice(h->device));
        mbr::opsapi::band_gather((const float2*)d_spec, B, h->model->channels(), 1025, T, h->model->d_freq_indices(),
                                 h->model->band_freqs(), h->model->band_tiles(), d_x, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_mask_scatter(mbr_handle* h, const float* d_spec, const void* d_masks, int B, int S, int T,
                                float* d_out, int dtype, void* stream) {
    return guard([&] {
        need(h && d_spec && d_masks && d_out && B > 0 && S > 0 && T > 0, "bad argument");
        MBR_CUDA(cudaSetDevice(h->device));
        mbr::opsapi::mask_scatter((const float2*)d_spec, d_masks, B, S, h->model->channels(), 1025, T,
                                  h->model->d_bands_per_freq(), h->model->band_freqs(), h->model->band_tiles(),
                                  (float2*)d_out, dtype, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_stft(const float* d_sig, int64_t n, int64_t L, int hop, float* d_spec, void* stream) {
    return guard([&] {
        need(d_sig && d_spec && n > 0, "bad argument");
        mbr::opsapi::stft(d_sig, n, L, hop, (float2*)d_spec, (cudaStream_t)stream);
    });
}

MBR_API int mbr_op_istft(const float* d_spec, int64_t n, int T, int hop, int64_t length, float* d_out,
                         void* stream) {
    return guard([&] {
        need(d_spec && d_out && n > 0 && T > 0 && hop > 0, "bad argument");
        cudaStream_t st = (cudaStream_t)stream;
        int64_t lout = length > 0 ? length : (int64_t)(T - 1) * hop;
        need(lout > 0, "empty output");
        // n * T * 2048 floats must fit in size_t
        need(n <= (int64_t)(SIZE_MAX / sizeof(float) / 2048) / T, "n * T too large");
        float* frames = nullptr;
        MBR_CUDA(cudaMallocAsync((void**)&frames, sizeof(float) * (size_t)n * T * 2048, st));
        try {
            mbr::opsapi::istft((const float2*)d_spec, n, T, hop, frames, lout, d_out, st);
        } catch (...) {
            cudaFreeAsync(frames, st);
            throw;
        }
        MBR_CUDA(cudaFreeAsync(frames, st));
    });
}

// Same result as mbr_op_istft, for callers that must not allocate device
// memory: the frame scratch is a fixed array compiled into the library (see
// the header for the limits and the sharing rules).
MBR_API int mbr_op_istft_noalloc(const float* d_spec, int64_t n, int T, int hop, int64_t length, float* d_out,
                                 void* stream) {
    return guard([&] {
        need(d_spec && d_out && n > 0 && T > 0 && hop > 0, "bad argument");
        int64_t lout = length > 0 ? length : (int64_t)(T - 1) * hop;
        need(lout > 0, "empty output");
        // compared by division so that no product can overflow
        const int64_t max_frames = mbr::opsapi::kIstftStaticFloats / 2048;
        if (n > max_frames / T)
            throw mbr::Error(MBR_ERR_INVALID,
                             "mbr_op_istft_noalloc: n = " + std::to_string(n) + ", T = " + std::to_string(T) +
                                 " exceeds the static scratch of " + std::to_string(max_frames) + " frames");
        float* frames = mbr::opsapi::istft_static_scratch();
        mbr::opsapi::istft((const float2*)d_spec, n, T, hop, frames, lout, d_out, (cudaStream_t)stream);
    });
}

}  // extern "C"
