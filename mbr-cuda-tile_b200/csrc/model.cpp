// model.cpp — MelBandRoformer host orchestration (weights upload, workspace,
// launch sequence).  Reference: src/model_mel_band_roformer.cu:46-845.
#include "model.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.h"
#include "gemm_tc.h"
#include "attention_tc.h"

namespace mbr {

MBRConfig MBRConfig::from_json(const JsonValue& j) {
    MBRConfig c;
    c.dim = j.get_int("dim", 384);
    c.depth = j.get_int("depth", 6);
    c.stereo = j.get_bool("stereo", true);
    c.num_stems = j.get_int("num_stems", 1);
    c.time_transformer_depth = j.get_int("time_transformer_depth", 1);
    c.freq_transformer_depth = j.get_int("freq_transformer_depth", 1);
    c.num_bands = j.get_int("num_bands", 60);
    c.dim_head = j.get_int("dim_head", 64);
    c.heads = j.get_int("heads", 8);
    c.mask_estimator_depth = j.get_int("mask_estimator_depth", 2);
    c.mlp_expansion_factor = j.get_int("mlp_expansion_factor", 4);
    c.zero_dc = j.get_bool("zero_dc", true);
    c.sample_rate = j.get_int("sample_rate", 44100);
    c.stft_n_fft = j.get_int("stft_n_fft", 2048);
    c.stft_hop_length = j.get_int("stft_hop_length", 441);
    c.stft_win_length = j.get_int("stft_win_length", 2048);
    c.stft_normalized = j.get_bool("stft_normalized", false);
    c.match_input_audio_length = j.get_bool("match_input_audio_length", false);
    c.dim_freqs_in = j.get_int("dim_freqs_in", 1025);
    c.skip_connection = j.get_bool("skip_connection", false);
    c.chunk_size = j.get_int("chunk_size", c.stft_n_fft * 256);
    c.num_overlap = std::max(1, j.get_int("num_overlap", 1));
    if (j.has("instruments") && j["instruments"].is_array())
        for (size_t i = 0; i < j["instruments"].size(); ++i) c.instruments.push_back(j["instruments"][i].as_string());
    return c;
}

namespace {

// Host staging of every weight in one buffer, uploaded with one copy.
struct Packer {
    std::vector<uint8_t> buf;
    size_t add(const void* p, size_t bytes) {
        size_t off = round_up((int64_t)buf.size(), 256);
        buf.resize(off + round_up((int64_t)bytes, 16), 0);
        if (p) std::memcpy(buf.data() + off, p, bytes);
        return off;
    }
    size_t zeros(size_t bytes) { return add(nullptr, bytes); }
};

float round_to(float x, int dt) {
    if (dt == DT_F16) return half_bits_to_float(float_to_half_bits(x));
    if (dt == DT_BF16) return bf16_bits_to_float(float_to_bf16_bits(x));
    return x;
}

// Writes `n` floats into dst as the compute dtype.
void store_as(uint8_t* dst, int dt, int64_t idx, float v) {
    if (dt == DT_F32) {
        std::memcpy(dst + 4 * idx, &v, 4);
    } else {
        uint16_t h = dt == DT_F16 ? float_to_half_bits(v) : float_to_bf16_bits(v);
        std::memcpy(dst + 2 * idx, &h, 2);
    }
}

std::vector<float> to_floats(const HostTensor& t) {
    std::vector<float> v((size_t)t.numel());
    for (int64_t i = 0; i < t.numel(); ++i) v[i] = t.f(i);
    return v;
}

}  // namespace

// compute_rotary_cos_sin (src/model_mel_band_roformer.cu:270-300), fp32 host math.
void rotary_tables(int n, int dim, std::vector<float>& cs, std::vector<float>& sn) {
    int half = dim / 2;
    cs.resize((size_t)n * half);
    sn.resize((size_t)n * half);
    for (int p = 0; p < n; ++p)
        for (int i = 0; i < half; ++i) {
            float freq = 1.0f / std::pow(10000.0f, (float)(2 * i) / (float)dim);
            float ang = (float)p * freq;
            cs[(size_t)p * half + i] = std::cos(ang);
            sn[(size_t)p * half + i] = std::sin(ang);
        }
}

MelBandRoformer::MelBandRoformer(const ModelWeights& w, int device, int dtype) : device_(device), dtype_(dtype) {
    MBR_CHECK(dtype == DT_F32 || dtype == DT_F16 || dtype == DT_BF16, "dtype must be fp32, fp16 or bf16");
    MBR_CUDA(cudaSetDevice(device));
    cfg_ = MBRConfig::from_json(w.config());
    const MBRConfig& c = cfg_;
    if (c.stft_n_fft != 2048 || c.stft_win_length != 2048)
        throw Error(ERR_UNSUPPORTED, "STFT supports n_fft = win_length = 2048 only");
    MBR_CHECK(c.dim % 32 == 0 && c.dim <= 1024, "dim must be a multiple of 32 and <= 1024");
    MBR_CHECK(c.dim_head == 64 || c.dim_head == 32, "dim_head must be 32 or 64");
    MBR_CHECK(c.heads >= 1 && c.heads <= 32, "heads must be in [1, 32]");
    MBR_CHECK(c.mask_estimator_depth >= 0, "mask_estimator_depth must be >= 0");
    MBR_CHECK(c.depth >= 1, "depth must be >= 1");
    C_ = c.stereo ? 2 : 1;
    F_ = c.stft_n_fft / 2 + 1;
    NB_ = c.num_bands;
    D_ = c.dim;
    H_ = c.heads;
    dh_ = c.dim_head;
    DI_ = H_ * dh_;
    hid_ = D_ * c.mlp_expansion_factor;
    int FC = F_ * C_;

    // ---- band maps (src/model_mel_band_roformer.cu:79-150) ----
    if (!w.has("__precomputed__.freq_indices"))
        throw Error(ERR_IO, "MelBandRoformer .csm must include precomputed mel band data");
    const HostTensor& fi_t = w.get("__precomputed__.freq_indices");
    const HostTensor& nfpb_t = w.get("__precomputed__.num_freqs_per_band");
    const HostTensor& nbpf_t = w.get("__precomputed__.num_bands_per_freq");
    MBR_CHECK(nfpb_t.numel() == NB_, "num_freqs_per_band size != num_bands");
    MBR_CHECK(nbpf_t.numel() == F_, "num_bands_per_freq size != n_fft/2+1");
    J_ = fi_t.numel();
    std::vector<int> fi(J_);
    for (int64_t j = 0; j < J_; ++j) {
        int64_t v = fi_t.i64(j);
        if (v < 0 || v >= FC) throw Error(ERR_IO, "MelBandRoformer: precomputed freq_indices out of range");
        fi[j] = (int)v;
    }
    band_bd_.resize(NB_);
    band_boff_.resize(NB_ + 1);
    band_kofs_.resize(NB_ + 1);
    std::vector<int> jofs(NB_ + 1);
    band_boff_[0] = band_kofs_[0] = jofs[0] = 0;
    for (int b = 0; b < NB_; ++b) {
        band_bd_[b] = (int)(2 * nfpb_t.i64(b) * C_);
        band_boff_[b + 1] = band_boff_[b] + band_bd_[b];
        jofs[b + 1] = band_boff_[b + 1] / 2;
        // each band's K range is padded to a multiple of 64 elements (one
        // 128-byte swizzle atom of 16-bit operands)
        band_kofs_[b + 1] = band_kofs_[b] + (int)round_up(band_bd_[b], 64);
    }
    MBR_CHECK(band_boff_[NB_] == 2 * J_, "band dims do not match freq_indices");
    KP_ = band_kofs_[NB_];
    std::vector<float> nbpf(FC);
    for (int f = 0; f < F_; ++f)
        for (int s = 0; s < C_; ++s) nbpf[f * C_ + s] = (float)nbpf_t.i64(f);
    // reverse map freq -> band-freq list (ascending j)
    std::vector<int> rev_off(FC + 1, 0), rev_idx(J_);
    for (int64_t j = 0; j < J_; ++j) rev_off[fi[j] + 1]++;
    for (int f = 0; f < FC; ++f) rev_off[f + 1] += rev_off[f];
    {
        std::vector<int> cur(rev_off.begin(), rev_off.end() - 1);
        for (int64_t j = 0; j < J_; ++j) rev_idx[cur[fi[j]]++] = (int)j;
    }

    {
        // tiles of the band map for the stand-alone band ops (one allocation)
        opsapi::BandTilesHost bh = opsapi::make_band_tiles(fi, C_, F_);
        Packer tp;
        size_t o_j = tp.add(bh.jl.data(), bh.jl.size() * 4);
        size_t o_jr = tp.add(bh.jr.data(), bh.jr.size() * 4);
        size_t o_k = tp.add(bh.bk.data(), bh.bk.size() * 4);
        size_t o_o = tp.add(bh.bo.data(), bh.bo.size() * 4);
        MBR_CUDA(cudaMalloc(&d_band_tiles_, tp.buf.size()));
        MBR_CUDA(cudaMemcpy(d_band_tiles_, tp.buf.data(), tp.buf.size(), cudaMemcpyHostToDevice));
        uint8_t* base = (uint8_t*)d_band_tiles_;
        band_tiles_.jl = (const int*)(base + o_j);
        band_tiles_.jr = (const int*)(base + o_jr);
        band_tiles_.bk = (const int*)(base + o_k);
        band_tiles_.bo = (const int*)(base + o_o);
        band_tiles_.count = bh.count;
        band_tiles_.stride = bh.stride;
        band_tiles_.max_n = bh.max_n;
    }
    Packer pk;
    size_t o_fi = pk.add(fi.data(), fi.size() * 4);
    size_t o_jofs = pk.add(jofs.data(), jofs.size() * 4);
    size_t o_kofs = pk.add(band_kofs_.data(), band_kofs_.size() * 4);
    size_t o_roff = pk.add(rev_off.data(), rev_off.size() * 4);
    size_t o_ridx = pk.add(rev_idx.data(), rev_idx.size() * 4);
    size_t o_nbpf = pk.add(nbpf.data(), nbpf.size() * 4);
    // periodic Hann (hann_window_kernel, src/stft_cuda_tile.cu:501-510) and twiddles
    std::vector<float> win(2048);
    for (int i = 0; i < 2048; ++i) win[i] = (float)(0.5 * (1.0 - std::cos(2.0 * M_PI * (double)i / 2048.0)));
    std::vector<float2> tw(1024);
    for (int k = 0; k < 1024; ++k)
        tw[k] = make_float2((float)std::cos(-2.0 * M_PI * k / 2048.0), (float)std::sin(-2.0 * M_PI * k / 2048.0));
    size_t o_win = pk.add(win.data(), win.size() * 4);
    size_t o_tw = pk.add(tw.data(), tw.size() * 8);

    const size_t es = dtype_bytes(dtype_);
    auto add_matrix = [&](const HostTensor& t, int rows, int cols) -> size_t {
        MBR_CHECK(t.ndim() == 2 && t.shape[0] == rows && t.shape[1] == cols, "weight shape mismatch");
        std::vector<uint8_t> tmp((size_t)rows * cols * es);
        for (int64_t i = 0; i < (int64_t)rows * cols; ++i) store_as(tmp.data(), dtype_, i, t.f(i));
        return pk.add(tmp.data(), tmp.size());
    };
    auto add_vec = [&](const HostTensor& t, int n) -> size_t {
        MBR_CHECK(t.numel() == n, "vector shape mismatch");
        std::vector<float> v = to_floats(t);
        return pk.add(v.data(), v.size() * 4);
    };

    // ---- band split: block-diagonal weight [D][KP], gammas [2J], biases [NB][D] ----
    size_t o_wbs, o_bsg, o_bsb;
    {
        std::vector<uint8_t> wbs((size_t)D_ * KP_ * es, 0);
        std::vector<float> g(2 * J_), bias((size_t)NB_ * D_);
        for (int b = 0; b < NB_; ++b) {
            std::string p = "band_split.to_features." + std::to_string(b);
            const HostTensor& gt = w.get(p + ".0.gamma");
            const HostTensor& wt = w.get(p + ".1.weight");
            const HostTensor& bt = w.get(p + ".1.bias");
            int bd = band_bd_[b];
            MBR_CHECK(gt.numel() == bd && wt.ndim() == 2 && wt.shape[0] == D_ && wt.shape[1] == bd &&
                          bt.numel() == D_,
                      "band_split weight shape mismatch in band " + std::to_string(b));
            for (int q = 0; q < bd; ++q) g[band_boff_[b] + q] = gt.f(q);
            for (int n = 0; n < D_; ++n) {
                bias[(size_t)b * D_ + n] = bt.f(n);
                for (int q = 0; q < bd; ++q)
                    store_as(wbs.data(), dtype_, (int64_t)n * KP_ + band_kofs_[b] + q, wt.f((int64_t)n * bd + q));
            }
        }
        o_wbs = pk.add(wbs.data(), wbs.size());
        o_bsg = pk.add(g.data(), g.size() * 4);
        o_bsb = pk.add(bias.data(), bias.size() * 4);
    }

    // ---- transformers ----
    struct LayerOff {
        size_t ag, qkv, wg, bg, wo, fg, w1, b1, w2, b2;
    };
    std::vector<std::vector<LayerOff>> loff;  // [depth*2][layers]
    std::vector<size_t> fgoff;
    for (int d = 0; d < c.depth; ++d)
        for (int kind = 0; kind < 2; ++kind) {
            std::string tp = "layers." + std::to_string(d) + "." + std::to_string(kind);
            int nl = kind == 0 ? c.time_transformer_depth : c.freq_transformer_depth;
            std::vector<LayerOff> lv;
            for (int l = 0; l < nl; ++l) {
                std::string lp = tp + ".layers." + std::to_string(l);
                LayerOff o;
                o.ag = add_vec(w.get(lp + ".0.norm.gamma"), D_);
                o.qkv = add_matrix(w.get(lp + ".0.to_qkv.weight"), 3 * DI_, D_);
                {
                    const HostTensor& g = w.get(lp + ".0.to_gates.weight");
                    MBR_CHECK(g.ndim() == 2 && g.shape[0] == H_ && g.shape[1] == D_, "to_gates shape mismatch");
                    std::vector<float> v((size_t)H_ * D_);
                    // 2-D weight: rounded to the compute dtype like every linear weight
                    for (int64_t i = 0; i < (int64_t)v.size(); ++i)
                        v[i] = g.dtype == DT_F32 ? round_to(g.f(i), dtype_) : g.f(i);
                    o.wg = pk.add(v.data(), v.size() * 4);
                }
                o.bg = add_vec(w.get(lp + ".0.to_gates.bias"), H_);
                o.wo = add_matrix(w.get(lp + ".0.to_out.0.weight"), D_, DI_);
                o.fg = add_vec(w.get(lp + ".1.net.0.gamma"), D_);
                o.w1 = add_matrix(w.get(lp + ".1.net.1.weight"), hid_, D_);
                o.b1 = add_vec(w.get(lp + ".1.net.1.bias"), hid_);
                o.w2 = add_matrix(w.get(lp + ".1.net.4.weight"), D_, hid_);
                o.b2 = add_vec(w.get(lp + ".1.net.4.bias"), D_);
                lv.push_back(o);
            }
            loff.push_back(lv);
            fgoff.push_back(add_vec(w.get(tp + ".norm.gamma"), D_));
        }

    // ---- mask estimators: per layer all bands stacked; the last layer's rows are
    // interleaved (value_j, gate_j) so the GLU pairs are adjacent columns ----
    int md = c.mask_estimator_depth;
    std::vector<std::vector<size_t>> mw(c.num_stems), mb(c.num_stems);
    for (int s = 0; s < c.num_stems; ++s) {
        for (int i = 0; i <= md; ++i) {
            int in = i == 0 ? D_ : hid_;
            bool last = i == md;
            int64_t rows = last ? 2 * (int64_t)band_boff_[NB_] : (int64_t)NB_ * hid_;
            std::vector<uint8_t> wm((size_t)rows * in * es);
            std::vector<float> bm((size_t)rows);
            for (int b = 0; b < NB_; ++b) {
                std::string p = "mask_estimators." + std::to_string(s) + ".to_freqs." + std::to_string(b) + ".0." +
                                std::to_string(2 * i);
                const HostTensor& wt = w.get(p + ".weight");
                const HostTensor& bt = w.get(p + ".bias");
                int out = last ? 2 * band_bd_[b] : hid_;
                MBR_CHECK(wt.ndim() == 2 && wt.shape[0] == out && wt.shape[1] == in && bt.numel() == out,
                          "mask estimator shape mismatch: " + p);
                int64_t r0 = last ? 2 * (int64_t)band_boff_[b] : (int64_t)b * hid_;
                for (int r = 0; r < out; ++r) {
                    int src = r;
                    if (last) {
                        int bd = band_bd_[b];
                        src = (r & 1) ? bd + r / 2 : r / 2;
                    }
                    bm[r0 + r] = bt.f(src);
                    for (int k = 0; k < in; ++k)
                        store_as(wm.data(), dtype_, (r0 + r) * in + k, wt.f((int64_t)src * in + k));
                }
            }
            mw[s].push_back(pk.add(wm.data(), wm.size()));
            mb[s].push_back(pk.add(bm.data(), bm.size() * 4));
        }
    }

    MBR_CUDA(cudaMalloc(&wbase_, pk.buf.size()));
    MBR_CUDA(cudaMemcpy(wbase_, pk.buf.data(), pk.buf.size(), cudaMemcpyHostToDevice));
    MBR_CUDA(cudaMalloc(&d_err_, 256));
    MBR_CUDA(cudaMemset(d_err_, 0, 256));
    uint8_t* base = (uint8_t*)wbase_;
    d_fi_ = (int*)(base + o_fi);
    d_band_jofs_ = (int*)(base + o_jofs);
    d_band_kofs_ = (int*)(base + o_kofs);
    d_rev_off_ = (int*)(base + o_roff);
    d_rev_idx_ = (int*)(base + o_ridx);
    d_nbpf_ = (float*)(base + o_nbpf);
    d_window_ = (float*)(base + o_win);
    d_twiddle_ = (float2*)(base + o_tw);
    d_wbs_ = base + o_wbs;
    d_bs_gamma_ = (float*)(base + o_bsg);
    d_bs_bias_ = (float*)(base + o_bsb);
    size_t li = 0;
    for (int d = 0; d < c.depth; ++d)
        for (int kind = 0; kind < 2; ++kind, ++li) {
            TransW tw2;
            for (auto& o : loff[li]) {
                LayerW lw;
                lw.attn_gamma = (float*)(base + o.ag);
                lw.wqkv = base + o.qkv;
                lw.wg = (float*)(base + o.wg);
                lw.bg = (float*)(base + o.bg);
                lw.wo = base + o.wo;
                lw.ff_gamma = (float*)(base + o.fg);
                lw.w1 = base + o.w1;
                lw.b1 = (float*)(base + o.b1);
                lw.w2 = base + o.w2;
                lw.b2 = (float*)(base + o.b2);
                tw2.layers.push_back(lw);
            }
            tw2.final_gamma = (float*)(base + fgoff[li]);
            (kind == 0 ? tt_ : ft_).push_back(tw2);
        }
    mask_.resize(c.num_stems);
    for (int s = 0; s < c.num_stems; ++s)
        for (int i = 0; i <= md; ++i) {
            mask_[s].w.push_back(base + mw[s][i]);
            mask_[s].b.push_back((float*)(base + mb[s][i]));
        }
    gemm_backend_ = dtype_ == DT_F32 ? BACKEND_SIMT : BACKEND_TC;
    attn_backend_ = dtype_ == DT_F32 ? BACKEND_SIMT : BACKEND_TC;
    const char* ff = std::getenv("MBR_FFN_FUSED");
    ffn_fused_ = ff && ff[0] == '1';
}

MelBandRoformer::~MelBandRoformer() {
    cudaSetDevice(device_);
    for (auto& kv : ws_) {
        cudaFree(kv.second->base);
        if (kv.second->d_tiles) cudaFree(kv.second->d_tiles);
        for (Workspace::Graph& g : kv.second->graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
    }
    cudaFree(d_err_);
    cudaFree(wbase_);
    if (d_band_tiles_) cudaFree(d_band_tiles_);
}

void MelBandRoformer::check_device_error() {
    int e = 0;
    MBR_CUDA(cudaSetDevice(device_));
    MBR_CUDA(cudaMemcpy(&e, d_err_, sizeof(int), cudaMemcpyDeviceToHost));
    if (e != 0) {
        MBR_CUDA(cudaMemset(d_err_, 0, sizeof(int)));
        if (e == 2) throw Error(ERR_CUDA, "a tensor-core kernel found its shared memory window misaligned");
        throw Error(ERR_TIMEOUT, "a tensor-core kernel timed out waiting on a pipeline barrier (error " +
                                     std::to_string(e) + ")");
    }
}

int64_t MelBandRoformer::frames(int64_t L) const {
    int n_fft = cfg_.stft_n_fft;
    return (L + 2 * (n_fft / 2) - n_fft) / cfg_.stft_hop_length + 1;
}

int64_t MelBandRoformer::out_length(int64_t L) const {
    return cfg_.match_input_audio_length ? L : (frames(L) - 1) * cfg_.stft_hop_length;
}

MelBandRoformer::Workspace& MelBandRoformer::workspace(int B, int64_t L) {
    auto key = std::make_pair(B, L);
    auto it = ws_.find(key);
    if (it != ws_.end()) return *it->second;
    MBR_CHECK(L > cfg_.stft_n_fft / 2, "input shorter than the STFT reflect padding");
    auto ws = std::make_unique<Workspace>();
    ws->B = B;
    ws->L = L;
    ws->T = frames(L);
    ws->MT = (int64_t)B * ws->T;
    ws->M = ws->MT * NB_;
    ws->lout = out_length(L);
    const int64_t T = ws->T, MT = ws->MT, M = ws->M;
    const int S = cfg_.num_stems;
    const size_t es = dtype_bytes(dtype_);
    size_t off = 0;
    std::vector<std::pair<void**, size_t>> items;
    auto take = [&](void** p, size_t bytes) { items.emplace_back(p, bytes); };
    take((void**)&ws->spec, sizeof(float2) * MT * F_ * C_);
    take(&ws->xb, es * MT * KP_);
    take((void**)&ws->R, 4 * M * D_);
    take(&ws->xn, es * M * D_);
    take((void**)&ws->gates, 4 * M * H_);
    take(&ws->qkv, es * M * 3 * DI_);
    take(&ws->q, es * M * DI_);
    take(&ws->k, es * M * DI_);
    take(&ws->v, es * M * DI_);
    take(&ws->merged, es * M * DI_);
    take(&ws->hf, es * M * hid_);
    take(&ws->rm, es * M * D_);
    take(&ws->mh[0], es * (size_t)NB_ * MT * hid_);
    take(&ws->mh[1], es * (size_t)NB_ * MT * hid_);
    take((void**)&ws->masks, 4 * (size_t)S * MT * 2 * J_);
    take((void**)&ws->y, sizeof(float2) * (size_t)B * S * C_ * T * F_);
    take((void**)&ws->frames, 4 * (size_t)B * S * C_ * T * 2048);
    take((void**)&ws->rope_t_cos, 4 * T * dh_ / 2);
    take((void**)&ws->rope_t_sin, 4 * T * dh_ / 2);
    take((void**)&ws->rope_f_cos, 4 * NB_ * dh_ / 2);
    take((void**)&ws->rope_f_sin, 4 * NB_ * dh_ / 2);
    if (cfg_.skip_connection) ws->skip.resize(cfg_.depth);
    for (auto& p : ws->skip) take((void**)&p, 4 * M * D_);
    // group descriptors: band split + 4 per transformer layer + mask layers
    size_t ngroups = NB_;
    for (int d = 0; d < cfg_.depth; ++d) ngroups += 4 * (cfg_.time_transformer_depth + cfg_.freq_transformer_depth);
    ngroups += (size_t)S * (cfg_.mask_estimator_depth + 1) * NB_;
    take((void**)&ws->d_groups, sizeof(ops::GemmGroup) * ngroups);
    for (auto& it2 : items) {
        off = round_up((int64_t)off, 256);
        size_t o = off;
        off += it2.second;
        *it2.first = (void*)o;  // offset for now
    }
    ws->bytes = off;
    MBR_CUDA(cudaMalloc(&ws->base, ws->bytes));
    for (auto& it2 : items) *it2.first = (uint8_t*)ws->base + (size_t)*it2.first;
    std::vector<float> cs, sn;
    rotary_tables((int)T, dh_, cs, sn);
    MBR_CUDA(cudaMemcpy(ws->rope_t_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    MBR_CUDA(cudaMemcpy(ws->rope_t_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    rotary_tables(NB_, dh_, cs, sn);
    MBR_CUDA(cudaMemcpy(ws->rope_f_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    MBR_CUDA(cudaMemcpy(ws->rope_f_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    build_plans(*ws);
    MBR_CUDA(cudaMemcpy(ws->d_groups, ws->h_groups.data(), ws->h_groups.size() * sizeof(ops::GemmGroup),
                        cudaMemcpyHostToDevice));
    if (dtype_ != DT_F32) {
        // tensor-core launches: tensor maps + tile lists of every GEMM plan
        std::vector<int4> tiles;
        std::vector<size_t> firsts;
        std::vector<Plan*> plans{&ws->band_split};
        for (auto& p : ws->layer_plans) plans.push_back(&p);
        for (auto& v : ws->mask_plans)
            for (auto& p : v) plans.push_back(&p);
        for (Plan* p : plans) {
            tc::GemmPlanTC tp;
            tp.groups = ws->d_groups + p->first;
            tp.h_groups = ws->h_groups.data() + p->first;
            tp.ngroups = p->n;
            tp.maxM = p->maxM;
            tp.maxN = p->maxN;
            tp.epi = p->epi;
            tp.a_base = p->a_base;
            tp.a_rows = p->a_rows;
            tp.a_cols = p->a_cols;
            tp.b_base = p->b_base;
            tp.b_rows = p->b_rows;
            tp.b_cols = p->b_cols;
            tp.c_base = p->c_base;
            tp.c_rows = p->c_rows;
            tp.c_cols = p->c_cols;
            tp.c_groups = p->c_groups;
            tp.c_row_stride = p->c_row_stride;
            tp.c_group_stride = p->c_group_stride;
            tp.c_dtype = p->c_dtype;
            tc::GemmLaunch L;
            const bool qkv = p->qkv_mode >= 0 && dh_ == 64;
            if (qkv) {
                L.qkv.mode = p->qkv_mode;
                L.qkv.NB = NB_;
                L.qkv.T = (int)ws->T;
                L.qkv.H = H_;
                L.qkv.cos_t = p->qkv_mode == ops::SEQ_TIME ? ws->rope_t_cos : ws->rope_f_cos;
                L.qkv.sin_t = p->qkv_mode == ops::SEQ_TIME ? ws->rope_t_sin : ws->rope_f_sin;
                L.qkv.q = ws->q;
                L.qkv.k = ws->k;
                L.qkv.v = ws->v;
                // RoPE in the epilogue, q|k|v stored token-major through TMA
                tp.epi = ops::EPI_ROPE_T;
                tp.c_base = ws->qkv, tp.c_rows = ws->M, tp.c_cols = 3 * DI_, tp.c_groups = 1;
                tp.c_row_stride = 3 * DI_, tp.c_group_stride = ws->M * 3 * DI_, tp.c_dtype = dtype_;
            }
            size_t first = 0;
            tc::gemm_prepare(tp, dtype_, tiles, L, first);
            p->launch = (int)ws->launches.size();
            ws->launches.push_back(L);
            firsts.push_back(first);
            if (qkv) {
                // RoPE + head-major scatter for the CUDA-core attention
                tc::GemmPlanTC ts = tp;
                ts.epi = ops::EPI_QKV;
                ts.c_dtype = -1;
                tc::GemmLaunch Ls;
                Ls.qkv = L.qkv;
                tc::gemm_prepare(ts, dtype_, tiles, Ls, first);
                p->launch_scatter = (int)ws->launches.size();
                ws->launches.push_back(Ls);
                firsts.push_back(first);
            }
        }
        // the fused FFN blocks (FFN1 + GELU + FFN2 + residual) of every layer
        std::vector<size_t> ffn_firsts;
        if (ffn_fused_ && tc::ffn_supported(D_, hid_, dtype_)) {
            for (size_t i = 0; i + 3 < ws->layer_plans.size(); i += 4) {
                Plan& p1 = ws->layer_plans[i + 2];
                const Plan& p2 = ws->layer_plans[i + 3];
                tc::FfnLaunch F;
                size_t first = 0;
                tc::ffn_prepare(p1.a_base, p1.b_base, ws->h_groups[p1.first].bias, p2.b_base,
                                ws->h_groups[p2.first].bias, ws->R, ws->M, D_, hid_, dtype_, tiles, F, first);
                p1.ffn = (int)ws->ffn_launches.size();
                ws->ffn_launches.push_back(F);
                ffn_firsts.push_back(first);
            }
        }
        MBR_CUDA(cudaMalloc(&ws->d_tiles, sizeof(int4) * std::max<size_t>(1, tiles.size())));
        MBR_CUDA(cudaMemcpy(ws->d_tiles, tiles.data(), sizeof(int4) * tiles.size(), cudaMemcpyHostToDevice));
        for (size_t i = 0; i < ws->launches.size(); ++i) ws->launches[i].tiles = ws->d_tiles + firsts[i];
        for (size_t i = 0; i < ws->ffn_launches.size(); ++i) ws->ffn_launches[i].items = ws->d_tiles + ffn_firsts[i];
    }
    Workspace& ref = *ws;
    ws_[key] = std::move(ws);
    return ref;
}

void MelBandRoformer::build_plans(Workspace& ws) {
    const size_t es = dtype_bytes(dtype_);
    const int64_t MT = ws.MT, M = ws.M;
    auto& G = ws.h_groups;
    G.clear();
    auto begin = [&](Plan& p, int epi) {
        p.first = G.size();
        p.epi = epi;
    };
    auto push = [&](Plan& p, const ops::GemmGroup& g) {
        G.push_back(g);
        p.n++;
        p.maxM = std::max(p.maxM, g.M);
        p.maxN = std::max(p.maxN, g.N);
        p.maxK = std::max(p.maxK, g.K);
    };
    auto view = [](Plan& p, const void* base, int64_t rows, int64_t cols, int64_t groups, int64_t row_stride,
                   int64_t group_stride, int cdt) {
        p.c_base = base;
        p.c_rows = rows;
        p.c_cols = cols;
        p.c_groups = groups;
        p.c_row_stride = row_stride;
        p.c_group_stride = group_stride;
        p.c_dtype = cdt;
    };
    auto mk = [](const void* A, int64_t lda, const void* B, int64_t ldb, void* Cp, int64_t ldc, const float* bias,
                 int64_t M, int N, int K) {
        ops::GemmGroup g{};
        g.A = A;
        g.B = B;
        g.C = Cp;
        g.bias = bias;
        g.lda = lda;
        g.ldb = ldb;
        g.ldc = ldc;
        g.M = (int)M;
        g.N = N;
        g.K = K;
        return g;
    };
    // band split (apply_band_split, src/model_mel_band_roformer.cu:572-604)
    begin(ws.band_split, ops::EPI_F32);
    ws.band_split.a_base = ws.xb;
    ws.band_split.a_rows = MT;
    ws.band_split.a_cols = KP_;
    ws.band_split.b_base = d_wbs_;
    ws.band_split.b_rows = D_;
    ws.band_split.b_cols = KP_;
    view(ws.band_split, ws.R, MT, D_, NB_, (int64_t)NB_ * D_, D_, DT_F32);
    for (int b = 0; b < NB_; ++b) {
        int k0 = band_kofs_[b], kn = band_kofs_[b + 1] - k0;
        ops::GemmGroup g = mk((uint8_t*)ws.xb + es * k0, KP_, (uint8_t*)d_wbs_ + es * k0, KP_, ws.R + (size_t)b * D_,
                              (int64_t)NB_ * D_, d_bs_bias_ + (size_t)b * D_, MT, D_, kn);
        g.k_col0 = k0;
        g.c_group = b;
        push(ws.band_split, g);
    }
    // transformer layers
    ws.layer_plans.clear();
    for (int d = 0; d < cfg_.depth; ++d)
        for (int kind = 0; kind < 2; ++kind) {
            const TransW& tw = kind == 0 ? tt_[d] : ft_[d];
            for (const LayerW& lw : tw.layers) {
                Plan p[4];
                begin(p[0], ops::EPI_T);
                p[0].qkv_mode = kind;
                p[0].a_base = ws.xn, p[0].a_rows = M, p[0].a_cols = D_;
                p[0].b_base = lw.wqkv, p[0].b_rows = 3 * DI_, p[0].b_cols = D_;
                push(p[0], mk(ws.xn, D_, lw.wqkv, D_, ws.qkv, 3 * DI_, nullptr, M, 3 * DI_, D_));
                begin(p[1], ops::EPI_ADD_F32);
                p[1].a_base = ws.merged, p[1].a_rows = M, p[1].a_cols = DI_;
                p[1].b_base = lw.wo, p[1].b_rows = D_, p[1].b_cols = DI_;
                view(p[1], ws.R, M, D_, 1, D_, M * D_, DT_F32);
                push(p[1], mk(ws.merged, DI_, lw.wo, DI_, ws.R, D_, nullptr, M, D_, DI_));
                begin(p[2], ops::EPI_GELU_T);
                p[2].a_base = ws.xn, p[2].a_rows = M, p[2].a_cols = D_;
                p[2].b_base = lw.w1, p[2].b_rows = hid_, p[2].b_cols = D_;
                view(p[2], ws.hf, M, hid_, 1, hid_, M * hid_, dtype_);
                push(p[2], mk(ws.xn, D_, lw.w1, D_, ws.hf, hid_, lw.b1, M, hid_, D_));
                begin(p[3], ops::EPI_ADD_F32);
                p[3].a_base = ws.hf, p[3].a_rows = M, p[3].a_cols = hid_;
                p[3].b_base = lw.w2, p[3].b_rows = D_, p[3].b_cols = hid_;
                view(p[3], ws.R, M, D_, 1, D_, M * D_, DT_F32);
                push(p[3], mk(ws.hf, hid_, lw.w2, hid_, ws.R, D_, lw.b2, M, D_, hid_));
                for (auto& q : p) ws.layer_plans.push_back(q);
            }
        }
    // mask estimators (apply_mask_estimator, src/model_mel_band_roformer.cu:610-676)
    int md = cfg_.mask_estimator_depth;
    ws.mask_plans.assign(cfg_.num_stems, {});
    for (int s = 0; s < cfg_.num_stems; ++s)
        for (int i = 0; i <= md; ++i) {
            bool last = i == md;
            int in = i == 0 ? D_ : hid_;
            const void* A = i == 0 ? ws.rm : ws.mh[(i - 1) & 1];
            Plan p;
            begin(p, last ? ops::EPI_GLU_F32 : ops::EPI_TANH_T);
            p.a_base = A, p.a_rows = (int64_t)NB_ * MT, p.a_cols = in;
            p.b_base = mask_[s].w[i];
            p.b_rows = last ? 2 * (int64_t)band_boff_[NB_] : (int64_t)NB_ * hid_;
            p.b_cols = in;
            if (!last) view(p, ws.mh[i & 1], MT, hid_, NB_, hid_, MT * hid_, dtype_);
            for (int b = 0; b < NB_; ++b) {
                const uint8_t* Ab = (const uint8_t*)A + es * (size_t)b * MT * in;
                ops::GemmGroup g;
                if (!last) {
                    g = mk(Ab, in, (uint8_t*)mask_[s].w[i] + es * (size_t)b * hid_ * in, in,
                           (uint8_t*)ws.mh[i & 1] + es * (size_t)b * MT * hid_, hid_,
                           mask_[s].b[i] + (size_t)b * hid_, MT, hid_, in);
                    g.b_row0 = b * hid_;
                    g.c_group = b;
                } else {
                    int r0 = 2 * band_boff_[b];
                    g = mk(Ab, in, (uint8_t*)mask_[s].w[i] + es * (size_t)r0 * in, in,
                           ws.masks + (size_t)s * MT * 2 * J_ + band_boff_[b], 2 * J_, mask_[s].b[i] + r0, MT,
                           2 * band_bd_[b], in);
                    g.b_row0 = r0;
                }
                g.a_row0 = (int)(b * MT);
                push(p, g);
            }
            ws.mask_plans[s].push_back(p);
        }
}

// ---- profiler ----
void MelBandRoformer::profile_enable(bool on) {
    prof_on_ = on;
    profile_reset();
}

void MelBandRoformer::profile_reset() {
    prof_recs_.clear();
    prof_used_ = 0;
    for (int i = 0; i < PK_COUNT; ++i) prof_ms_[i] = 0.0, prof_n_[i] = 0;
}

int MelBandRoformer::prof_begin(int kind, cudaStream_t st) {
    while (prof_pool_.size() < prof_used_ + 2) {
        cudaEvent_t e;
        MBR_CUDA(cudaEventCreate(&e));
        prof_pool_.push_back(e);
    }
    ProfRec r{kind, prof_pool_[prof_used_], prof_pool_[prof_used_ + 1]};
    prof_used_ += 2;
    MBR_CUDA(cudaEventRecord(r.a, st));
    prof_recs_.push_back(r);
    return (int)prof_recs_.size() - 1;
}

void MelBandRoformer::prof_end(int rec, cudaStream_t st) { MBR_CUDA(cudaEventRecord(prof_recs_[rec].b, st)); }

void MelBandRoformer::prof_collect() {
    for (auto& r : prof_recs_) {
        MBR_CUDA(cudaEventSynchronize(r.b));
        float ms = 0.f;
        MBR_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        prof_ms_[r.kind] += ms;
        prof_n_[r.kind] += 1;
    }
    prof_recs_.clear();
    prof_used_ = 0;
}

void MelBandRoformer::profile_read(int kind, double* ms, int64_t* count) {
    MBR_CHECK(kind >= 0 && kind < PK_COUNT, "profile kind out of range");
    MBR_CUDA(cudaSetDevice(device_));
    prof_collect();
    *ms = prof_ms_[kind];
    *count = prof_n_[kind];
}

// Runs `fn` (one kernel launch) bracketed by profiler events when enabled.
#define MBR_LAUNCH(kind, ...)                                    \
    do {                                                         \
        int rec_ = prof_on_ ? prof_begin((kind), st) : -1;       \
        __VA_ARGS__;                                             \
        if (rec_ >= 0) prof_end(rec_, st);                       \
        ++launches_;                                             \
    } while (0)

void MelBandRoformer::run_gemm(const Workspace& ws, const Plan& p, int kind, cudaStream_t st, int launch) {
    if (launch < 0) launch = p.launch;
    if (gemm_backend_ != BACKEND_SIMT && dtype_ != DT_F32 && launch >= 0) {
        if (gemm_backend_ == BACKEND_TC_DIRECT && ws.launches[launch].c_tma) {
            tc::GemmLaunch L = ws.launches[launch];
            L.c_tma = 0;  // epilogue stores from registers
            MBR_LAUNCH(kind, tc::gemm_launch(L, dtype_, d_err_, st));
        } else {
            MBR_LAUNCH(kind, tc::gemm_launch(ws.launches[launch], dtype_, d_err_, st));
        }
    } else {
        MBR_LAUNCH(kind, ops::gemm_simt(ws.d_groups + p.first, p.n, p.maxM, p.maxN, dtype_, p.epi, st));
    }
}

void MelBandRoformer::run_transformer(Workspace& ws, const TransW& tw, int mode, const Plan* plans,
                                      bool last_of_model, cudaStream_t st, bool first_norm_done,
                                      const LayerW* next_first) {
    const float scale = std::sqrt((float)D_);
    const float attn_scale = 1.0f / std::sqrt((float)dh_);
    const int64_t M = ws.M;
    const int L = mode == ops::SEQ_TIME ? (int)ws.T : NB_;
    const int64_t nseq = M / L;
    const float* rc = mode == ops::SEQ_TIME ? ws.rope_t_cos : ws.rope_f_cos;
    const float* rs = mode == ops::SEQ_TIME ? ws.rope_t_sin : ws.rope_f_sin;
    const int attn_kind = mode == ops::SEQ_TIME ? PK_ATTN_TIME : PK_ATTN_FREQ;
    for (size_t l = 0; l < tw.layers.size(); ++l) {
        const LayerW& lw = tw.layers[l];
        const Plan* p = plans + 4 * l;
        if (l > 0 || !first_norm_done)  // else the previous block's final norm produced xn and the gates
            MBR_LAUNCH(PK_NORM, ops::rms_norm(ws.R, M, D_, lw.attn_gamma, scale, ws.xn, dtype_, 0, NB_, nullptr,
                                              lw.wg, lw.bg, H_, ws.gates, st));
        const bool tc_gemm = gemm_backend_ != BACKEND_SIMT && dtype_ != DT_F32 && p[0].launch >= 0;
        const bool tc_attn = attn_backend_ == BACKEND_TC && dtype_ != DT_F32 && tc::attention_supported(dh_);
        // tensor cores end to end: the QKV GEMM applies RoPE and stores q|k|v
        // token-major; the attention reads them there through strided TMA views
        const bool in_place = tc_gemm && tc_attn && p[0].launch_scatter >= 0;
        if (in_place) {
            run_gemm(ws, p[0], PK_GEMM_QKV, st);
        } else if (tc_gemm && p[0].launch_scatter >= 0) {
            run_gemm(ws, p[0], PK_GEMM_QKV, st, p[0].launch_scatter);  // RoPE + head-major scatter
        } else {
            run_gemm(ws, p[0], PK_GEMM_QKV, st);
            MBR_LAUNCH(PK_ROPE, ops::rope_scatter(ws.qkv, M, H_, dh_, rc, rs, mode, NB_, (int)ws.T, ws.q, ws.k, ws.v,
                                                  dtype_, st));
        }
        if (in_place) {
            const int64_t row = 3 * (int64_t)DI_;  // elements per token of q|k|v
            tc::AttnLayout lay;
            lay.head = dh_;
            if (mode == ops::SEQ_TIME) {  // sequence (b, band k), position = frame t
                lay.pos = (int64_t)NB_ * row;
                lay.lo = row;
                lay.n_lo = NB_;
            } else {  // sequence (b, frame t), position = band k
                lay.pos = row;
                lay.lo = (int64_t)NB_ * row;
                lay.n_lo = (int)ws.T;
            }
            lay.hi = ws.T * NB_ * row;
            lay.n_hi = ws.B;
            const size_t es = dtype_bytes(dtype_);
            const uint8_t* q = (const uint8_t*)ws.qkv;
            MBR_LAUNCH(attn_kind, tc::attention(q, q + es * DI_, q + 2 * es * DI_, lay, nseq, H_, L, dh_, attn_scale,
                                                ws.gates, mode, NB_, (int)ws.T, ws.merged, dtype_, d_err_, st));
        } else if (tc_attn) {
            MBR_LAUNCH(attn_kind, tc::attention(ws.q, ws.k, ws.v, tc::head_major_layout(nseq, H_, L, dh_), nseq, H_, L,
                                                dh_, attn_scale, ws.gates, mode, NB_, (int)ws.T, ws.merged, dtype_,
                                                d_err_, st));
        } else {
            MBR_LAUNCH(attn_kind, ops::attention_simt(ws.q, ws.k, ws.v, nseq, H_, L, dh_, attn_scale, ws.gates, mode,
                                                      NB_, (int)ws.T, ws.merged, dtype_, st));
        }
        run_gemm(ws, p[1], PK_GEMM_OUT, st);
        MBR_LAUNCH(PK_NORM, ops::rms_norm(ws.R, M, D_, lw.ff_gamma, scale, ws.xn, dtype_, 0, NB_, nullptr, nullptr,
                                          nullptr, 0, nullptr, st));
        if (p[2].ffn >= 0) {
            MBR_LAUNCH(PK_FFN, tc::ffn_launch(ws.ffn_launches[p[2].ffn], dtype_, d_err_, st));
        } else {
            run_gemm(ws, p[2], PK_GEMM_FFN1, st);
            run_gemm(ws, p[3], PK_GEMM_FFN2, st);
        }
    }
    // final RMSNorm of the transformer; the model's last one also writes the
    // band-major 16-bit copy the mask estimators read
    if (next_first) {
        // fused with the next block's pre-norm: xn and the gates of its first layer
        MBR_LAUNCH(PK_NORM, ops::rms_norm(ws.R, M, D_, tw.final_gamma, scale, ws.xn, dtype_, 0, NB_, ws.R,
                                          next_first->wg, next_first->bg, H_, ws.gates, st,
                                          next_first->attn_gamma));
    } else {
        MBR_LAUNCH(PK_NORM, ops::rms_norm(ws.R, M, D_, tw.final_gamma, scale, last_of_model ? ws.rm : nullptr,
                                          dtype_, last_of_model ? ws.MT : 0, NB_, ws.R, nullptr, nullptr, 0, nullptr,
                                          st));
    }
}

void MelBandRoformer::run_forward(Workspace& ws, const float* d_audio, float* d_out, int tap, float* d_tap,
                                  int64_t* tap_n, cudaStream_t st) {
    const MBRConfig& c = cfg_;
    const int B = ws.B, S = c.num_stems;
    const int64_t T = ws.T, MT = ws.MT, M = ws.M;
    launches_ = 0;
    auto emit_tap = [&](int id, const void* src, int64_t n) {
        if (tap != id) return;
        *tap_n = n;
        if (d_tap) MBR_CUDA(cudaMemcpyAsync(d_tap, src, 4 * n, cudaMemcpyDeviceToDevice, st));
    };
    // 1-6: STFT, stereo merge, band gather (src/model_mel_band_roformer.cu:700-728)
    MBR_LAUNCH(PK_STFT, ops::stft(d_audio, B, C_, ws.L, c.stft_hop_length, d_window_, d_twiddle_,
                                  c.stft_normalized ? 1.0f / std::sqrt((float)c.stft_n_fft) : 1.0f, ws.spec, (int)T,
                                  st));
    MBR_LAUNCH(PK_BAND_GATHER, ops::band_gather_norm(ws.spec, MT, F_ * C_, d_fi_, d_band_jofs_, d_band_kofs_,
                                                     d_bs_gamma_, NB_, ws.xb, KP_, dtype_, st));
    // 7: band split
    run_gemm(ws, ws.band_split, PK_GEMM_BANDSPLIT, st);
    emit_tap(0, ws.R, M * D_);
    if (tap == 0) return;
    // 8: depth loop (:740-801)
    size_t pi = 0;
    // A block's final RMSNorm also computes the next block's first pre-norm
    // (and gates) when nothing happens to the residual stream in between.
    bool norm_done = false;
    for (int d = 0; d < c.depth; ++d) {
        if (c.skip_connection)
            for (int j = 0; j < d; ++j) MBR_LAUNCH(PK_NORM, ops::add_inplace_f32(ws.R, ws.skip[j], M * D_, st));
        bool last = d == c.depth - 1;
        const LayerW* nf = ft_[d].layers.empty() ? nullptr : &ft_[d].layers[0];
        run_transformer(ws, tt_[d], ops::SEQ_TIME, ws.layer_plans.data() + pi, false, st, norm_done, nf);
        norm_done = nf != nullptr;
        pi += 4 * tt_[d].layers.size();
        const LayerW* nt = (!last && !c.skip_connection && !tt_[d + 1].layers.empty()) ? &tt_[d + 1].layers[0]
                                                                                       : nullptr;
        run_transformer(ws, ft_[d], ops::SEQ_FREQ, ws.layer_plans.data() + pi, last, st, norm_done, nt);
        norm_done = nt != nullptr;
        pi += 4 * ft_[d].layers.size();
        if (c.skip_connection) MBR_CUDA(cudaMemcpyAsync(ws.skip[d], ws.R, 4 * M * D_, cudaMemcpyDeviceToDevice, st));
        if (d == 0) {
            emit_tap(1, ws.R, M * D_);
            if (tap == 1) return;
        }
    }
    emit_tap(2, ws.R, M * D_);
    if (tap == 2) return;
    // 9: mask estimators
    for (int s = 0; s < S; ++s)
        for (size_t i = 0; i < ws.mask_plans[s].size(); ++i)
            run_gemm(ws, ws.mask_plans[s][i], i + 1 < ws.mask_plans[s].size() ? PK_GEMM_MASK_HIDDEN : PK_GEMM_MASK_OUT,
                     st);
    emit_tap(3, ws.masks, MT * 2 * J_);
    if (tap == 3) return;
    // 10-11: mask apply + scatter-average + zero_dc
    MBR_LAUNCH(PK_MASK_SCATTER, ops::mask_scatter(ws.spec, ws.masks, B, S, (int)T, C_, F_, d_rev_off_, d_rev_idx_,
                                                  d_nbpf_, J_, c.zero_dc, ws.y, st));
    emit_tap(4, ws.y, (int64_t)B * S * C_ * T * F_ * 2);
    if (tap == 4) return;
    // 12: iSTFT
    int64_t nsig = (int64_t)B * S * C_;
    MBR_LAUNCH(PK_ISTFT, ops::istft_frames(ws.y, nsig, (int)T, d_window_, d_twiddle_,
                                           c.stft_normalized ? std::sqrt((float)c.stft_n_fft) : 1.0f, ws.frames, st));
    MBR_LAUNCH(PK_ISTFT, ops::istft_ola(ws.frames, nsig, (int)T, c.stft_hop_length, d_window_, ws.lout, d_out, st));
}

void MelBandRoformer::forward(const float* d_audio, int B, int64_t L, float* d_out, cudaStream_t st) {
    MBR_CHECK(B >= 1, "batch must be >= 1");
    MBR_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(B, L);
    // The legacy default stream cannot be captured; a stream the caller is
    // capturing already records our launches into the caller's graph.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool capturable = graphs_on_ && !prof_on_ && st != nullptr && st != cudaStreamLegacy &&
                            st != cudaStreamPerThread && cudaStreamIsCapturing(st, &cs) == cudaSuccess &&
                            cs == cudaStreamCaptureStatusNone;
    if (!capturable) {
        run_forward(ws, d_audio, d_out, -1, nullptr, nullptr, st);
        return;
    }
    for (const Workspace::Graph& g : ws.graphs)
        if (g.in == d_audio && g.out == d_out) {
            if (!g.exec) break;
            MBR_CUDA(cudaGraphLaunch(g.exec, st));
            launches_ = g.launches;
            return;
        }
    // first use of this buffer pair: run eagerly (sets kernel attributes and
    // computes the result), then capture the same launch sequence for reuse
    run_forward(ws, d_audio, d_out, -1, nullptr, nullptr, st);
    bool known = false;
    for (const Workspace::Graph& g : ws.graphs) known |= g.in == d_audio && g.out == d_out;
    if (known) return;  // capture failed before: stay eager
    Workspace::Graph g{d_audio, d_out, nullptr, launches_};
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        bool ok = true;
        try {
            run_forward(ws, d_audio, d_out, -1, nullptr, nullptr, st);
        } catch (const Error&) {
            ok = false;
        }
        const cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (ok && e == cudaSuccess && graph &&
            cudaGraphInstantiateWithFlags(&g.exec, graph, 0) != cudaSuccess)
            g.exec = nullptr;
        if (graph) cudaGraphDestroy(graph);
    }
    cudaGetLastError();  // a failed capture leaves no sticky error; clear the last one
    launches_ = g.launches;
    ws.graphs.push_back(g);
}

void MelBandRoformer::drop_graphs() {
    for (auto& kv : ws_)
        for (Workspace::Graph& g : kv.second->graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
    for (auto& kv : ws_) kv.second->graphs.clear();
}

int64_t MelBandRoformer::forward_tap(const float* d_audio, int B, int64_t L, int tap, float* d_tap, cudaStream_t st) {
    MBR_CHECK(tap >= 0 && tap <= 4, "tap must be in [0, 4]");
    MBR_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(B, L);
    int64_t n = 0;
    if (!d_tap) {
        const int64_t M = ws.M, MT = ws.MT;
        const int64_t sizes[5] = {M * D_, M * D_, M * D_, MT * 2 * J_,
                                  (int64_t)B * cfg_.num_stems * C_ * ws.T * F_ * 2};
        return sizes[tap];
    }
    run_forward(ws, d_audio, nullptr, tap, d_tap, &n, st);
    return n;
}

}  // namespace mbr
