// mbr_oracle.cpp — CPU oracle of the reference MelBandRoformer forward.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA product and the
// CPU baseline of bench.py.  Nothing in the product links or calls this file.
//
// Every function cites the reference file:line (baicai-1145/MBR-CUDA-Tile) whose
// behaviour it restates.  Storage is fp32; every reduction runs in fp64.
#include "mbr_oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <complex>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;
int g_threads = 0;

int nthreads() {
    if (g_threads > 0) return g_threads;
    unsigned hc = std::thread::hardware_concurrency();
    return hc == 0 ? 1 : (int)hc;
}

// Dynamic-scheduled parallel loop over [0, n).
template <class F>
void parallel_for(int64_t n, F&& f) {
    int nt = (int)std::min<int64_t>(nthreads(), n);
    if (nt <= 1) {
        for (int64_t i = 0; i < n; ++i) f(i);
        return;
    }
    std::atomic<int64_t> next(0);
    std::vector<std::thread> th;
    th.reserve(nt);
    for (int t = 0; t < nt; ++t) {
        th.emplace_back([&]() {
            for (;;) {
                int64_t i = next.fetch_add(1);
                if (i >= n) break;
                f(i);
            }
        });
    }
    for (auto& x : th) x.join();
}

// ---------------------------------------------------------------------------
// Minimal JSON (restates the parser of src/weights.cu:170-406 for the subset
// the .csm config uses: objects, arrays, numbers, strings, bools, null).
// ---------------------------------------------------------------------------
struct Json {
    enum T { Null, Bool, Num, Str, Arr, Obj } t = Null;
    bool b = false;
    double n = 0;
    std::string s;
    std::vector<Json> a;
    std::vector<std::pair<std::string, Json>> o;
    const Json* get(const std::string& k) const {
        for (auto& kv : o)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JsonParser {
    const std::string& src;
    size_t p = 0;
    explicit JsonParser(const std::string& s) : src(s) {}
    void ws() {
        while (p < src.size() && (src[p] == ' ' || src[p] == '\n' || src[p] == '\r' || src[p] == '\t')) ++p;
    }
    [[noreturn]] void fail(const char* m) { throw std::runtime_error(std::string("json: ") + m); }
    std::string str() {
        if (src[p] != '"') fail("expected string");
        ++p;
        std::string out;
        while (p < src.size() && src[p] != '"') {
            char c = src[p++];
            if (c == '\\') {
                if (p >= src.size()) fail("bad escape");
                char e = src[p++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (p + 4 > src.size()) fail("bad \\u");
                        unsigned cp = (unsigned)std::stoul(src.substr(p, 4), nullptr, 16);
                        p += 4;
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
                        else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (p >= src.size()) fail("unterminated string");
        ++p;
        return out;
    }
    Json val() {
        ws();
        if (p >= src.size()) fail("eof");
        Json j;
        char c = src[p];
        if (c == '{') {
            j.t = Json::Obj;
            ++p;
            ws();
            if (src[p] == '}') { ++p; return j; }
            for (;;) {
                ws();
                std::string k = str();
                ws();
                if (src[p] != ':') fail("expected :");
                ++p;
                j.o.emplace_back(k, val());
                ws();
                if (src[p] == ',') { ++p; continue; }
                if (src[p] == '}') { ++p; break; }
                fail("expected , or }");
            }
        } else if (c == '[') {
            j.t = Json::Arr;
            ++p;
            ws();
            if (src[p] == ']') { ++p; return j; }
            for (;;) {
                j.a.push_back(val());
                ws();
                if (src[p] == ',') { ++p; continue; }
                if (src[p] == ']') { ++p; break; }
                fail("expected , or ]");
            }
        } else if (c == '"') {
            j.t = Json::Str;
            j.s = str();
        } else if (src.compare(p, 4, "true") == 0) {
            j.t = Json::Bool; j.b = true; p += 4;
        } else if (src.compare(p, 5, "false") == 0) {
            j.t = Json::Bool; j.b = false; p += 5;
        } else if (src.compare(p, 4, "null") == 0) {
            p += 4;
        } else {
            size_t q = p;
            while (q < src.size() && (std::isdigit((unsigned char)src[q]) || src[q] == '-' || src[q] == '+' ||
                                      src[q] == '.' || src[q] == 'e' || src[q] == 'E'))
                ++q;
            if (q == p) fail("bad value");
            j.t = Json::Num;
            j.n = std::strtod(src.substr(p, q - p).c_str(), nullptr);
            p = q;
        }
        return j;
    }
};

int jint(const Json& j, const char* k, int def) {
    const Json* v = j.get(k);
    if (!v) return def;
    if (v->t == Json::Num) return (int)v->n;
    if (v->t == Json::Bool) return v->b ? 1 : 0;
    return def;
}
bool jbool(const Json& j, const char* k, bool def) {
    const Json* v = j.get(k);
    if (!v) return def;
    if (v->t == Json::Bool) return v->b;
    if (v->t == Json::Num) return v->n != 0;
    return def;
}

// ---------------------------------------------------------------------------
// fp16 / bf16 rounding (round-to-nearest-even), used to restate
// ModelWeights::convert_linear_weights_to_{fp16,bf16} (src/weights.cu:511-540).
// ---------------------------------------------------------------------------
float round_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}
float round_fp16(float x) { return (float)(_Float16)x; }
float half_bits_to_float(uint16_t h) {
    _Float16 v;
    std::memcpy(&v, &h, 2);
    return (float)v;
}
float bf16_bits_to_float(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// ---------------------------------------------------------------------------
// .csm v1 reader (restates ModelWeights::load, src/weights.cu:412-509 and the
// byte layout documented at src/weights.h:82-96).
// ---------------------------------------------------------------------------
struct CsmTensor {
    std::vector<int64_t> shape;
    int dtype = 0;  // 0 f32, 1 f16, 2 i64, 3 bf16
    std::vector<float> f;
    std::vector<int64_t> i;
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
};

struct Csm {
    Json config;
    std::map<std::string, CsmTensor> t;
    const CsmTensor& get(const std::string& k) const {
        auto it = t.find(k);
        if (it == t.end()) throw std::runtime_error("ModelWeights: tensor not found: " + k);
        return it->second;
    }
    bool has(const std::string& k) const { return t.count(k) > 0; }
};

Csm read_csm(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("ModelWeights: cannot open file: " + path);
    auto rd = [&](void* d, size_t n) {
        f.read((char*)d, (std::streamsize)n);
        if (!f) throw std::runtime_error("ModelWeights: unexpected EOF");
    };
    char magic[4];
    rd(magic, 4);
    if (magic[0] != 'C' || magic[1] != 'S' || magic[2] != 'M' || magic[3] != 0)
        throw std::runtime_error("ModelWeights: invalid magic (expected CSM\\0)");
    uint32_t ver, jlen, nt;
    rd(&ver, 4);
    if (ver != 1) throw std::runtime_error("ModelWeights: unsupported version");
    rd(&jlen, 4);
    std::string js(jlen, '\0');
    rd(&js[0], jlen);
    Csm c;
    JsonParser jp(js);
    c.config = jp.val();
    rd(&nt, 4);
    for (uint32_t k = 0; k < nt; ++k) {
        uint32_t nl;
        rd(&nl, 4);
        std::string name(nl, '\0');
        rd(&name[0], nl);
        uint32_t nd;
        rd(&nd, 4);
        CsmTensor t;
        t.shape.resize(nd);
        for (uint32_t d = 0; d < nd; ++d) rd(&t.shape[d], 8);
        uint32_t dt;
        rd(&dt, 4);
        t.dtype = (int)dt;
        int64_t n = t.numel();
        if (dt == 0) {
            t.f.resize(n);
            rd(t.f.data(), n * 4);
        } else if (dt == 1 || dt == 3) {
            std::vector<uint16_t> h(n);
            rd(h.data(), n * 2);
            t.f.resize(n);
            for (int64_t q = 0; q < n; ++q) t.f[q] = dt == 1 ? half_bits_to_float(h[q]) : bf16_bits_to_float(h[q]);
        } else if (dt == 2) {
            t.i.resize(n);
            rd(t.i.data(), n * 8);
        } else {
            throw std::runtime_error("ModelWeights: unknown dtype for tensor " + name);
        }
        c.t[name] = std::move(t);
    }
    return c;
}

// ---------------------------------------------------------------------------
// Mel band map.  The reference reads it precomputed from the .csm
// (src/model_mel_band_roformer.cu:79-150); the converter that writes it is not
// in the reference.  This restates the published MelBandRoformer construction
// (lucidrains BS-RoFormer `MelBandRoformer.__init__`): a slaney-scale mel
// filterbank as in librosa.filters.mel (htk=False, fmin=0, fmax=sr/2), a bin
// belongs to band i where the triangular weight is > 0, bin 0 is forced into
// band 0 and bin n_fft/2 into the last band; stereo interleaves 2f+s.
// Weight > 0 <=> mel_f[i] < fft_f[j] < mel_f[i+2] (strict), computed in fp64
// with numpy's operation order.
// ---------------------------------------------------------------------------
double hz_to_mel(double f) {
    const double f_sp = 200.0 / 3;
    double mels = (f - 0.0) / f_sp;
    const double min_log_hz = 1000.0;
    const double min_log_mel = (min_log_hz - 0.0) / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    if (f >= min_log_hz) mels = min_log_mel + std::log(f / min_log_hz) / logstep;
    return mels;
}
double mel_to_hz(double m) {
    const double f_sp = 200.0 / 3;
    double freqs = 0.0 + f_sp * m;
    const double min_log_hz = 1000.0;
    const double min_log_mel = (min_log_hz - 0.0) / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    if (m >= min_log_mel) freqs = min_log_hz * std::exp(logstep * (m - min_log_mel));
    return freqs;
}

void band_map(int sr, int n_fft, int nb, bool stereo, std::vector<int64_t>& fi, std::vector<int64_t>& nfpb,
              std::vector<int64_t>& nbpf) {
    int nf = n_fft / 2 + 1;
    std::vector<double> fft_f(nf);
    double val = 1.0 / ((double)n_fft * (1.0 / (double)sr));
    for (int j = 0; j < nf; ++j) fft_f[j] = (double)j * val;
    double mn = hz_to_mel(0.0), mx = hz_to_mel((double)sr / 2.0);
    int nm = nb + 2;
    std::vector<double> mel_f(nm);
    double step = (mx - mn) / (double)(nm - 1);
    for (int i = 0; i < nm; ++i) mel_f[i] = mel_to_hz((double)i * step + mn);
    mel_f[nm - 1] = mel_to_hz(mx);
    std::vector<uint8_t> in(nb * (size_t)nf, 0);
    for (int i = 0; i < nb; ++i)
        for (int j = 0; j < nf; ++j) {
            double lower = -(mel_f[i] - fft_f[j]) / (mel_f[i + 1] - mel_f[i]);
            double upper = (mel_f[i + 2] - fft_f[j]) / (mel_f[i + 2] - mel_f[i + 1]);
            double w = std::max(0.0, std::min(lower, upper));
            in[(size_t)i * nf + j] = w > 0.0;
        }
    in[0] = 1;
    in[(size_t)(nb - 1) * nf + (nf - 1)] = 1;
    fi.clear();
    nfpb.assign(nb, 0);
    nbpf.assign(nf, 0);
    for (int i = 0; i < nb; ++i)
        for (int j = 0; j < nf; ++j)
            if (in[(size_t)i * nf + j]) {
                nfpb[i]++;
                nbpf[j]++;
                if (stereo) {
                    fi.push_back(2 * j);
                    fi.push_back(2 * j + 1);
                } else {
                    fi.push_back(j);
                }
            }
    for (int j = 0; j < nf; ++j)
        if (nbpf[j] == 0) throw std::runtime_error("band map leaves a frequency bin uncovered");
}

// ---------------------------------------------------------------------------
// FFT (fp64 radix-2) and STFT / iSTFT.  Restates stft_tile::stft/istft
// (src/stft_cuda_tile.cu:530-715): reflect pad n_fft/2, periodic Hann
// (hann_window_kernel, :501-510), onesided forward transform; inverse uses the
// Hermitian mirror X[n] = conj(X[N-n]) (:254-345), x/N * w overlap-add (:426-449),
// division by sum w^2 where > 1e-8 (:462-499) and centre crop (:700-704).
// ---------------------------------------------------------------------------
struct Fft {
    int n = 0, lg = 0;
    std::vector<std::complex<double>> tw;
    std::vector<int> rev;
    explicit Fft(int N) : n(N) {
        while ((1 << lg) < n) ++lg;
        if ((1 << lg) != n) throw std::runtime_error("FFT size must be a power of two");
        tw.resize(n / 2);
        for (int k = 0; k < n / 2; ++k) tw[k] = std::polar(1.0, -2.0 * M_PI * (double)k / (double)n);
        rev.resize(n);
        for (int i = 0; i < n; ++i) {
            int r = 0;
            for (int b = 0; b < lg; ++b)
                if (i & (1 << b)) r |= 1 << (lg - 1 - b);
            rev[i] = r;
        }
    }
    // In-place; inverse=true uses e^{+i}, unnormalised.
    void run(std::complex<double>* x, bool inverse) const {
        for (int i = 0; i < n; ++i)
            if (i < rev[i]) std::swap(x[i], x[rev[i]]);
        for (int len = 2; len <= n; len <<= 1) {
            int half = len / 2, stride = n / len;
            for (int s = 0; s < n; s += len)
                for (int k = 0; k < half; ++k) {
                    std::complex<double> w = tw[k * stride];
                    if (inverse) w = std::conj(w);
                    std::complex<double> a = x[s + k], b = x[s + k + half] * w;
                    x[s + k] = a + b;
                    x[s + k + half] = a - b;
                }
        }
    }
};

std::vector<double> hann(int n) {
    std::vector<double> w(n);
    for (int i = 0; i < n; ++i) w[i] = 0.5 * (1.0 - std::cos(2.0 * M_PI * (double)i / (double)n));
    return w;
}

int64_t reflect_index(int64_t p, int64_t L) {
    // torch / Tensor::pad_reflect semantics (no edge repeat); valid for pad < L.
    while (p < 0 || p >= L) {
        if (p < 0) p = -p;
        if (p >= L) p = 2 * (L - 1) - p;
    }
    return p;
}

// sig [L] -> spec [F][T] (complex, fp64)
void stft_one(const float* sig, int64_t L, int n_fft, int hop, const Fft& fft, const std::vector<double>& win,
              std::vector<std::complex<double>>& spec, int64_t T) {
    int F = n_fft / 2 + 1;
    int pad = n_fft / 2;
    spec.assign((size_t)F * T, 0.0);
    std::vector<std::complex<double>> buf(n_fft);
    for (int64_t t = 0; t < T; ++t) {
        for (int n = 0; n < n_fft; ++n) {
            int64_t p = reflect_index(t * hop + n - pad, L);
            buf[n] = std::complex<double>((double)sig[p] * win[n], 0.0);
        }
        fft.run(buf.data(), false);
        for (int f = 0; f < F; ++f) spec[(size_t)f * T + t] = buf[f];
    }
}

// spec [F][T] -> out (signal_length - n_fft samples, centre cropped), then length rule.
std::vector<double> istft_one(const std::complex<double>* spec, int64_t T, int n_fft, int hop, const Fft& fft,
                              const std::vector<double>& win, int64_t length) {
    int F = n_fft / 2 + 1;
    int64_t sl = n_fft + (T - 1) * hop;
    std::vector<double> out(sl, 0.0), ws(sl, 0.0);
    std::vector<std::complex<double>> buf(n_fft);
    for (int64_t t = 0; t < T; ++t) {
        for (int n = 0; n < n_fft; ++n) {
            if (n < F) buf[n] = spec[(size_t)n * T + t];
            else buf[n] = std::conj(spec[(size_t)(n_fft - n) * T + t]);
        }
        fft.run(buf.data(), true);
        for (int n = 0; n < n_fft; ++n) {
            out[t * hop + n] += buf[n].real() / (double)n_fft * win[n];
            ws[t * hop + n] += win[n] * win[n];
        }
    }
    for (int64_t p = 0; p < sl; ++p)
        if (ws[p] > 1e-8) out[p] /= ws[p];
    int pad = n_fft / 2;
    std::vector<double> r(out.begin() + pad, out.end() - pad);
    if (length > 0) r.resize(length, 0.0);
    return r;
}

// ---------------------------------------------------------------------------
// Model
// ---------------------------------------------------------------------------
struct Cfg {
    // MBRConfig::from_json defaults (src/model_mel_band_roformer.cu:46-69)
    int dim = 384, depth = 6, stereo = 1, num_stems = 1, ttd = 1, ftd = 1, num_bands = 60, dim_head = 64,
        heads = 8, mask_depth = 2, mlp_mult = 4, zero_dc = 1, sr = 44100, n_fft = 2048, hop = 441,
        win = 2048, normalized = 0, match_len = 0, dim_freqs_in = 1025, skip = 0;
    int chunk_size = 0, num_overlap = 1;
};

struct Lin {
    int out = 0, in = 0;
    std::vector<float> w, b;  // w [out][in]
};
struct AttnW {
    std::vector<float> gamma;
    Lin qkv, gates, out;
};
struct FfW {
    std::vector<float> gamma;
    Lin l1, l2;
};
struct TransW {
    std::vector<AttnW> attn;
    std::vector<FfW> ff;
    std::vector<float> final_gamma;
};

struct Model {
    Cfg c;
    int C = 2;
    std::vector<int64_t> fi, nfpb, nbpf;  // nbpf expanded to C*F (stereo interleaved)
    std::vector<int> bd, boff;            // band feature dims (2*nf*C) and offsets
    std::vector<std::vector<float>> bs_gamma;
    std::vector<Lin> bs_lin;
    std::vector<TransW> tt, ft;
    std::vector<std::vector<std::vector<Lin>>> mask;  // [stem][band][linear]
    std::vector<double> win;
    // Reference-bf16 mode (weight_dtype 4): activations are rounded to bf16
    // where the reference's default --bf16 path stores them (see rb()).
    bool ref_bf16 = false;
};

// Round v to bf16 in the reference-bf16 mode, keep it otherwise.  With --bf16
// and no CUDASEP_* overrides the reference takes its custom bf16 path
// (custom_bf16_path_enabled, src/mbr_cuda_tile.cu:110-112), which turns on
// every bf16 storage switch (all_bf16_experiments_enabled /
// remaining_bf16_experiments_enabled, :120-140): bf16 outputs of the band
// gather (:326), RMSNorm (:147), linear layers (:182, :338), attention P.V
// (:186), sigmoid gates and the gate merge (:139, :143), the residual stream
// (:333; src/model_mel_band_roformer.cu:22-26), tanh and GLU inputs / outputs
// (:317-323) and the masks of the scatter (:305); bf16 norm gammas, biases and
// rotary tables (:337-354; src/model_mel_band_roformer.cu:28-38, :294-296).
inline float rb(const Model& m, double v) { return m.ref_bf16 ? round_bf16((float)v) : (float)v; }

Lin get_lin(const Csm& w, const std::string& p, bool bias, int round_mode) {
    Lin l;
    const CsmTensor& W = w.get(p + ".weight");
    if (W.shape.size() != 2) throw std::runtime_error("linear weight must be 2-D: " + p);
    l.out = (int)W.shape[0];
    l.in = (int)W.shape[1];
    l.w = W.f;
    if (W.dtype == 0 && round_mode == 1)
        for (auto& v : l.w) v = round_fp16(v);
    if (W.dtype == 0 && (round_mode == 3 || round_mode == 4))
        for (auto& v : l.w) v = round_bf16(v);
    if (bias) l.b = w.get(p + ".bias").f;
    if (round_mode == 4)  // bias_bf16_enabled (src/mbr_cuda_tile.cu:337-339)
        for (auto& v : l.b) v = round_bf16(v);
    return l;
}

// Restates MelBandRoformer::load (src/model_mel_band_roformer.cu:75-264).
Model load_model(const std::string& path, int round_mode) {
    Csm w = read_csm(path);
    Model m;
    Cfg& c = m.c;
    const Json& j = w.config;
    c.dim = jint(j, "dim", 384);
    c.depth = jint(j, "depth", 6);
    c.stereo = jbool(j, "stereo", true);
    c.num_stems = jint(j, "num_stems", 1);
    c.ttd = jint(j, "time_transformer_depth", 1);
    c.ftd = jint(j, "freq_transformer_depth", 1);
    c.num_bands = jint(j, "num_bands", 60);
    c.dim_head = jint(j, "dim_head", 64);
    c.heads = jint(j, "heads", 8);
    c.mask_depth = jint(j, "mask_estimator_depth", 2);
    c.mlp_mult = jint(j, "mlp_expansion_factor", 4);
    c.zero_dc = jbool(j, "zero_dc", true);
    c.sr = jint(j, "sample_rate", 44100);
    c.n_fft = jint(j, "stft_n_fft", 2048);
    c.hop = jint(j, "stft_hop_length", 441);
    c.win = jint(j, "stft_win_length", 2048);
    c.normalized = jbool(j, "stft_normalized", false);
    c.match_len = jbool(j, "match_input_audio_length", false);
    c.dim_freqs_in = jint(j, "dim_freqs_in", 1025);
    c.skip = jbool(j, "skip_connection", false);
    // src/inference_app.cpp:298-299 and :42-44
    c.chunk_size = jint(j, "chunk_size", c.n_fft * 256);
    c.num_overlap = std::max(1, jint(j, "num_overlap", 1));
    if (c.n_fft != 2048 || c.win != 2048)
        throw std::runtime_error("custom STFT only supports n_fft=2048, win_length=2048");
    m.C = c.stereo ? 2 : 1;
    int F = c.n_fft / 2 + 1;
    if (!w.has("__precomputed__.freq_indices"))
        throw std::runtime_error("MelBandRoformer .csm must include precomputed mel band data");
    m.fi = w.get("__precomputed__.freq_indices").i;
    m.nfpb = w.get("__precomputed__.num_freqs_per_band").i;
    std::vector<int64_t> nbpf = w.get("__precomputed__.num_bands_per_freq").i;
    m.nbpf.resize((size_t)F * m.C);
    for (int f = 0; f < F; ++f)
        for (int s = 0; s < m.C; ++s) m.nbpf[(size_t)f * m.C + s] = nbpf[f];
    for (int64_t v : m.fi)
        if (v < 0 || v >= (int64_t)F * m.C)
            throw std::runtime_error("MelBandRoformer: precomputed freq_indices out of range");
    int nb = c.num_bands;
    m.bd.resize(nb);
    m.boff.resize(nb + 1);
    m.boff[0] = 0;
    for (int b = 0; b < nb; ++b) {
        m.bd[b] = (int)(2 * m.nfpb[b] * m.C);
        m.boff[b + 1] = m.boff[b] + m.bd[b];
    }
    if ((int64_t)m.boff[nb] != 2 * (int64_t)m.fi.size())
        throw std::runtime_error("band dims do not match freq_indices");
    m.win = hann(c.win);
    for (int b = 0; b < nb; ++b) {
        std::string p = "band_split.to_features." + std::to_string(b);
        m.bs_gamma.push_back(w.get(p + ".0.gamma").f);
        m.bs_lin.push_back(get_lin(w, p + ".1", true, round_mode));
    }
    auto load_t = [&](const std::string& tp, int depth, TransW& tw) {
        tw.attn.resize(depth);
        tw.ff.resize(depth);
        for (int l = 0; l < depth; ++l) {
            std::string lp = tp + ".layers." + std::to_string(l);
            tw.attn[l].gamma = w.get(lp + ".0.norm.gamma").f;
            tw.attn[l].qkv = get_lin(w, lp + ".0.to_qkv", false, round_mode);
            tw.attn[l].gates = get_lin(w, lp + ".0.to_gates", true, round_mode);
            tw.attn[l].out = get_lin(w, lp + ".0.to_out.0", false, round_mode);
            tw.ff[l].gamma = w.get(lp + ".1.net.0.gamma").f;
            tw.ff[l].l1 = get_lin(w, lp + ".1.net.1", true, round_mode);
            tw.ff[l].l2 = get_lin(w, lp + ".1.net.4", true, round_mode);
        }
        tw.final_gamma = w.get(tp + ".norm.gamma").f;
    };
    m.tt.resize(c.depth);
    m.ft.resize(c.depth);
    for (int d = 0; d < c.depth; ++d) {
        std::string dp = "layers." + std::to_string(d);
        load_t(dp + ".0", c.ttd, m.tt[d]);
        load_t(dp + ".1", c.ftd, m.ft[d]);
    }
    m.mask.resize(c.num_stems);
    for (int s = 0; s < c.num_stems; ++s) {
        m.mask[s].resize(nb);
        for (int b = 0; b < nb; ++b)
            for (int i = 0; i < c.mask_depth + 1; ++i)
                m.mask[s][b].push_back(get_lin(w,
                                               "mask_estimators." + std::to_string(s) + ".to_freqs." +
                                                   std::to_string(b) + ".0." + std::to_string(2 * i),
                                               true, round_mode));
    }
    if (round_mode == 4) {
        // norm_gamma_bf16_enabled (src/mbr_cuda_tile.cu:341-344)
        m.ref_bf16 = true;
        auto rg = [](std::vector<float>& g) {
            for (auto& v : g) v = round_bf16(v);
        };
        for (auto& g : m.bs_gamma) rg(g);
        for (auto* tws : {&m.tt, &m.ft})
            for (auto& tw : *tws) {
                for (auto& a : tw.attn) rg(a.gamma);
                for (auto& f : tw.ff) rg(f.gamma);
                rg(tw.final_gamma);
            }
    }
    return m;
}

// Y[m][n] = act(sum_k X[m*ldx + k] * W[n][k] + b[n]), fp64 accumulation.
enum Act { A_NONE, A_GELU, A_TANH };
inline double dot(const float* a, const float* b, int64_t K) {
    double acc = 0.0;
#pragma omp simd reduction(+ : acc)
    for (int64_t k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
    return acc;
}
// GELU of the reference's bf16 FFN: erf from an odd degree-17 polynomial in
// |x| evaluated in fp32 and clamped to [0, 1] (gelu_erf_poly9_l30_fast,
// src/mbr_ffn12_cutile.cu:53-66; coefficients as published there).
inline double gelu_poly9(double xd) {
    float x = (float)xd, ax = std::fabs(x), z = ax * ax;
    float p = ((((((((0.00000005422539767f * z - 0.000002440964777f) * z + 0.00004855766724f) * z -
                   0.0005709642654f) * z + 0.004507274577f) * z - 0.02579950512f) * z + 0.1120213868f) * z -
               0.3758834075f) * z + 1.128367753f);
    float e = std::min(std::max(ax * p, 0.0f), 1.0f);
    if (x < 0.0f) e = -e;
    return (double)(0.5f * x * (1.0f + e));
}
// GELU as the reference computes it in every precision: 0.5 v (1 + erf(v)).
// Its erf-based GELU kernels take erf of the value itself, not of v / sqrt 2
// (add_bias_gelu_kernel, src/mbr_cuda_tile.cu:5536-5558, the fp32 path;
// gelu_erf_approx, :565-583; gelu_erf_poly9_l30, src/mbr_ffn12_cutile.cu:33-66),
// which is v * Phi(sqrt(2) v), not torch's nn.GELU.  The oracle follows the
// reference.
inline double act_apply(double v, Act a) {
    if (a == A_GELU) return 0.5 * v * (1.0 + std::erf(v));
    if (a == A_TANH) return std::tanh(v);
    return v;
}
// Output rounding of one linear in the reference-bf16 mode:
//  RB_OUT: bf16(act(acc + b)) — the bf16-output linears (src/mbr_cuda_tile.cu:6880-6885)
//  RB_ACC: bf16(act(bf16(acc) + b)) — the FFN GEMMs round the accumulator before the
//          bias (src/mbr_ffn12_cutile.cu:325-330, :366-371), GELU = gelu_poly9
//  RB_TANH: bf16(tanh(bf16(acc + b))) — tanh with a bf16 input (src/mbr_cuda_tile.cu:3501-3548)
// A residual linear (accumulate) then stores bf16(y + out).
enum Rb { RB_OUT, RB_ACC, RB_TANH };
void linear(const float* X, int64_t M, int64_t ldx, const Lin& L, float* Y, int64_t ldy, Act act, bool accumulate,
            const Model* rbm = nullptr, Rb rbk = RB_OUT) {
    if (rbm && !rbm->ref_bf16) rbm = nullptr;
    const int64_t MB = 8;
    int64_t nblk = (M + MB - 1) / MB;
    parallel_for(nblk, [&](int64_t blk) {
        int64_t m0 = blk * MB, m1 = std::min(M, m0 + MB);
        for (int n0 = 0; n0 < L.out; n0 += 64) {
            int n1 = std::min(L.out, n0 + 64);
            for (int64_t m = m0; m < m1; ++m)
                for (int n = n0; n < n1; ++n) {
                    double v = dot(X + m * ldx, L.w.data() + (size_t)n * L.in, L.in);
                    float* y = Y + m * ldy + n;
                    if (rbm) {
                        double bias = L.b.empty() ? 0.0 : (double)L.b[n];
                        double o;
                        if (rbk == RB_ACC) {
                            o = (double)round_bf16((float)v) + bias;
                            o = act == A_GELU ? gelu_poly9(o) : act_apply(o, act);
                        } else if (rbk == RB_TANH) {
                            o = std::tanh((double)round_bf16((float)(v + bias)));
                        } else {
                            o = act_apply(v + bias, act);
                        }
                        float ob = round_bf16((float)o);
                        *y = accumulate ? round_bf16((float)((double)*y + ob)) : ob;
                        continue;
                    }
                    if (!L.b.empty()) v += (double)L.b[n];
                    v = act_apply(v, act);
                    *y = accumulate ? (float)((double)*y + v) : (float)v;
                }
        }
    });
}

// rms_norm (src/mbr_cuda_tile.cu:4791-4813): x * rsqrt(sum x^2 + 1e-12) * gamma * scale
void rms_norm(const float* X, int64_t M, int D, int64_t ldx, const std::vector<float>& g, float scale, float* Y,
              int64_t ldy, const Model* rbm = nullptr) {
    const bool r16 = rbm && rbm->ref_bf16;
    parallel_for((M + 63) / 64, [&](int64_t blk) {
        for (int64_t m = blk * 64; m < std::min(M, blk * 64 + 64); ++m) {
            const float* x = X + m * ldx;
            double ss = 0;
            for (int d = 0; d < D; ++d) ss += (double)x[d] * x[d];
            double inv = 1.0 / std::sqrt(ss + 1e-12);
            float* y = Y + m * ldy;
            for (int d = 0; d < D; ++d) {
                double v = (double)x[d] * inv * (double)g[d] * (double)scale;
                y[d] = r16 ? round_bf16((float)v) : (float)v;
            }
        }
    });
}

// Rotary tables exactly as compute_rotary_cos_sin (src/model_mel_band_roformer.cu:270-300),
// fp32 host arithmetic.
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

// One transformer (apply_transformer, src/model_mel_band_roformer.cu:447-566) over
// sequences; token(s, p) gives the token row of position p of sequence s.
// R [tokens][D] is updated in place and ends RMS-normed by the final gamma.
void transformer(const Model& m, const TransW& tw, float* R, int64_t ntok, int64_t nseq, int64_t L,
                 const std::function<int64_t(int64_t, int64_t)>& token) {
    const Cfg& c = m.c;
    int D = c.dim, H = c.heads, dh = c.dim_head, DI = H * dh;
    float scale = std::sqrt((float)D);
    float attn_scale = 1.0f / std::sqrt((float)dh);
    std::vector<float> cs, sn;
    rotary_tables((int)L, dh, cs, sn);
    if (m.ref_bf16) {  // rotary_freqs_bf16 (src/model_mel_band_roformer.cu:294-296)
        for (auto& v : cs) v = round_bf16(v);
        for (auto& v : sn) v = round_bf16(v);
    }
    std::vector<float> xn((size_t)ntok * D), qkv((size_t)ntok * 3 * DI), gates((size_t)ntok * H),
        merged((size_t)ntok * DI), hid;
    for (size_t l = 0; l < tw.attn.size(); ++l) {
        const AttnW& a = tw.attn[l];
        rms_norm(R, ntok, D, D, a.gamma, scale, xn.data(), D, &m);
        linear(xn.data(), ntok, D, a.qkv, qkv.data(), 3 * DI, A_NONE, false);  // rounded after RoPE
        // gates = sigmoid(linear(normed)) (src/model_mel_band_roformer.cu:394-398)
        linear(xn.data(), ntok, D, a.gates, gates.data(), H, A_NONE, false);
        for (auto& g : gates) g = rb(m, 1.0 / (1.0 + std::exp(-(double)g)));
        parallel_for(nseq * H, [&](int64_t sh) {
            int64_t s = sh / H;
            int h = (int)(sh % H);
            int half = dh / 2;
            std::vector<double> q((size_t)L * dh), k((size_t)L * dh), v((size_t)L * dh), p(L);
            for (int64_t pos = 0; pos < L; ++pos) {
                const float* row = qkv.data() + token(s, pos) * 3 * DI;
                for (int i = 0; i < half; ++i) {
                    // interleaved-pair rotary (src/mbr_cuda_tile.cu:3928-3943)
                    double cc = cs[(size_t)pos * half + i], ss = sn[(size_t)pos * half + i];
                    double q0 = row[h * dh + 2 * i], q1 = row[h * dh + 2 * i + 1];
                    double k0 = row[DI + h * dh + 2 * i], k1 = row[DI + h * dh + 2 * i + 1];
                    q[pos * dh + 2 * i] = rb(m, q0 * cc - q1 * ss);
                    q[pos * dh + 2 * i + 1] = rb(m, q0 * ss + q1 * cc);
                    k[pos * dh + 2 * i] = rb(m, k0 * cc - k1 * ss);
                    k[pos * dh + 2 * i + 1] = rb(m, k0 * ss + k1 * cc);
                    v[pos * dh + 2 * i] = rb(m, row[2 * DI + h * dh + 2 * i]);
                    v[pos * dh + 2 * i + 1] = rb(m, row[2 * DI + h * dh + 2 * i + 1]);
                }
            }
            for (int64_t i = 0; i < L; ++i) {
                double mx = -1e300;
                for (int64_t jj = 0; jj < L; ++jj) {
                    double sc = 0;
                    for (int d = 0; d < dh; ++d) sc += q[i * dh + d] * k[jj * dh + d];
                    sc *= (double)attn_scale;
                    p[jj] = sc;
                    mx = std::max(mx, sc);
                }
                double sum = 0;
                for (int64_t jj = 0; jj < L; ++jj) {
                    p[jj] = std::exp(p[jj] - mx);
                    sum += p[jj];
                    // P.V takes bf16 probabilities; the row sum uses fp32 ones
                    // (src/mbr_time_attention_cutile.cu:255-261)
                    if (m.ref_bf16) p[jj] = round_bf16((float)p[jj]);
                }
                int64_t tok = token(s, i);
                double g = gates[(size_t)tok * H + h];
                for (int d = 0; d < dh; ++d) {
                    double o = 0;
                    for (int64_t jj = 0; jj < L; ++jj) o += p[jj] * v[jj * dh + d];
                    // apply_gates_and_merge_heads (src/mbr_cuda_tile.cu:4603-4628)
                    merged[(size_t)tok * DI + h * dh + d] = rb(m, (double)rb(m, o / sum) * g);
                }
            }
        });
        linear(merged.data(), ntok, DI, a.out, R, D, A_NONE, true, &m);  // residual add
        const FfW& f = tw.ff[l];
        rms_norm(R, ntok, D, D, f.gamma, scale, xn.data(), D, &m);
        hid.resize((size_t)ntok * f.l1.out);
        linear(xn.data(), ntok, D, f.l1, hid.data(), f.l1.out, A_GELU, false, &m, RB_ACC);
        linear(hid.data(), ntok, f.l1.out, f.l2, R, D, A_NONE, true, &m, RB_ACC);
    }
    rms_norm(R, ntok, D, D, tw.final_gamma, scale, R, D, &m);
}

struct FwdOut {
    std::vector<float> audio;  // [B][S][C][Lout]
    int64_t lout = 0;
    std::vector<float> taps[5];
    std::vector<int64_t> tap_shape[5];
};

// MelBandRoformer::forward (src/model_mel_band_roformer.cu:682-845).
FwdOut forward(const Model& m, const float* audio, int B, int64_t L, int want_tap) {
    const Cfg& c = m.c;
    int C = m.C, F = c.n_fft / 2 + 1, NB = c.num_bands, D = c.dim, S = c.num_stems;
    int64_t J = (int64_t)m.fi.size();
    int pad = c.n_fft / 2;
    if (L <= pad) throw std::runtime_error("input shorter than the reflect padding");
    int64_t T = (L + 2 * pad - c.n_fft) / c.hop + 1;
    Fft fft(c.n_fft);
    // spec[b][t][f*C + ch] complex (time-major; "b s f t c -> b (f s) t c")
    std::vector<std::complex<double>> spec((size_t)B * T * F * C);
    parallel_for((int64_t)B * C, [&](int64_t bc) {
        int64_t b = bc / C, ch = bc % C;
        std::vector<std::complex<double>> sp;
        stft_one(audio + (size_t)bc * L, L, c.n_fft, c.hop, fft, m.win, sp, T);
        double nrm = c.normalized ? 1.0 / std::sqrt((double)c.n_fft) : 1.0;
        for (int f = 0; f < F; ++f)
            for (int64_t t = 0; t < T; ++t) {
                // the GPU path stores the spectrum as fp32; round the same way
                std::complex<double> v = sp[(size_t)f * T + t] * nrm;
                spec[((size_t)(b * T + t) * F + f) * C + ch] = {(double)(float)v.real(), (double)(float)v.imag()};
            }
    });
    int64_t MT = (int64_t)B * T;
    // gather_freqs_fold_complex (src/mbr_cuda_tile.cu:4554-4576) + apply_band_split (:572-604)
    std::vector<float> R((size_t)MT * NB * D);
    {
        std::vector<float> xg((size_t)MT * 2 * J);
        parallel_for(MT, [&](int64_t mt) {
            const std::complex<double>* row = spec.data() + (size_t)mt * F * C;
            float* o = xg.data() + (size_t)mt * 2 * J;
            for (int64_t jj = 0; jj < J; ++jj) {
                o[2 * jj] = rb(m, row[m.fi[jj]].real());
                o[2 * jj + 1] = rb(m, row[m.fi[jj]].imag());
            }
        });
        std::vector<float> nrm;
        for (int b = 0; b < NB; ++b) {
            nrm.resize((size_t)MT * m.bd[b]);
            rms_norm(xg.data() + m.boff[b], MT, m.bd[b], 2 * J, m.bs_gamma[b], std::sqrt((float)m.bd[b]), nrm.data(),
                     m.bd[b], &m);
            linear(nrm.data(), MT, m.bd[b], m.bs_lin[b], R.data() + (size_t)b * D, (int64_t)NB * D, A_NONE, false,
                   &m);
        }
    }
    FwdOut out;
    auto tap = [&](int id, const std::vector<float>& v, std::vector<int64_t> shp) {
        if (want_tap == id) {
            out.taps[id] = v;
            out.tap_shape[id] = shp;
        }
    };
    tap(0, R, {B, T, NB, D});
    std::vector<std::vector<float>> skip;
    int64_t ntok = MT * NB;
    for (int d = 0; d < c.depth; ++d) {
        if (c.skip)
            for (int jj = 0; jj < d; ++jj)
                for (size_t q = 0; q < R.size(); ++q) R[q] += skip[jj][q];
        transformer(m, m.tt[d], R.data(), ntok, (int64_t)B * NB, T,
                    [&](int64_t s, int64_t p) { return ((s / NB) * T + p) * NB + (s % NB); });
        transformer(m, m.ft[d], R.data(), ntok, MT, NB, [&](int64_t s, int64_t p) { return s * NB + p; });
        if (c.skip) skip.push_back(R);
        if (d == 0) tap(1, R, {B, T, NB, D});
    }
    tap(2, R, {B, T, NB, D});
    // apply_mask_estimator (src/model_mel_band_roformer.cu:610-676): per band MLP with tanh, GLU
    std::vector<float> masks((size_t)S * MT * 2 * J);
    for (int s = 0; s < S; ++s) {
        for (int b = 0; b < NB; ++b) {
            const auto& mlp = m.mask[s][b];
            std::vector<float> h, h2;
            const float* in = R.data() + (size_t)b * D;
            int64_t ld = (int64_t)NB * D;
            for (size_t i = 0; i < mlp.size(); ++i) {
                h2.resize((size_t)MT * mlp[i].out);
                bool last = i + 1 == mlp.size();
                linear(in, MT, ld, mlp[i], h2.data(), mlp[i].out, last ? A_NONE : A_TANH, false, &m,
                       last ? RB_OUT : RB_TANH);
                h.swap(h2);
                in = h.data();
                ld = mlp[i].out;
            }
            int bd = m.bd[b];
            for (int64_t mt = 0; mt < MT; ++mt)
                for (int q = 0; q < bd; ++q) {
                    double a = h[(size_t)mt * 2 * bd + q], g = h[(size_t)mt * 2 * bd + bd + q];
                    masks[((size_t)s * MT + mt) * 2 * J + m.boff[b] + q] = rb(m, a / (1.0 + std::exp(-g)));
                }
        }
    }
    if (want_tap == 3) tap(3, std::vector<float>(masks.begin(), masks.begin() + (size_t)MT * 2 * J), {B, T, 2 * J});
    // apply_mask_and_scatter (src/mbr_cuda_tile.cu:5587-5649) + zero_dc (:5805-5820)
    // out spectrum [B][S][C][F][T] complex
    std::vector<std::complex<double>> os((size_t)B * S * C * F * T, 0.0);
    parallel_for((int64_t)B * S, [&](int64_t bs) {
        int64_t b = bs / S, s = bs % S;
        for (int64_t t = 0; t < T; ++t) {
            const float* mk = masks.data() + ((size_t)s * MT + b * T + t) * 2 * J;
            for (int64_t jj = 0; jj < J; ++jj) {
                int64_t fs = m.fi[jj];
                std::complex<double> x = spec[((size_t)(b * T + t) * F * C) + fs];
                std::complex<double> mm((double)mk[2 * jj], (double)mk[2 * jj + 1]);
                double den = std::max((double)m.nbpf[fs], 1e-8);
                int64_t f = fs / C, ch = fs % C;
                os[((((size_t)b * S + s) * C + ch) * F + f) * T + t] += x * mm / den;
            }
        }
    });
    if (c.zero_dc)
        for (int64_t o = 0; o < (int64_t)B * S * C; ++o)
            for (int64_t t = 0; t < T; ++t) os[(size_t)o * F * T + t] = 0.0;
    if (want_tap == 4) {
        std::vector<float> v(os.size() * 2);
        for (size_t q = 0; q < os.size(); ++q) {
            v[2 * q] = (float)os[q].real();
            v[2 * q + 1] = (float)os[q].imag();
        }
        tap(4, v, {(int64_t)B * S * C, F, T, 2});
    }
    int64_t length = c.match_len ? L : -1;
    int64_t lout = length > 0 ? length : (T - 1) * c.hop;
    out.lout = lout;
    out.audio.assign((size_t)B * S * C * lout, 0.f);
    double spec_scale = c.normalized ? std::sqrt((double)c.n_fft) : 1.0;
    parallel_for((int64_t)B * S * C, [&](int64_t o) {
        std::vector<std::complex<double>> sp(os.begin() + (size_t)o * F * T, os.begin() + (size_t)(o + 1) * F * T);
        for (auto& v : sp) v *= spec_scale;
        std::vector<double> r = istft_one(sp.data(), T, c.n_fft, c.hop, fft, m.win, length);
        for (int64_t q = 0; q < lout; ++q) out.audio[(size_t)o * lout + q] = (float)r[q];
    });
    return out;
}

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

// process_chunked (src/inference_app.cpp:72-232) + run_inference's single-chunk
// branch (:330-344).  track [C][N] -> out [S][C][N].
void separate(const Model& m, const float* track, int64_t N, float overlap, int chunk_batch, float* out) {
    const Cfg& c = m.c;
    int C = m.C, S = c.num_stems;
    int chunk = c.chunk_size;
    if (!(chunk > 0 && N > chunk)) {
        FwdOut r = forward(m, track, 1, N, -1);
        for (int64_t o = 0; o < (int64_t)S * C; ++o)
            for (int64_t q = 0; q < N; ++q)
                out[(size_t)o * N + q] = q < r.lout ? r.audio[(size_t)o * r.lout + q] : 0.f;
        return;
    }
    int step = resolve_step(chunk, overlap, c.num_overlap);
    int fade = chunk / 10;
    int64_t border = chunk - step;
    bool padded = N > 2 * border && border > 0;
    int64_t total = padded ? N + 2 * border : N;
    std::vector<float> mix((size_t)C * total);
    for (int ch = 0; ch < C; ++ch)
        for (int64_t q = 0; q < total; ++q)
            mix[(size_t)ch * total + q] = track[(size_t)ch * N + (padded ? reflect_index(q - border, N) : q)];
    std::vector<int64_t> starts;
    for (int64_t s0 = 0; s0 < total; s0 += step) starts.push_back(s0);
    std::vector<float> fw(chunk, 1.0f);
    if (fade > 0) {
        if (fade == 1) {
            fw.front() = 0.f;
            fw.back() = 0.f;
        } else {
            for (int i = 0; i < fade; ++i) {
                float alpha = (float)i / (float)(fade - 1);
                fw[i] = alpha;
                fw[chunk - fade + i] = 1.0f - alpha;
            }
        }
    }
    std::vector<double> acc((size_t)S * C * total, 0.0);
    std::vector<float> accf((size_t)S * C * total, 0.f), wsum(total, 0.f);
    (void)chunk_batch;  // chunk batching groups forwards but does not change the results
    std::vector<float> in((size_t)C * chunk);
    for (size_t ci = 0; ci < starts.size(); ++ci) {
        int64_t st = starts[ci], en = std::min<int64_t>(st + chunk, total), al = en - st;
        bool last = en >= total;
        for (int ch = 0; ch < C; ++ch)
            for (int64_t q = 0; q < chunk; ++q) {
                float v;
                if (q < al) v = mix[(size_t)ch * total + st + q];
                else if (al > chunk / 2) v = mix[(size_t)ch * total + st + reflect_index(q, al)];
                else v = 0.f;
                in[(size_t)ch * chunk + q] = v;
            }
        FwdOut r = forward(m, in.data(), 1, chunk, -1);
        if (r.lout < al) throw std::runtime_error("model output shorter than the chunk");
        std::vector<float> w = fw;
        if (fade > 0 && (st == 0 || last)) {
            if (st == 0) std::fill(w.begin(), w.begin() + fade, 1.0f);
            if (last) std::fill(w.end() - fade, w.end(), 1.0f);
        }
        // accumulate_chunk (src/chunk_cuda_tile.cu:18-42): fp32 adds in chunk order
        for (int64_t o = 0; o < (int64_t)S * C; ++o)
            for (int64_t q = 0; q < al; ++q) accf[(size_t)o * total + st + q] += r.audio[(size_t)o * r.lout + q] * w[q];
        for (int64_t q = 0; q < al; ++q) wsum[st + q] += w[q];
    }
    // normalize_by_weights (src/chunk_cuda_tile.cu:44-58) + crop (src/inference_app.cpp:225-229)
    for (int64_t o = 0; o < (int64_t)S * C; ++o)
        for (int64_t q = 0; q < N; ++q) {
            int64_t p = padded ? q + border : q;
            float wv = wsum[p], v = accf[(size_t)o * total + p];
            out[(size_t)o * N + q] = wv > 1e-8f ? v / wv : v;
        }
}

template <class F>
int guard(F&& f) {
    try {
        g_err.clear();
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

}  // namespace

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }
void orc_set_threads(int n) { g_threads = n; }
int orc_get_threads(void) { return nthreads(); }

int orc_band_map(int sr, int n_fft, int nb, int stereo, int64_t* fi, int64_t cap, int64_t* n_out, int64_t* nfpb,
                 int64_t* nbpf) {
    return guard([&] {
        std::vector<int64_t> a, b, c;
        band_map(sr, n_fft, nb, stereo != 0, a, b, c);
        *n_out = (int64_t)a.size();
        if ((int64_t)a.size() > cap) throw std::runtime_error("freq_indices capacity too small");
        std::copy(a.begin(), a.end(), fi);
        std::copy(b.begin(), b.end(), nfpb);
        std::copy(c.begin(), c.end(), nbpf);
    });
}

int orc_stft(const float* sig, int64_t n_sig, int64_t L, int n_fft, int hop, float* out, int64_t* T_out) {
    return guard([&] {
        int pad = n_fft / 2;
        if (L <= pad) throw std::runtime_error("signal shorter than reflect padding");
        int64_t T = (L + 2 * pad - n_fft) / hop + 1;
        *T_out = T;
        if (!out) return;
        Fft fft(n_fft);
        std::vector<double> win = hann(n_fft);
        int F = n_fft / 2 + 1;
        parallel_for(n_sig, [&](int64_t i) {
            std::vector<std::complex<double>> sp;
            stft_one(sig + i * L, L, n_fft, hop, fft, win, sp, T);
            for (size_t q = 0; q < (size_t)F * T; ++q) {
                out[((size_t)i * F * T + q) * 2] = (float)sp[q].real();
                out[((size_t)i * F * T + q) * 2 + 1] = (float)sp[q].imag();
            }
        });
    });
}

int orc_istft(const float* spec, int64_t n_sig, int64_t T, int n_fft, int hop, int64_t length, float* out,
              int64_t* len_out) {
    return guard([&] {
        int64_t lo = length > 0 ? length : (T - 1) * hop;
        *len_out = lo;
        if (!out) return;
        Fft fft(n_fft);
        std::vector<double> win = hann(n_fft);
        int F = n_fft / 2 + 1;
        parallel_for(n_sig, [&](int64_t i) {
            std::vector<std::complex<double>> sp((size_t)F * T);
            for (size_t q = 0; q < sp.size(); ++q)
                sp[q] = {spec[((size_t)i * F * T + q) * 2], spec[((size_t)i * F * T + q) * 2 + 1]};
            std::vector<double> r = istft_one(sp.data(), T, n_fft, hop, fft, win, length);
            for (int64_t q = 0; q < lo; ++q) out[(size_t)i * lo + q] = (float)r[q];
        });
    });
}

// softmax(q k^T * scale) v per slice, as the transformer's attention above
// computes it (src/mbr_cuda_tile.cu:6419-6462 is the reference's op).
int orc_attention(const float* q, const float* k, const float* v, int64_t nsh, int64_t L, int dh, float scale,
                  float* out) {
    return guard([&] {
        if (nsh <= 0 || L <= 0 || dh <= 0) throw std::runtime_error("orc_attention: bad shape");
        parallel_for(nsh * L, [&](int64_t si) {
            const int64_t s = si / L, i = si % L;
            const float* qi = q + (s * L + i) * dh;
            std::vector<double> p(L);
            double mx = -1e300;
            for (int64_t j = 0; j < L; ++j) {
                const float* kj = k + (s * L + j) * dh;
                double sc = 0;
                for (int d = 0; d < dh; ++d) sc += (double)qi[d] * kj[d];
                p[j] = sc * (double)scale;
                mx = std::max(mx, p[j]);
            }
            double sum = 0;
            for (int64_t j = 0; j < L; ++j) sum += (p[j] = std::exp(p[j] - mx));
            for (int d = 0; d < dh; ++d) {
                double o = 0;
                for (int64_t j = 0; j < L; ++j) o += p[j] * v[(s * L + j) * dh + d];
                out[(s * L + i) * dh + d] = (float)(o / sum);
            }
        });
    });
}

void* orc_model_load(const char* path, int weight_dtype) {
    Model* m = nullptr;
    int rc = guard([&] { m = new Model(load_model(path, weight_dtype)); });
    return rc == 0 ? m : nullptr;
}
void orc_model_free(void* m) { delete (Model*)m; }

int64_t orc_model_info(void* mp, int what) {
    const Model& m = *(Model*)mp;
    const Cfg& c = m.c;
    switch (what) {
        case 0: return c.dim;
        case 1: return c.depth;
        case 2: return c.num_stems;
        case 3: return m.C;
        case 4: return c.num_bands;
        case 5: return c.sr;
        case 6: return c.chunk_size;
        case 7: return c.num_overlap;
        case 8: return c.n_fft;
        case 9: return c.hop;
        case 10: return c.heads;
        case 11: return c.dim_head;
        case 12: return (int64_t)m.fi.size();
        case 13: return c.zero_dc;
        case 14: return c.match_len;
    }
    return -1;
}

int orc_forward(void* mp, const float* audio, int B, int64_t L, float* out, int64_t* lout) {
    return guard([&] {
        FwdOut r = forward(*(Model*)mp, audio, B, L, -1);
        *lout = r.lout;
        std::copy(r.audio.begin(), r.audio.end(), out);
    });
}

int orc_forward_tap(void* mp, const float* audio, int B, int64_t L, int tap, float* buf, int64_t* n) {
    return guard([&] {
        if (tap < 0 || tap > 4) throw std::runtime_error("bad tap");
        FwdOut r = forward(*(Model*)mp, audio, B, L, tap);
        *n = (int64_t)r.taps[tap].size();
        if (buf) std::copy(r.taps[tap].begin(), r.taps[tap].end(), buf);
    });
}

int orc_separate(void* mp, const float* track, int64_t N, float overlap, int chunk_batch, float* out) {
    return guard([&] { separate(*(Model*)mp, track, N, overlap, chunk_batch, out); });
}

int64_t orc_chunk_plan(int64_t N, int chunk, float overlap, int def, int64_t* starts, int64_t cap, int64_t* step,
                       int64_t* border, int64_t* total) {
    int st = resolve_step(chunk, overlap, def);
    int64_t bd = chunk - st;
    bool padded = N > 2 * bd && bd > 0;
    int64_t tot = padded ? N + 2 * bd : N;
    *step = st;
    *border = padded ? bd : 0;
    *total = tot;
    int64_t n = 0;
    for (int64_t s0 = 0; s0 < tot; s0 += st) {
        if (n < cap && starts) starts[n] = s0;
        ++n;
    }
    return n;
}

}  // extern "C"
