// model.h — MelBandRoformer forward on one B200 (host orchestration).
//
// Mirrors the reference class of src/model_mel_band_roformer.h:11-141
// (MBRConfig::from_json, MelBandRoformer::load/forward/config).  The forward is
// a fixed sequence of kernel launches on one stream over a workspace that is
// allocated once per input shape; weights are uploaded once, converted to the
// compute dtype and packed for the kernels (band-split weights as one
// block-diagonal matrix, per-band mask-estimator weights stacked per layer).
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "ops_api.h"
#include "ffn_tc.h"
#include "gemm_tc.h"
#include "ops.h"
#include "weights.h"

namespace mbr {

struct MBRConfig {
    int dim = 384;
    int depth = 6;
    bool stereo = true;
    int num_stems = 1;
    int time_transformer_depth = 1;
    int freq_transformer_depth = 1;
    int num_bands = 60;
    int dim_head = 64;
    int heads = 8;
    int mask_estimator_depth = 2;
    int mlp_expansion_factor = 4;
    bool zero_dc = true;
    int sample_rate = 44100;
    int stft_n_fft = 2048;
    int stft_hop_length = 441;
    int stft_win_length = 2048;
    bool stft_normalized = false;
    bool match_input_audio_length = false;
    int dim_freqs_in = 1025;
    bool skip_connection = false;
    // app-level keys (src/inference_app.cpp:42-44, :298)
    int chunk_size = 0;
    int num_overlap = 1;
    std::vector<std::string> instruments;
    static MBRConfig from_json(const JsonValue& j);
};

// Rotary cos/sin tables [n][dim/2] exactly as compute_rotary_cos_sin
// (src/model_mel_band_roformer.cu:270-300): fp32 host arithmetic.
void rotary_tables(int n, int dim, std::vector<float>& cs, std::vector<float>& sn);

// Kernel backends selectable per model (the tensor-core path is the default for
// fp16/bf16; the CUDA-core path is the fp32 path and a cross-check).
// BACKEND_TC_DIRECT: tensor-core GEMMs whose epilogues store from registers
// instead of staging through shared memory for TMA stores (A/B comparisons).
enum Backend { BACKEND_SIMT = 0, BACKEND_TC = 1, BACKEND_TC_DIRECT = 2 };

// Kernel classes timed by the optional per-launch profiler (CUDA events on the
// launching stream).
enum ProfKind {
    PK_STFT = 0,
    PK_BAND_GATHER,
    PK_GEMM_BANDSPLIT,
    PK_NORM,
    PK_GEMM_QKV,
    PK_ROPE,
    PK_ATTN_TIME,
    PK_ATTN_FREQ,
    PK_GEMM_OUT,
    PK_GEMM_FFN1,
    PK_GEMM_FFN2,
    PK_GEMM_MASK_HIDDEN,
    PK_GEMM_MASK_OUT,
    PK_MASK_SCATTER,
    PK_ISTFT,
    PK_FFN,  // fused FFN1 + GELU + FFN2 (+ residual)
    PK_COUNT
};

class MelBandRoformer {
public:
    // Loads and uploads the weights to `device`; dtype DT_F32 / DT_F16 / DT_BF16.
    MelBandRoformer(const ModelWeights& w, int device, int dtype);
    ~MelBandRoformer();
    MelBandRoformer(const MelBandRoformer&) = delete;
    MelBandRoformer& operator=(const MelBandRoformer&) = delete;

    const MBRConfig& config() const { return cfg_; }
    int device() const { return device_; }
    int dtype() const { return dtype_; }
    int channels() const { return C_; }
    int64_t band_freqs() const { return J_; }
    // device band maps (for the stand-alone band ops)
    const int* d_freq_indices() const { return d_fi_; }
    const int* d_rev_off() const { return d_rev_off_; }
    const int* d_rev_idx() const { return d_rev_idx_; }
    const float* d_bands_per_freq() const { return d_nbpf_; }
    // Frequency-range tiles of the band map for the stand-alone band ops.
    const opsapi::BandTiles& band_tiles() const { return band_tiles_; }
    int64_t frames(int64_t L) const;      // STFT frames T of an L-sample input
    int64_t out_length(int64_t L) const;  // output samples of an L-sample input

    // audio [B][C][L] (device, fp32) -> out [B][S][C][out_length(L)] (device, fp32).
    void forward(const float* d_audio, int B, int64_t L, float* d_out, cudaStream_t st);

    // Per-stage taps for parity tests (same numbering as the oracle):
    //  0 band-split output, 1 after depth block 0, 2 final residual stream,
    //  3 stem-0 mask, 4 masked spectrum.  Copies into d_tap (fp32) and
    //  returns the element count (d_tap == nullptr only sizes).
    int64_t forward_tap(const float* d_audio, int B, int64_t L, int tap, float* d_tap, cudaStream_t st);

    void set_backend(int gemm, int attention) {
        gemm_backend_ = gemm;
        attn_backend_ = attention;
        drop_graphs();
    }
    // Replay the forward from a CUDA graph captured per input shape and buffer
    // pair (on by default; streams that cannot be captured run eagerly).
    void set_graphs(bool on) {
        graphs_on_ = on;
        if (!on) drop_graphs();
    }
    bool graphs() const { return graphs_on_; }
    int gemm_backend() const { return gemm_backend_; }
    int attn_backend() const { return attn_backend_; }
    // Kernel launches issued by the last forward().
    int64_t last_launches() const { return launches_; }
    // Reads (synchronously) and clears the device error word the tensor-core
    // kernels set when a bounded wait gives up; throws ERR_TIMEOUT if set.
    void check_device_error();

    // Per-kernel-class profiler: when enabled every launch is bracketed by CUDA
    // events; profile_read() synchronises on the recorded events and returns the
    // accumulated milliseconds and launch count of `kind` since the last reset.
    void profile_enable(bool on);
    void profile_reset();
    void profile_read(int kind, double* ms, int64_t* count);

private:
    struct Plan {
        size_t first = 0;  // index into the workspace's group array
        int n = 0, maxM = 0, maxN = 0, maxK = 0, epi = 0;
        int launch = -1;  // index into Workspace::launches (tensor-core path)
        // QKV projections: the launch above writes RoPE'd q|k|v token-major
        // (read in place by the tensor-core attention); this one scatters them
        // head-major for the CUDA-core attention
        int launch_scatter = -1;
        int qkv_mode = -1;  // QKV projection of a time (0) / band (1) transformer
        int ffn = -1;       // FFN1 plan: index into Workspace::ffn_launches of the fused FFN block
        // operand tensor shapes for the tensor-core path (rows x cols, elements)
        const void* a_base = nullptr;
        int64_t a_rows = 0, a_cols = 0;
        const void* b_base = nullptr;
        int64_t b_rows = 0, b_cols = 0;
        // output view C[group][row][col] for TMA-staged epilogue stores
        // (c_dtype < 0: stores from registers)
        const void* c_base = nullptr;
        int64_t c_rows = 0, c_cols = 0, c_groups = 1, c_row_stride = 0, c_group_stride = 0;
        int c_dtype = -1;
    };
    struct LayerW {
        float* attn_gamma;
        void* wqkv;
        float* wg;
        float* bg;
        void* wo;
        float* ff_gamma;
        void* w1;
        float* b1;
        void* w2;
        float* b2;
    };
    struct TransW {
        std::vector<LayerW> layers;
        float* final_gamma;
    };
    struct Workspace {
        int B = 0;
        int64_t L = 0, T = 0, MT = 0, M = 0, lout = 0;
        void* base = nullptr;
        size_t bytes = 0;
        float2* spec;
        void* xb;
        float* R;
        void* xn;
        float* gates;
        void* qkv;
        void* q;
        void* k;
        void* v;
        void* merged;
        void* hf;
        void* rm;
        void* mh[2];
        float* masks;
        float2* y;
        float* frames;
        std::vector<float*> skip;
        float *rope_t_cos, *rope_t_sin, *rope_f_cos, *rope_f_sin;
        ops::GemmGroup* d_groups;
        std::vector<ops::GemmGroup> h_groups;
        std::vector<tc::GemmLaunch> launches;
        std::vector<tc::FfnLaunch> ffn_launches;
        int4* d_tiles = nullptr;
        Plan band_split;
        std::vector<Plan> layer_plans;  // [depth][2][layers][4]: qkv, out, ffn1, ffn2
        std::vector<std::vector<Plan>> mask_plans;  // [stem][linear]
        // CUDA graphs of the whole forward, one per (input, output) buffer pair
        struct Graph {
            const float* in;
            float* out;
            cudaGraphExec_t exec;  // null: capture failed, run eagerly
            int64_t launches;
        };
        std::vector<Graph> graphs;
    };

    Workspace& workspace(int B, int64_t L);
    void build_plans(Workspace& ws);
    // launch: a prepared tensor-core launch other than p.launch (-1: p.launch)
    void run_gemm(const Workspace& ws, const Plan& p, int kind, cudaStream_t st, int launch = -1);
    void run_transformer(Workspace& ws, const TransW& tw, int mode, const Plan* plans, bool last_of_model,
                         cudaStream_t st, bool first_norm_done = false, const LayerW* next_first = nullptr);
    void run_forward(Workspace& ws, const float* d_audio, float* d_out, int tap, float* d_tap, int64_t* tap_n,
                     cudaStream_t st);

    MBRConfig cfg_;
    int device_ = 0, dtype_ = DT_F16, C_ = 2, F_ = 1025, NB_ = 60, D_ = 384, H_ = 8, dh_ = 64, DI_ = 512,
        hid_ = 1536;
    int64_t J_ = 0, KP_ = 0;
    int gemm_backend_ = BACKEND_SIMT, attn_backend_ = BACKEND_SIMT;
    // FFN1 + GELU + FFN2 as one kernel where it applies (MBR_FFN_FUSED=1; the
    // default keeps the two GEMMs, measured faster on B200)
    bool ffn_fused_ = false;
    int64_t launches_ = 0;
    bool graphs_on_ = true;
    void drop_graphs();

    // profiler state
    bool prof_on_ = false;
    struct ProfRec {
        int kind;
        cudaEvent_t a, b;
    };
    std::vector<ProfRec> prof_recs_;
    std::vector<cudaEvent_t> prof_pool_;
    size_t prof_used_ = 0;
    double prof_ms_[PK_COUNT] = {};
    int64_t prof_n_[PK_COUNT] = {};
    int prof_begin(int kind, cudaStream_t st);
    void prof_end(int rec, cudaStream_t st);
    void prof_collect();

    std::vector<int> band_bd_, band_boff_, band_kofs_;  // host copies
    void* wbase_ = nullptr;  // single device allocation holding every weight
    int* d_err_ = nullptr;   // error word of the tensor-core kernels
    int *d_fi_, *d_band_jofs_, *d_band_kofs_, *d_rev_off_, *d_rev_idx_;
    opsapi::BandTiles band_tiles_;
    void* d_band_tiles_ = nullptr;
    float *d_nbpf_, *d_window_, *d_bs_gamma_, *d_bs_bias_;
    float2* d_twiddle_;
    void* d_wbs_;
    std::vector<TransW> tt_, ft_;
    struct MaskW {
        std::vector<void*> w;
        std::vector<float*> b;
        std::vector<int> in, out;  // per-band dims (out of the last layer varies per band)
    };
    std::vector<MaskW> mask_;
    std::map<std::pair<int, int64_t>, std::unique_ptr<Workspace>> ws_;
};

}  // namespace mbr
