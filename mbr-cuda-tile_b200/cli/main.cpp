// cudasep_infer — command-line separator with the reference CLI's flags
// (src/main.cpp:27-68): --model/-m, --input/-i, --output/-o, --stem/-s,
// --overlap, --device/-d, --fp16, --bf16, --chunk-batch-size, --help; plus
// --fp32 (the reference accepts --bf16 only, src/main.cpp:87-90) and --gpus N
// (contiguous chunk ranges on devices device .. device+N-1).
// Runs entirely through the C ABI of libmbr_b200.so.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <iostream>
#include <string>
#include <vector>

#include "../../include/mbr_b200.h"

namespace fs = std::filesystem;

struct Args {
    std::string model, input, output = "output";
    int stem = 0, device = 0, gpus = 1, chunk_batch = 0;
    float overlap = -1.0f;
    bool fp16 = false, bf16 = false, fp32 = false, help = false;
};

static Args parse(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        std::string s = argv[i];
        auto next = [&]() -> std::string { return i + 1 < argc ? argv[++i] : std::string(); };
        if ((s == "--model" || s == "-m") && i + 1 < argc) a.model = next();
        else if ((s == "--input" || s == "-i") && i + 1 < argc) a.input = next();
        else if ((s == "--output" || s == "-o") && i + 1 < argc) a.output = next();
        else if ((s == "--stem" || s == "-s") && i + 1 < argc) a.stem = std::stoi(next());
        else if (s == "--overlap" && i + 1 < argc) a.overlap = std::stof(next());
        else if ((s == "--device" || s == "-d") && i + 1 < argc) a.device = std::stoi(next());
        else if (s == "--gpus" && i + 1 < argc) a.gpus = std::stoi(next());
        else if (s == "--fp16") a.fp16 = true;
        else if (s == "--bf16") a.bf16 = true;
        else if (s == "--fp32") a.fp32 = true;
        else if (s == "--chunk-batch-size" && i + 1 < argc) a.chunk_batch = std::stoi(next());
        else if (s == "--help" || s == "-h") a.help = true;
    }
    return a;
}

static void usage(const char* prog) {
    std::cout << "B200 MelBandRoformer WAV CLI\n\n"
              << "Usage:\n  " << prog << " --model <model.csm> --input <audio.wav> [options]\n\n"
              << "Options:\n"
              << "  --output, -o <path>       Output directory or WAV file path (default: output)\n"
              << "  --stem, -s <int>          Stem index to save (default: 0, -1 saves all)\n"
              << "  --bf16 | --fp16 | --fp32  Compute dtype (default bf16)\n"
              << "  --chunk-batch-size <n>    Chunks per forward (default 1)\n"
              << "  --overlap <float>         (0,1)=overlap ratio, >=1=num_overlap\n"
              << "  --device, -d <int>        First CUDA device (default: 0)\n"
              << "  --gpus <n>                Number of GPUs (default: 1)\n"
              << "  --help, -h                Show this help message\n";
}

static int fail(const std::string& m) {
    std::cerr << "Error: " << m << std::endl;
    return 1;
}

int main(int argc, char** argv) {
    Args a = parse(argc, argv);
    if (a.help) {
        usage(argv[0]);
        return 0;
    }
    if (a.model.empty()) return fail("--model is required");
    if (a.input.empty()) return fail("--input is required");
    if ((int)a.fp16 + (int)a.bf16 + (int)a.fp32 > 1) return fail("--fp16, --bf16 and --fp32 are mutually exclusive");
    const int dtype = a.fp16 ? MBR_FP16 : a.fp32 ? MBR_FP32 : MBR_BF16;

    std::cout << "Loading model: " << a.model << std::endl;
    mbr_handle* h = nullptr;
    if (mbr_create(a.model.c_str(), a.device, dtype, &h) != MBR_OK) return fail(mbr_last_error());
    int64_t S = 0, C = 0, sr = 0, chunk = 0, ov = 0;
    mbr_get_info(h, MBR_INFO_NUM_STEMS, &S);
    mbr_get_info(h, MBR_INFO_CHANNELS, &C);
    mbr_get_info(h, MBR_INFO_SAMPLE_RATE, &sr);
    mbr_get_info(h, MBR_INFO_CHUNK_SIZE, &chunk);
    mbr_get_info(h, MBR_INFO_NUM_OVERLAP, &ov);
    std::cout << "  Model type: MelBandRoformer\n  Sources: " << S << ", Sample rate: " << sr
              << ", Chunk size: " << chunk << ", Num overlap: " << ov << std::endl;

    int wsr = 0, wch = 0;
    int64_t frames = 0;
    std::cout << "\nLoading WAV: " << a.input << std::endl;
    if (mbr_wav_info(a.input.c_str(), &wsr, &wch, &frames) != MBR_OK) return fail(mbr_last_error());
    std::vector<float> wav((size_t)wch * frames);
    if (mbr_wav_read(a.input.c_str(), wav.data(), (int64_t)wav.size()) != MBR_OK) return fail(mbr_last_error());
    std::cout << "  " << wch << "ch, " << wsr << " Hz, " << frames << " samples (" << (double)frames / wsr << "s)"
              << std::endl;
    if (wsr != sr) std::cerr << "Warning: WAV sample rate (" << wsr << ") != model sample rate (" << sr << ")." << std::endl;
    // the model's channel count: duplicate mono into stereo or keep the first channels
    std::vector<float> track((size_t)C * frames);
    for (int64_t c = 0; c < C; ++c)
        std::memcpy(track.data() + c * frames, wav.data() + (std::min<int64_t>(c, wch - 1)) * frames,
                    sizeof(float) * frames);
    std::vector<float> stems((size_t)S * C * frames);
    std::cout << "\nRunning inference..." << std::endl;
    auto t0 = std::chrono::high_resolution_clock::now();
    int rc = mbr_separate(h, track.data(), frames, a.overlap, std::max(1, a.chunk_batch), std::max(1, a.gpus),
                          stems.data());
    auto t1 = std::chrono::high_resolution_clock::now();
    if (rc != MBR_OK) return fail(mbr_last_error());
    double ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    std::printf("  Inference time: %.1f ms (RTF: %.2fx)\n", ms, (double)frames / sr / (ms / 1000.0));

    // save_outputs (src/inference_app.cpp:377-420)
    auto save = [&](int s, const fs::path& p) {
        if (mbr_wav_write(p.string().c_str(), stems.data() + (size_t)s * C * frames, (int)C, frames, (int)sr) != MBR_OK)
            throw std::runtime_error(mbr_last_error());
        std::cout << "Saving: " << p.string() << std::endl;
    };
    try {
        fs::path out(a.output);
        static const char* names[] = {"vocals", "instrumental", "drums", "bass"};
        auto label = [&](int s) { return S <= 4 ? std::string(names[s]) : "stem_" + std::to_string(s); };
        if (S == 1) {
            fs::path f = out;
            if (out.extension() != ".wav") {
                fs::create_directories(out);
                f = out / "output.wav";
            }
            save(0, f);
        } else if (a.stem >= 0) {
            if (a.stem >= S) return fail("Stem index out of range");
            fs::path f = out;
            if (out.extension() != ".wav") {
                fs::create_directories(out);
                f = out / (label(a.stem) + ".wav");
            }
            save(a.stem, f);
        } else {
            fs::create_directories(out);
            for (int s = 0; s < S; ++s) save(s, out / (label(s) + ".wav"));
        }
    } catch (const std::exception& e) {
        return fail(e.what());
    }
    mbr_destroy(h);
    std::cout << "Done." << std::endl;
    return 0;
}
