// audio_io.h — WAV read/write (reference interface: src/audio_io.h:7-18).
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

#include "tensor.h"

namespace cudasep {

struct AudioData {
    Tensor samples;  // [channels, num_samples] Float32 on the GPU
    int sample_rate = 0;
    int channels = 0;
    int64_t num_samples = 0;
};

// PCM 16/24/32-bit and IEEE float32 WAV (WAVE_FORMAT_EXTENSIBLE included) ->
// planar float samples on the GPU; integer PCM scaled by 1/2^(bits-1).
AudioData load_wav(const std::string& path);
// [channels, num_samples] Float32 (GPU) -> IEEE float32 WAV.
void save_wav(const std::string& path, const Tensor& samples, int sample_rate);

// Host-memory forms used by the above and by the C ABI.
struct HostAudio {
    int sample_rate = 0;
    int channels = 0;
    int64_t frames = 0;
    std::vector<float> planar;  // [channels][frames]
};
HostAudio read_wav_host(const std::string& path);

// The fmt and data chunks of a WAV file held in memory (validated as
// read_wav_host validates them): data_off / data_bytes locate the interleaved
// samples in `bytes`; format 1 = integer PCM, 3 = IEEE float.
struct WavLayout {
    int format = 0, channels = 0, bits = 0, sample_rate = 0;
    size_t data_off = 0, data_bytes = 0;
    int64_t frames = 0;
};
WavLayout parse_wav(const uint8_t* bytes, size_t size, const std::string& what);
std::vector<uint8_t> read_file(const std::string& path);
void write_wav_host(const std::string& path, const float* planar, int channels, int64_t frames, int sample_rate);
// Float WAV from samples already interleaved [frames][channels].
void write_wav_interleaved(const std::string& path, const float* interleaved, int channels, int64_t frames,
                           int sample_rate);

}  // namespace cudasep
