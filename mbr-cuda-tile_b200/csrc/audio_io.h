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
void write_wav_host(const std::string& path, const float* planar, int channels, int64_t frames, int sample_rate);

}  // namespace cudasep
