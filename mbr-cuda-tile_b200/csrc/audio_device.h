// audio_device.h — WAV sample conversion kernels (see audio_device.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mbr {
namespace audio {

// Interleaved PCM [frames][channels] (16 / 24 / 32-bit integer, or 32-bit
// float) -> planar fp32 [channels][frames]; integer PCM / 2^(bits-1).
void pcm_to_planar(const void* d_pcm, int64_t frames, int channels, int bits, bool is_float, float* d_planar,
                   cudaStream_t st);
// Planar fp32 [channels][frames] -> interleaved fp32 [frames][channels].
void planar_to_interleaved(const float* d_planar, int64_t frames, int channels, float* d_out, cudaStream_t st);

}  // namespace audio
}  // namespace mbr
