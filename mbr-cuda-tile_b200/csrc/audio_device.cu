// audio_device.cu — WAV sample conversion on the GPU: interleaved PCM (16 / 24
// / 32-bit integer or 32-bit float) to planar fp32, and planar fp32 back to
// interleaved for a float WAV.  The reference converts on the host, one sample
// at a time (src/audio_io.cpp:200-334); here the file's data chunk is copied
// to the device as raw bytes and converted there, with the same scaling
// (integer PCM divided by 2^(bits-1), so results equal the host reader's).
#include "audio_device.h"
#include "common.cuh"

namespace mbr {
namespace audio {

namespace {

// One thread per interleaved sample: consecutive threads read consecutive
// bytes; the planar writes of a warp fall into `ch` contiguous runs.
template <int BITS, bool FLOAT>
__global__ void pcm_to_planar_kernel(const uint8_t* __restrict__ pcm, int64_t frames, int ch,
                                     float* __restrict__ out) {
    const int64_t n = frames * ch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f = i / ch;
        const int c = (int)(i - f * ch);
        float v;
        if constexpr (FLOAT) {
            v = reinterpret_cast<const float*>(pcm)[i];
        } else if constexpr (BITS == 16) {
            v = (float)reinterpret_cast<const int16_t*>(pcm)[i] / 32768.0f;
        } else if constexpr (BITS == 24) {
            const uint8_t* s = pcm + 3 * i;
            int32_t x = (int32_t)((uint32_t)s[0] | ((uint32_t)s[1] << 8) | ((uint32_t)s[2] << 16));
            if (x & 0x800000) x |= ~0xFFFFFF;
            v = (float)x / 8388608.0f;
        } else {
            v = (float)reinterpret_cast<const int32_t*>(pcm)[i] / 2147483648.0f;
        }
        out[(int64_t)c * frames + f] = v;
    }
}

__global__ void planar_to_interleaved_kernel(const float* __restrict__ planar, int64_t frames, int ch,
                                             float* __restrict__ out) {
    const int64_t n = frames * ch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t f = i / ch;
        const int c = (int)(i - f * ch);
        out[i] = planar[(int64_t)c * frames + f];
    }
}

unsigned grid_for(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace

void pcm_to_planar(const void* d_pcm, int64_t frames, int channels, int bits, bool is_float, float* d_planar,
                   cudaStream_t st) {
    MBR_CHECK(frames >= 0 && channels >= 1, "pcm_to_planar: bad shape");
    if (frames == 0) return;
    const uint8_t* p = (const uint8_t*)d_pcm;
    const int64_t n = frames * channels;
    if (is_float) {
        MBR_CHECK(bits == 32 && ((uintptr_t)p & 3) == 0, "pcm_to_planar: float samples must be 32-bit, aligned");
        pcm_to_planar_kernel<32, true><<<grid_for(n), 256, 0, st>>>(p, frames, channels, d_planar);
    } else if (bits == 16) {
        MBR_CHECK(((uintptr_t)p & 1) == 0, "pcm_to_planar: misaligned 16-bit samples");
        pcm_to_planar_kernel<16, false><<<grid_for(n), 256, 0, st>>>(p, frames, channels, d_planar);
    } else if (bits == 24) {
        pcm_to_planar_kernel<24, false><<<grid_for(n), 256, 0, st>>>(p, frames, channels, d_planar);
    } else if (bits == 32) {
        MBR_CHECK(((uintptr_t)p & 3) == 0, "pcm_to_planar: misaligned 32-bit samples");
        pcm_to_planar_kernel<32, false><<<grid_for(n), 256, 0, st>>>(p, frames, channels, d_planar);
    } else {
        throw Error(ERR_INVALID, "pcm_to_planar: integer PCM must be 16, 24 or 32-bit");
    }
    MBR_CUDA(cudaGetLastError());
}

void planar_to_interleaved(const float* d_planar, int64_t frames, int channels, float* d_out, cudaStream_t st) {
    MBR_CHECK(frames >= 0 && channels >= 1, "planar_to_interleaved: bad shape");
    if (frames == 0) return;
    planar_to_interleaved_kernel<<<grid_for(frames * channels), 256, 0, st>>>(d_planar, frames, channels, d_out);
    MBR_CUDA(cudaGetLastError());
}

}  // namespace audio
}  // namespace mbr
