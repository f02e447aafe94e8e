// audio_io.cpp — WAV reader / writer (reference behaviour: src/audio_io.cpp:59-334).
#include "audio_io.h"

#include <cstring>
#include <fstream>
#include <stdexcept>

namespace cudasep {

namespace {

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }

void put16(std::ofstream& f, uint16_t v) {
    uint8_t b[2] = {(uint8_t)v, (uint8_t)(v >> 8)};
    f.write((const char*)b, 2);
}
void put32(std::ofstream& f, uint32_t v) {
    uint8_t b[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    f.write((const char*)b, 4);
}

}  // namespace

std::vector<uint8_t> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("Failed to open WAV file: " + path);
    return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

WavLayout parse_wav(const uint8_t* bytes, size_t size, const std::string& path) {
    struct View {
        const uint8_t* p;
        size_t n;
        size_t size() const { return n; }
        const uint8_t* data() const { return p; }
    } buf{bytes, size};
    if (buf.size() < 12 || std::memcmp(buf.data(), "RIFF", 4) != 0)
        throw std::runtime_error("Not a valid WAV file (missing RIFF header): " + path);
    if (std::memcmp(buf.data() + 8, "WAVE", 4) != 0)
        throw std::runtime_error("Not a valid WAV file (missing WAVE tag): " + path);
    uint16_t fmt = 0, ch = 0, bits = 0;
    uint32_t sr = 0;
    const uint8_t* data = nullptr;
    size_t data_size = 0;
    bool have_fmt = false;
    size_t p = 12;
    while (p + 8 <= buf.size() && !(have_fmt && data)) {
        const uint8_t* id = buf.data() + p;
        uint32_t sz = rd32(buf.data() + p + 4);
        size_t body = p + 8;
        if (std::memcmp(id, "fmt ", 4) == 0 && body + 16 <= buf.size()) {
            fmt = rd16(buf.data() + body);
            ch = rd16(buf.data() + body + 2);
            sr = rd32(buf.data() + body + 4);
            bits = rd16(buf.data() + body + 14);
            if (fmt == 0xFFFE && sz >= 40 && body + 26 <= buf.size()) fmt = rd16(buf.data() + body + 24);  // SubFormat
            have_fmt = true;
        } else if (std::memcmp(id, "data", 4) == 0) {
            data = buf.data() + body;
            data_size = std::min<size_t>(sz, buf.size() - body);
        }
        p = body + sz + (sz & 1);
    }
    if (!have_fmt) throw std::runtime_error("WAV file has no fmt chunk: " + path);
    if (!data) throw std::runtime_error("WAV file has no data chunk: " + path);
    if (fmt != 1 && fmt != 3) throw std::runtime_error("Unsupported WAV audio format: " + std::to_string(fmt) + ": " + path);
    if (fmt == 1 && bits != 16 && bits != 24 && bits != 32)
        throw std::runtime_error("Unsupported PCM bit depth: " + std::to_string(bits) + ": " + path);
    if (fmt == 3 && bits != 32) throw std::runtime_error("Unsupported float bit depth: " + std::to_string(bits) + ": " + path);
    if (ch == 0) throw std::runtime_error("WAV file has zero channels: " + path);
    WavLayout w;
    w.format = fmt;
    w.channels = ch;
    w.bits = bits;
    w.sample_rate = (int)sr;
    w.data_off = (size_t)(data - buf.data());
    w.frames = (int64_t)(data_size / ((size_t)(bits / 8) * ch));
    w.data_bytes = (size_t)w.frames * (bits / 8) * ch;
    return w;
}

HostAudio read_wav_host(const std::string& path) {
    std::vector<uint8_t> buf = read_file(path);
    const WavLayout w = parse_wav(buf.data(), buf.size(), path);
    const int fmt = w.format, bits = w.bits, ch = w.channels;
    const uint8_t* data = buf.data() + w.data_off;
    const int bps = bits / 8;
    HostAudio a;
    a.sample_rate = w.sample_rate;
    a.channels = ch;
    a.frames = w.frames;
    a.planar.resize((size_t)a.frames * ch);
    for (int64_t i = 0; i < a.frames; ++i)
        for (int c = 0; c < ch; ++c) {
            const uint8_t* s = data + ((size_t)i * ch + c) * bps;
            float v;
            if (fmt == 3) {
                std::memcpy(&v, s, 4);
            } else if (bits == 16) {
                v = (float)(int16_t)rd16(s) / 32768.0f;
            } else if (bits == 24) {
                int32_t x = (int32_t)(s[0] | (s[1] << 8) | (s[2] << 16));
                if (x & 0x800000) x |= ~0xFFFFFF;
                v = (float)x / 8388608.0f;
            } else {
                v = (float)(int32_t)rd32(s) / 2147483648.0f;
            }
            a.planar[(size_t)c * a.frames + i] = v;
        }
    return a;
}

void write_wav_host(const std::string& path, const float* planar, int ch, int64_t frames, int sr) {
    std::vector<float> inter((size_t)frames * ch);
    for (int64_t i = 0; i < frames; ++i)
        for (int c = 0; c < ch; ++c) inter[(size_t)i * ch + c] = planar[(size_t)c * frames + i];
    write_wav_interleaved(path, inter.data(), ch, frames, sr);
}

void write_wav_interleaved(const std::string& path, const float* inter, int ch, int64_t frames, int sr) {
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("Failed to create WAV file: " + path);
    const uint32_t data_bytes = (uint32_t)(frames * ch * 4);
    f.write("RIFF", 4);
    put32(f, 36 + data_bytes);
    f.write("WAVE", 4);
    f.write("fmt ", 4);
    put32(f, 16);
    put16(f, 3);  // IEEE float
    put16(f, (uint16_t)ch);
    put32(f, (uint32_t)sr);
    put32(f, (uint32_t)(sr * ch * 4));
    put16(f, (uint16_t)(ch * 4));
    put16(f, 32);
    f.write("data", 4);
    put32(f, data_bytes);
    f.write((const char*)inter, (std::streamsize)((size_t)frames * ch * 4));
    if (!f) throw std::runtime_error("Failed to write WAV file: " + path);
}

AudioData load_wav(const std::string& path) {
    HostAudio h = read_wav_host(path);
    AudioData a;
    a.sample_rate = h.sample_rate;
    a.channels = h.channels;
    a.num_samples = h.frames;
    a.samples = Tensor::from_cpu_f32(h.planar.data(), {(int64_t)h.channels, h.frames});
    return a;
}

void save_wav(const std::string& path, const Tensor& samples, int sample_rate) {
    Tensor s = samples.ndim() == 1 ? samples.unsqueeze(0) : samples;
    if (s.ndim() != 2) throw std::runtime_error("save_wav: expected [channels, samples]");
    std::vector<float> h = s.to_cpu_f32();
    write_wav_host(path, h.data(), (int)s.size(0), s.size(1), sample_rate);
}

}  // namespace cudasep
