// weights.cpp — `.csm` v1 reader and JSON config parser (reference interface:
// src/weights.h:19-130, file layout src/weights.h:82-96).
#include "weights.h"

#include <cmath>
#include <cstring>
#include <fstream>

#include "common.h"

namespace mbr {

// ---------------------------------------------------------------------------
// 16-bit conversions
// ---------------------------------------------------------------------------
uint16_t float_to_half_bits(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) {  // below the smallest normal half: subnormal / zero
        float v = std::fabs(x) * 16777216.0f;  // exact scaling by 2^24
        return (uint16_t)(sign | (uint32_t)std::nearbyint(v));
    }
    uint32_t mant = a & 0x7fffffu;
    uint32_t e = (a >> 23) - 127 + 15;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        float v = (float)m / 16777216.0f;
        std::memcpy(&u, &v, 4);
        u |= sign;
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

uint16_t float_to_bf16_bits(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float bf16_bits_to_float(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// ---------------------------------------------------------------------------
// JSON
// ---------------------------------------------------------------------------
struct JsonReader {
    const std::string& s;
    size_t p = 0;
    explicit JsonReader(const std::string& src) : s(src) {}
    [[noreturn]] void fail(const std::string& m) { throw Error(ERR_IO, "JSON parse error: " + m); }
    void ws() {
        while (p < s.size() && (s[p] == ' ' || s[p] == '\t' || s[p] == '\n' || s[p] == '\r')) ++p;
    }
    char peek() {
        ws();
        if (p >= s.size()) fail("unexpected end");
        return s[p];
    }
    std::string string() {
        if (peek() != '"') fail("expected string");
        ++p;
        std::string out;
        while (true) {
            if (p >= s.size()) fail("unterminated string");
            char c = s[p++];
            if (c == '"') break;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p >= s.size()) fail("bad escape");
            char e = s[p++];
            switch (e) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {
                    if (p + 4 > s.size()) fail("bad unicode escape");
                    unsigned cp = (unsigned)std::stoul(s.substr(p, 4), nullptr, 16);
                    p += 4;
                    if (cp < 0x80) {
                        out += (char)cp;
                    } else if (cp < 0x800) {
                        out += (char)(0xc0 | (cp >> 6));
                        out += (char)(0x80 | (cp & 0x3f));
                    } else {
                        out += (char)(0xe0 | (cp >> 12));
                        out += (char)(0x80 | ((cp >> 6) & 0x3f));
                        out += (char)(0x80 | (cp & 0x3f));
                    }
                    break;
                }
                default: out += e;
            }
        }
        return out;
    }
    JsonValue value() {
        JsonValue v;
        char c = peek();
        if (c == '{') {
            ++p;
            v.type_ = JsonValue::Object;
            if (peek() == '}') {
                ++p;
                return v;
            }
            while (true) {
                std::string k = string();
                if (peek() != ':') fail("expected ':'");
                ++p;
                v.obj_.emplace_back(k, value());
                char d = peek();
                ++p;
                if (d == '}') break;
                if (d != ',') fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++p;
            v.type_ = JsonValue::Array;
            if (peek() == ']') {
                ++p;
                return v;
            }
            while (true) {
                v.arr_.push_back(value());
                char d = peek();
                ++p;
                if (d == ']') break;
                if (d != ',') fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.type_ = JsonValue::String;
            v.str_ = string();
        } else if (s.compare(p, 4, "true") == 0) {
            p += 4;
            v.type_ = JsonValue::Bool;
            v.bool_ = true;
        } else if (s.compare(p, 5, "false") == 0) {
            p += 5;
            v.type_ = JsonValue::Bool;
        } else if (s.compare(p, 4, "null") == 0) {
            p += 4;
        } else {
            const char* b = s.c_str() + p;
            char* e = nullptr;
            double d = std::strtod(b, &e);
            if (e == b) fail("bad value at offset " + std::to_string(p));
            p += (size_t)(e - b);
            v.type_ = JsonValue::Number;
            v.num_ = d;
        }
        return v;
    }
};

JsonValue JsonValue::parse(const std::string& json) {
    JsonReader r(json);
    JsonValue v = r.value();
    r.ws();
    if (r.p != json.size()) r.fail("trailing characters");
    return v;
}

bool JsonValue::as_bool() const {
    if (type_ != Bool) throw Error(ERR_INVALID, "JsonValue: not a bool");
    return bool_;
}
double JsonValue::as_number() const {
    if (type_ != Number) throw Error(ERR_INVALID, "JsonValue: not a number");
    return num_;
}
const std::string& JsonValue::as_string() const {
    if (type_ != String) throw Error(ERR_INVALID, "JsonValue: not a string");
    return str_;
}
size_t JsonValue::size() const { return type_ == Array ? arr_.size() : type_ == Object ? obj_.size() : 0; }
const JsonValue& JsonValue::operator[](size_t i) const {
    if (type_ != Array || i >= arr_.size()) throw Error(ERR_INVALID, "JsonValue: bad array index");
    return arr_[i];
}
const JsonValue& JsonValue::operator[](const std::string& k) const {
    for (auto& kv : obj_)
        if (kv.first == k) return kv.second;
    throw Error(ERR_INVALID, "JsonValue: missing key " + k);
}
bool JsonValue::has(const std::string& k) const {
    if (type_ != Object) return false;
    for (auto& kv : obj_)
        if (kv.first == k) return true;
    return false;
}
int JsonValue::get_int(const std::string& k, int def) const {
    if (!has(k)) return def;
    const JsonValue& v = (*this)[k];
    if (v.is_number()) return v.as_int();
    if (v.is_bool()) return v.as_bool() ? 1 : 0;
    return def;
}
float JsonValue::get_float(const std::string& k, float def) const {
    if (!has(k)) return def;
    const JsonValue& v = (*this)[k];
    return v.is_number() ? v.as_float() : def;
}
bool JsonValue::get_bool(const std::string& k, bool def) const {
    if (!has(k)) return def;
    const JsonValue& v = (*this)[k];
    if (v.is_bool()) return v.as_bool();
    if (v.is_number()) return v.as_number() != 0.0;
    return def;
}
std::string JsonValue::get_string(const std::string& k, const std::string& def) const {
    if (!has(k)) return def;
    const JsonValue& v = (*this)[k];
    return v.is_string() ? v.as_string() : def;
}

// ---------------------------------------------------------------------------
// tensors
// ---------------------------------------------------------------------------
int64_t HostTensor::numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
}
float HostTensor::f(int64_t i) const {
    switch (dtype) {
        case DT_F32: {
            float v;
            std::memcpy(&v, data.data() + 4 * i, 4);
            return v;
        }
        case DT_F16: {
            uint16_t h;
            std::memcpy(&h, data.data() + 2 * i, 2);
            return half_bits_to_float(h);
        }
        case DT_BF16: {
            uint16_t h;
            std::memcpy(&h, data.data() + 2 * i, 2);
            return bf16_bits_to_float(h);
        }
        default: return (float)i64(i);
    }
}
int64_t HostTensor::i64(int64_t i) const {
    if (dtype != DT_I64) return (int64_t)f(i);
    int64_t v;
    std::memcpy(&v, data.data() + 8 * i, 8);
    return v;
}

// Restates ModelWeights::load (src/weights.cu:412-509).
ModelWeights ModelWeights::load(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error(ERR_IO, "ModelWeights: cannot open file: " + path);
    auto rd = [&](void* d, size_t n) {
        f.read((char*)d, (std::streamsize)n);
        if (!f) throw Error(ERR_IO, "ModelWeights: unexpected EOF in " + path);
    };
    char magic[4];
    rd(magic, 4);
    if (std::memcmp(magic, "CSM\0", 4) != 0) throw Error(ERR_IO, "ModelWeights: invalid magic (expected CSM\\0)");
    uint32_t ver, jl, nt;
    rd(&ver, 4);
    if (ver != 1) throw Error(ERR_IO, "ModelWeights: unsupported version " + std::to_string(ver));
    rd(&jl, 4);
    std::string js(jl, '\0');
    rd(&js[0], jl);
    ModelWeights w;
    w.config_ = JsonValue::parse(js);
    rd(&nt, 4);
    for (uint32_t t = 0; t < nt; ++t) {
        uint32_t nl;
        rd(&nl, 4);
        std::string name(nl, '\0');
        rd(&name[0], nl);
        uint32_t nd;
        rd(&nd, 4);
        HostTensor ht;
        ht.shape.resize(nd);
        for (uint32_t d = 0; d < nd; ++d) rd(&ht.shape[d], 8);
        uint32_t dt;
        rd(&dt, 4);
        if (dt > 3) throw Error(ERR_IO, "ModelWeights: unknown dtype " + std::to_string(dt) + " for tensor " + name);
        ht.dtype = (int)dt;
        ht.data.resize((size_t)ht.numel() * dtype_bytes((int)dt));
        if (!ht.data.empty()) rd(ht.data.data(), ht.data.size());
        w.tensors_[std::move(name)] = std::move(ht);
    }
    return w;
}

const HostTensor& ModelWeights::get(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw Error(ERR_IO, "ModelWeights: tensor not found: " + name);
    return it->second;
}
bool ModelWeights::has(const std::string& name) const { return tensors_.count(name) > 0; }
std::vector<std::string> ModelWeights::tensor_names() const {
    std::vector<std::string> v;
    for (auto& kv : tensors_) v.push_back(kv.first);
    return v;
}

static void convert_2d(std::map<std::string, HostTensor>& ts, int to) {
    for (auto& kv : ts) {
        HostTensor& t = kv.second;
        if (t.ndim() != 2 || t.dtype != DT_F32) continue;
        int64_t n = t.numel();
        std::vector<uint8_t> d((size_t)n * 2);
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h = to == DT_F16 ? float_to_half_bits(t.f(i)) : float_to_bf16_bits(t.f(i));
            std::memcpy(d.data() + 2 * i, &h, 2);
        }
        t.data.swap(d);
        t.dtype = to;
    }
}
void ModelWeights::convert_linear_weights_to_fp16() { convert_2d(tensors_, DT_F16); }
void ModelWeights::convert_linear_weights_to_bf16() { convert_2d(tensors_, DT_BF16); }

}  // namespace mbr
