// weights.h — `.csm` v1 checkpoint loader and its JSON config.
//
// Mirrors the reference interface of src/weights.h:19-130 (JsonValue,
// ModelWeights::load/get/has/tensor_names/convert_linear_weights_to_{fp16,bf16})
// so callers port unchanged.  Difference by design: tensors stay in host memory
// here; the model uploads them once, already converted and packed into the
// layouts its kernels read (one device allocation for all weights), instead of
// one device allocation per tensor.
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace mbr {

class JsonValue {
public:
    enum Type { Null, Bool, Number, String, Array, Object };
    JsonValue() = default;

    bool is_null() const { return type_ == Null; }
    bool is_bool() const { return type_ == Bool; }
    bool is_number() const { return type_ == Number; }
    bool is_string() const { return type_ == String; }
    bool is_array() const { return type_ == Array; }
    bool is_object() const { return type_ == Object; }

    bool as_bool() const;
    double as_number() const;
    int as_int() const { return (int)as_number(); }
    int64_t as_int64() const { return (int64_t)as_number(); }
    float as_float() const { return (float)as_number(); }
    const std::string& as_string() const;

    size_t size() const;
    const JsonValue& operator[](size_t index) const;
    const JsonValue& operator[](const std::string& key) const;
    bool has(const std::string& key) const;

    int get_int(const std::string& key, int def) const;
    float get_float(const std::string& key, float def) const;
    bool get_bool(const std::string& key, bool def) const;
    std::string get_string(const std::string& key, const std::string& def) const;

    static JsonValue parse(const std::string& json);

private:
    friend struct JsonReader;
    Type type_ = Null;
    bool bool_ = false;
    double num_ = 0.0;
    std::string str_;
    std::vector<JsonValue> arr_;
    std::vector<std::pair<std::string, JsonValue>> obj_;
};

// Host tensor as stored in the .csm file.  dtype codes: 0 f32, 1 f16, 2 i64, 3 bf16.
struct HostTensor {
    std::vector<int64_t> shape;
    int dtype = 0;
    std::vector<uint8_t> data;
    int64_t numel() const;
    int ndim() const { return (int)shape.size(); }
    // Element i converted to float (f32/f16/bf16) or int64 (i64).
    float f(int64_t i) const;
    int64_t i64(int64_t i) const;
};

class ModelWeights {
public:
    static ModelWeights load(const std::string& path);
    const JsonValue& config() const { return config_; }
    const HostTensor& get(const std::string& name) const;
    bool has(const std::string& name) const;
    std::vector<std::string> tensor_names() const;
    size_t num_tensors() const { return tensors_.size(); }
    // Round every 2-D fp32 tensor to fp16 / bf16 (round to nearest even), as the
    // reference does for --fp16 / --bf16 (src/weights.cu:511-540).
    void convert_linear_weights_to_fp16();
    void convert_linear_weights_to_bf16();

private:
    JsonValue config_;
    std::map<std::string, HostTensor> tensors_;
};

// Host-side float <-> 16-bit conversions (round to nearest even).
uint16_t float_to_half_bits(float x);
float half_bits_to_float(uint16_t h);
uint16_t float_to_bf16_bits(float x);
float bf16_bits_to_float(uint16_t h);

}  // namespace mbr
