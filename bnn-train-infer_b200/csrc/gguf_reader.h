// gguf_reader.h - read-only GGUF v3 view (mmap) for the device engine's loader.
//
// Accepts what the reference engine accepts (bnn-sw-v2/gguf.c:404-490):
// GGUF version 3, tensor types F32 (0), F16 (1) and Q1_0 (41), alignment
// from general.alignment (default 32). Metadata values are kept generically
// (integers, floats, strings, and string arrays for the tokenizer table).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <string_view>
#include <vector>

namespace bnn {

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t bytes = 0;
    const uint8_t* data = nullptr;
};

class GgufFile {
  public:
    ~GgufFile();
    // Returns false and sets error() on failure.
    bool open(const char* path);
    const std::string& error() const { return error_; }

    bool has(const std::string& key) const;
    bool get_u64(const std::string& key, uint64_t* out) const;
    bool get_f32(const std::string& key, float* out) const;
    bool get_str(const std::string& key, std::string* out) const;
    size_t array_len(const std::string& key) const;
    // Elements of a string array, as views into the mapped file (valid while
    // this object lives). False when the key is absent or not a string array.
    bool get_str_array(const std::string& key, std::vector<std::string_view>* out) const;
    // Elements of an int32 or uint32 array, as their 32-bit patterns. False
    // when the key is absent or holds another element type.
    bool get_u32_array(const std::string& key, std::vector<uint32_t>* out) const;

    const GgufTensor* tensor(const std::string& name) const;

  private:
    struct Value {
        int kind = 0;  // 1 int, 2 float, 3 string, 4 array
        uint64_t u = 0;
        double f = 0;
        std::string s;
        size_t n = 0;
        uint32_t elem = 0;               // arrays: GGUF element type
        const uint8_t* first = nullptr;  // arrays: first element in the map
    };
    bool fail(const std::string& why);
    std::map<std::string, Value> kv_;
    std::map<std::string, GgufTensor> tensors_;
    uint8_t* map_ = nullptr;
    size_t map_bytes_ = 0;
    std::string error_;
};

}  // namespace bnn
