// s2d_gguf.h -- read-only GGUF v3 container view (mmap), host side.
//
// Parses the same container as crates/fish_s2_core/src/gguf.rs:35-120:
// header, metadata (typed here; the reference stringifies values,
// gguf.rs:396-453), tensor directory, 32-byte aligned data start
// (gguf.rs:371-377) and per-tensor bounds (gguf.rs:343-362).  Tensor payloads
// stay in the page cache until the loader copies them to the device.
#pragma once

#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace s2d {

struct GgufMeta {
    uint32_t type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    bool b = false;
    std::string s;
};

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t rel_offset = 0;
    uint64_t bytes = 0;
    uint64_t elements = 0;
    const uint8_t *data = nullptr;
};

class Gguf {
  public:
    ~Gguf();
    bool open(const std::string &path, std::string *err);
    const GgufTensor *tensor(const std::string &name) const;
    const GgufMeta *meta(const std::string &key) const;
    bool meta_u32(const std::string &key, uint32_t *out, std::string *err) const;
    bool meta_f32(const std::string &key, float *out, std::string *err) const;
    bool meta_bool(const std::string &key, bool *out, std::string *err) const;
    bool meta_str(const std::string &key, std::string *out, std::string *err) const;

    uint32_t version = 0;
    std::vector<GgufTensor> tensors;

  private:
    int fd_ = -1;
    const uint8_t *map_ = nullptr;
    size_t size_ = 0;
    std::unordered_map<std::string, GgufMeta> meta_;
    std::unordered_map<std::string, size_t> index_;
};

// ggml block byte length (gguf.rs:233-258) for the types this library reads.
int64_t ggml_byte_len(uint32_t type, uint64_t elements);

}  // namespace s2d
