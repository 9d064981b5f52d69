// cw_gguf.h -- GGUF v3 reader for the model loader (chat-wgpu
// src/loader/gguf.rs:65-208): header, metadata, tensor infos, aligned data
// section.  The file is memory-mapped; tensor bytes are handed to the loader
// without dequantisation (Q4_0 stays Q4_0 all the way into HBM).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace cw {

enum GgmlType : uint32_t {
    GGML_F32 = 0,
    GGML_F16 = 1,
    GGML_Q4_0 = 2,
    GGML_Q4_1 = 3,
    GGML_Q8_0 = 8,
    GGML_Q4_K = 12,
    GGML_Q5_K = 13,
    GGML_Q6_K = 14,
    GGML_BF16 = 30,
};

const char* ggml_type_name(uint32_t t);
// Bytes of one row of `n` elements, 0 if the type is unknown or n is ragged.
size_t ggml_row_bytes(uint32_t type, size_t n);

struct GgufMeta {
    enum Kind { U, F, S, OTHER } kind = OTHER;
    uint64_t u = 0;
    double f = 0;
    std::string s;
};

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;  // ne[0] = innermost
    uint64_t n_elems = 0;
    uint64_t offset = 0;         // within the data section
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
};

class GgufFile {
public:
    ~GgufFile();
    // Returns a cw_status; on failure `err` says why.
    int open(const std::string& path, std::string& err);

    const GgufMeta* meta(const std::string& key) const;
    // gguf.rs:165-186 accessors: numeric metadata as u32 / f32 (0 if absent).
    uint32_t meta_u32(const std::string& key, uint32_t dflt = 0) const;
    float meta_f32(const std::string& key, float dflt = 0.f) const;
    std::string meta_str(const std::string& key) const;
    const GgufTensor* tensor(const std::string& name) const;
    bool has(const std::string& name) const { return tensor(name) != nullptr; }

    std::vector<GgufTensor> tensors;
    size_t data_bytes = 0;  // size of the data section

private:
    std::unordered_map<std::string, GgufMeta> meta_;
    std::unordered_map<std::string, size_t> index_;
    void* map_ = nullptr;
    size_t map_len_ = 0;
};

}  // namespace cw
