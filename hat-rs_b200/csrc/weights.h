// The checkpoint: a safetensors file in the layout tools/convert.py writes, plus the
// architecture its __metadata__ names (src/weights.rs).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace hat {

struct TensorInfo {
    std::string dtype;           // "F32" or "I64"
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0; // byte range within the data section
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

// A safetensors container read fully into host memory.
struct SafeTensors {
    std::vector<uint8_t> bytes;
    size_t data_off = 0;
    std::map<std::string, TensorInfo> tensors;
    std::vector<std::string> order;
    std::map<std::string, std::string> meta;
    void open(const std::string& path);  // throws hat::Error(2, ...)
    const float* f32(const std::string& name) const;
    std::vector<int64_t> i64(const std::string& name) const;
};

// Weights::load (src/weights.rs:60-129) and validate (src/weights.rs:133-265).
struct Weights {
    SafeTensors st;
    std::string variant;
    int scale = 0, window = 0, owin = 0, embed = 0, heads = 0, head_dim = 0, mlp_ratio = 0;
    std::vector<int> depths;
    int compressed = 0, squeezed = 0, head_feat = 0;
    float conv_scale = 0.f, img_range = 1.f, mean[3] = {0, 0, 0};
    uint64_t f32_bytes = 0;  // what the upload puts on the device

    void load(const std::string& path);
    // (factor, widened channels) per upsampling block (src/weights.rs:290-305).
    std::vector<std::pair<int, int>> up_blocks() const;
    std::vector<int64_t> shape(const std::string& name) const;
    bool has(const std::string& name) const { return st.tensors.count(name) != 0; }
};

}  // namespace hat
