// Safetensors + config.json reader for the engine (host side, no CUDA).
//
// Same file contract as the reference loader (metal_infrence_engine/src/cpu_inference.rs:58-96):
// an 8-byte little-endian header length, a JSON header mapping tensor names to
// {dtype, shape, data_offsets}, then the data section; config.json beside the file supplies the
// ten Config fields (cpu_inference.rs:21-33). Unlike the reference, which panics, every problem is
// reported as an error code with a message, and the tensor set, dtypes, shapes and bounds are all
// checked up front against the geometry the kernels support.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace qw {

struct ModelConfig {
    uint64_t hidden = 0, inter = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
    float eps = 0.f, theta = 0.f;
    uint32_t eos = 0;
};

struct TensorView {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte offsets into the data section
};

class ModelFile {
public:
    ~ModelFile();
    // returns 0 or a QW_ERR_* code; `msg` receives the reason
    int open(const std::string& path, std::string& msg);
    const ModelConfig& config() const { return cfg_; }
    // pointer to a tensor's bytes (after validate(), every tensor the engine reads is present)
    const uint8_t* data(const std::string& name) const;
    const TensorView* find(const std::string& name) const;
    // tests/mbu.rs:19-30: all tensors except the embedding table, plus one bf16 embedding row
    uint64_t weight_bytes_per_token() const;
    const std::unordered_map<std::string, TensorView>& tensors() const { return tensors_; }

private:
    int validate(std::string& msg);
    void* map_ = nullptr;
    size_t map_len_ = 0;
    const uint8_t* data_ = nullptr;
    ModelConfig cfg_;
    std::unordered_map<std::string, TensorView> tensors_;
};

// geometry limits of the decode kernel; returns 0 or QW_ERR_UNSUPPORTED with a message
int check_supported(const ModelConfig& c, std::string& msg);

}  // namespace qw
