// Device-resident Llama-3.2-1B weights read from a .cudallm file.
// Counterpart of wasiqnauman/cudallm src/model/weights.h:11-44 (Linear, LayerWeights, ModelConfig,
// Weights). All tensors live in one device allocation; pointers below point into it.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "common/dtype.h"

namespace cudallm {

struct Linear {
    const void* w = nullptr;       // device, row-major [rows][cols] in the stored type
    const void* scales = nullptr;  // device; int8: fp32 [rows]; int4: fp16 [rows][cols/128]; bf16: null
    int rows = 0, cols = 0;
    WeightType wtype = WeightType::BF16;
};

struct LayerWeights {
    const float* attn_norm = nullptr;
    Linear wqkv;  // [q(2048) | k(512) | v(512)] x 2048
    Linear wo;
    const float* ffn_norm = nullptr;
    Linear w_gate_up;  // [gate(8192) | up(8192)] x 2048
    Linear w_down;
};

struct ModelConfig {
    WeightType wtype = WeightType::BF16;
    int hidden = 0, inter = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, vocab = 0;
    int max_seq_len = 0, group_size = 0;
    float rms_eps = 0.f, rope_theta = 0.f;
};

// Llama-3.2-1B dimensions. Like the reference loader (weights.cpp:19-29) this engine accepts only
// this architecture; the kernels are specialised for it.
namespace llama1b {
constexpr int kHidden = 2048, kInter = 8192, kLayers = 16, kHeads = 32, kKvHeads = 8, kHeadDim = 64;
constexpr int kVocab = 128256, kInt4Group = 128;
constexpr int kQkvRows = (kHeads + 2 * kKvHeads) * kHeadDim;  // 3072
}  // namespace llama1b

// Host-side result of validating a .cudallm file (no CUDA calls).
struct ParsedFile {
    std::string path;
    ModelConfig config;
    uint64_t data_begin = 0, data_end = 0, total_bytes = 0;
    std::vector<uint64_t> offsets;  // per tensor, file order
};
// Validates header and tensor table; throws IoError / FormatError.
ParsedFile parse_cudallm(const std::string& path);

class Weights {
public:
    // Uploads a parsed file to the current device. Throws IoError / CudaError.
    explicit Weights(const ParsedFile& file);
    ~Weights();
    Weights(const Weights&) = delete;
    Weights& operator=(const Weights&) = delete;

    const ModelConfig& config() const { return config_; }
    uint64_t total_tensor_bytes() const { return total_bytes_; }  // sum of nbytes, each tensor once

    const float* rope_inv_freq = nullptr;
    const float* final_norm = nullptr;
    Linear tok_embeddings;  // tied with the lm_head
    std::vector<LayerWeights> layers;

private:
    ModelConfig config_{};
    void* base_ = nullptr;
    uint64_t total_bytes_ = 0;
};

}  // namespace cudallm
