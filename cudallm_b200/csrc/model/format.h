// On-disk layout of a .cudallm file. Byte-compatible with wasiqnauman/cudallm
// src/model/cudallm_format.h:12-46 and python/cudallm/format.py:22-26 (the format is shared with
// that project's exporter, so the field order and sizes are fixed by it).
//   header (256 B) | tensor table (n_tensors x 80 B) at table_offset | tensor data, each 256-B aligned
#pragma once

#include <cstddef>
#include <cstdint>

namespace cudallm {

constexpr char kFileMagic[5] = "CLLM";
constexpr uint32_t kFileVersion = 1;
constexpr uint64_t kTensorAlign = 256;

#pragma pack(push, 1)
struct FileHeader {
    char magic[4];
    uint32_t version;
    uint32_t weight_dtype;
    uint32_t hidden_size;
    uint32_t intermediate_size;
    uint32_t n_layers;
    uint32_t n_heads;
    uint32_t n_kv_heads;
    uint32_t head_dim;
    uint32_t vocab_size;
    uint32_t max_seq_len;
    float rms_eps;
    float rope_theta;
    uint32_t group_size;
    uint32_t n_tensors;
    uint32_t reserved0;
    uint64_t table_offset;
    uint8_t zero[184];
};

struct TensorEntry {
    char name[48];
    uint32_t dtype;
    uint32_t rows;
    uint32_t cols;
    uint32_t reserved;
    uint64_t offset;
    uint64_t nbytes;
};
#pragma pack(pop)

static_assert(sizeof(FileHeader) == 256, "FileHeader must be 256 bytes");
static_assert(offsetof(FileHeader, table_offset) == 64, "table_offset must sit at byte 64");
static_assert(sizeof(TensorEntry) == 80, "TensorEntry must be 80 bytes");

}  // namespace cudallm
