// .cudallm loader. Validation rules follow wasiqnauman/cudallm src/model/weights.cpp:99-219 (they are
// part of the file format's contract: fixed tensor sequence, 256-B aligned non-overlapping offsets,
// exact nbytes). The upload is B200-side: the whole data region goes into one device allocation
// through two pinned staging buffers, so file reads overlap host-to-device copies.
#include "model/weights.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "common/check.h"
#include "model/format.h"

namespace cudallm {

namespace {

using namespace llama1b;

constexpr size_t kStageBytes = 64ull << 20;

struct Expected {
    std::string name;
    DType dtype;
    uint32_t rows, cols;
};

uint64_t tensor_nbytes(DType dt, uint64_t rows, uint64_t cols) {
    switch (dt) {
        case DType::F32: return rows * cols * 4;
        case DType::BF16:
        case DType::F16: return rows * cols * 2;
        case DType::I8: return rows * cols;
        case DType::I4X2: return rows * cols / 2;
    }
    throw FormatError("unknown tensor dtype");
}

void push_linear(std::vector<Expected>& v, const std::string& name, WeightType wt, uint32_t rows, uint32_t cols) {
    if (wt == WeightType::BF16) {
        v.push_back({name + ".weight", DType::BF16, rows, cols});
    } else if (wt == WeightType::INT8) {
        v.push_back({name + ".weight", DType::I8, rows, cols});
        v.push_back({name + ".scales", DType::F32, rows, 1});
    } else {
        v.push_back({name + ".weight", DType::I4X2, rows, cols});
        v.push_back({name + ".scales", DType::F16, rows, cols / kInt4Group});
    }
}

// Tensor sequence of the format (python/cudallm/format.py:53-70; 99 entries bf16, 164 quantized).
std::vector<Expected> expected_sequence(WeightType wt) {
    std::vector<Expected> v;
    v.push_back({"rope.inv_freq", DType::F32, kHeadDim / 2, 1});
    push_linear(v, "tok_embeddings", wt, kVocab, kHidden);
    v.push_back({"norm.weight", DType::F32, kHidden, 1});
    for (int i = 0; i < kLayers; ++i) {
        const std::string p = "layers." + std::to_string(i) + ".";
        v.push_back({p + "attn_norm.weight", DType::F32, kHidden, 1});
        push_linear(v, p + "wqkv", wt, kQkvRows, kHidden);
        push_linear(v, p + "wo", wt, kHidden, kHidden);
        v.push_back({p + "ffn_norm.weight", DType::F32, kHidden, 1});
        push_linear(v, p + "w_gate_up", wt, 2 * kInter, kHidden);
        push_linear(v, p + "w_down", wt, kHidden, kInter);
    }
    return v;
}

void check_field(uint64_t got, uint64_t want, const char* field) {
    if (got != want) {
        throw FormatError(std::string("header field ") + field + " = " + std::to_string(got) + ", expected " +
                          std::to_string(want));
    }
}

struct FileCloser {
    void operator()(FILE* f) const {
        if (f) std::fclose(f);
    }
};

void read_at(FILE* f, uint64_t offset, void* dst, size_t n, const std::string& path, const char* what) {
    if (fseeko(f, static_cast<off_t>(offset), SEEK_SET) != 0) throw IoError(path + ": seek failed (" + what + ")");
    if (std::fread(dst, 1, n, f) != n) throw IoError(path + ": short read (" + what + ")");
}

}  // namespace

ParsedFile parse_cudallm(const std::string& path) {
    std::unique_ptr<FILE, FileCloser> f(std::fopen(path.c_str(), "rb"));
    if (!f) throw IoError("cannot open " + path);
    if (fseeko(f.get(), 0, SEEK_END) != 0) throw IoError(path + ": seek failed");
    const uint64_t file_size = static_cast<uint64_t>(ftello(f.get()));

    FileHeader h{};
    if (file_size < sizeof(h)) throw FormatError(path + ": file too small for header");
    read_at(f.get(), 0, &h, sizeof(h), path, "header");
    if (std::memcmp(h.magic, kFileMagic, 4) != 0) throw FormatError(path + ": bad magic");
    check_field(h.version, kFileVersion, "version");
    if (h.weight_dtype != 1 && h.weight_dtype != 3 && h.weight_dtype != 4) {
        throw FormatError("unsupported weight_dtype " + std::to_string(h.weight_dtype));
    }
    const auto wt = static_cast<WeightType>(h.weight_dtype);
    check_field(h.hidden_size, kHidden, "hidden_size");
    check_field(h.intermediate_size, kInter, "intermediate_size");
    check_field(h.n_layers, kLayers, "n_layers");
    check_field(h.n_heads, kHeads, "n_heads");
    check_field(h.n_kv_heads, kKvHeads, "n_kv_heads");
    check_field(h.head_dim, kHeadDim, "head_dim");
    check_field(h.vocab_size, kVocab, "vocab_size");
    if (h.max_seq_len == 0 || h.max_seq_len % 128 != 0) throw FormatError("max_seq_len must be a positive multiple of 128");
    check_field(h.n_tensors, wt == WeightType::BF16 ? 99 : 164, "n_tensors");
    check_field(h.table_offset, sizeof(FileHeader), "table_offset");
    check_field(h.group_size, wt == WeightType::INT4 ? kInt4Group : 0, "group_size");

    const std::vector<Expected> want = expected_sequence(wt);
    CLLM_CHECK(want.size() == h.n_tensors, "internal: tensor sequence length mismatch");
    std::vector<TensorEntry> table(h.n_tensors);
    const uint64_t table_end = h.table_offset + uint64_t(h.n_tensors) * sizeof(TensorEntry);
    if (file_size < table_end) throw FormatError(path + ": file too small for tensor table");
    read_at(f.get(), h.table_offset, table.data(), table.size() * sizeof(TensorEntry), path, "tensor table");

    ParsedFile pf;
    pf.path = path;
    uint64_t prev_end = table_end;
    for (size_t k = 0; k < table.size(); ++k) {
        const TensorEntry& e = table[k];
        const Expected& x = want[k];
        const std::string name(e.name, strnlen(e.name, sizeof(e.name)));
        if (name != x.name) throw FormatError("tensor " + std::to_string(k) + " is '" + name + "', expected '" + x.name + "'");
        if (e.dtype != static_cast<uint32_t>(x.dtype) || e.rows != x.rows || e.cols != x.cols) {
            throw FormatError("tensor '" + name + "' has wrong dtype or shape");
        }
        if (e.offset % kTensorAlign != 0) throw FormatError("tensor '" + name + "' offset not 256-aligned");
        if (e.offset < prev_end) throw FormatError("tensor '" + name + "' offset overlaps previous data");
        if (e.nbytes != tensor_nbytes(x.dtype, x.rows, x.cols)) throw FormatError("tensor '" + name + "' has wrong nbytes");
        prev_end = e.offset + e.nbytes;
        pf.total_bytes += e.nbytes;
        pf.offsets.push_back(e.offset);
    }
    pf.data_begin = table.front().offset;
    pf.data_end = table.back().offset + table.back().nbytes;
    if (file_size < pf.data_end) throw FormatError(path + ": file truncated (data region)");

    ModelConfig& c = pf.config;
    c.wtype = wt;
    c.hidden = kHidden;
    c.inter = kInter;
    c.n_layers = kLayers;
    c.n_heads = kHeads;
    c.n_kv_heads = kKvHeads;
    c.head_dim = kHeadDim;
    c.vocab = kVocab;
    c.max_seq_len = static_cast<int>(h.max_seq_len);
    c.group_size = static_cast<int>(h.group_size);
    c.rms_eps = h.rms_eps;
    c.rope_theta = h.rope_theta;
    return pf;
}

Weights::Weights(const ParsedFile& pfile) {
    const std::string& path = pfile.path;
    config_ = pfile.config;
    total_bytes_ = pfile.total_bytes;
    const WeightType wt = config_.wtype;
    std::unique_ptr<FILE, FileCloser> f(std::fopen(path.c_str(), "rb"));
    if (!f) throw IoError("cannot open " + path);
    const uint64_t data_begin = pfile.data_begin;
    const uint64_t data_end = pfile.data_end;

    // Upload: read chunk k into pinned buffer k%2 while chunk k-1 copies on a private stream.
    const uint64_t span = data_end - data_begin;
    CLLM_CUDA(cudaMalloc(&base_, span));
    void* pinned[2] = {nullptr, nullptr};
    cudaStream_t stream = nullptr;
    cudaEvent_t done[2] = {nullptr, nullptr};
    auto cleanup = [&] {
        if (stream) cudaStreamSynchronize(stream);
        for (int i = 0; i < 2; ++i) {
            if (done[i]) cudaEventDestroy(done[i]);
            if (pinned[i]) cudaFreeHost(pinned[i]);
        }
        if (stream) cudaStreamDestroy(stream);
    };
    try {
        CLLM_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        for (int i = 0; i < 2; ++i) {
            CLLM_CUDA(cudaMallocHost(&pinned[i], kStageBytes));
            CLLM_CUDA(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        if (fseeko(f.get(), static_cast<off_t>(data_begin), SEEK_SET) != 0) throw IoError(path + ": seek failed (data)");
        int k = 0;
        for (uint64_t off = 0; off < span; off += kStageBytes, ++k) {
            const int b = k & 1;
            const size_t n = static_cast<size_t>(std::min<uint64_t>(kStageBytes, span - off));
            if (k >= 2) CLLM_CUDA(cudaEventSynchronize(done[b]));
            if (std::fread(pinned[b], 1, n, f.get()) != n) throw IoError(path + ": short read (data region)");
            CLLM_CUDA(cudaMemcpyAsync(static_cast<char*>(base_) + off, pinned[b], n, cudaMemcpyHostToDevice, stream));
            CLLM_CUDA(cudaEventRecord(done[b], stream));
        }
        CLLM_CUDA(cudaStreamSynchronize(stream));
        cleanup();
    } catch (...) {
        cleanup();
        cudaFree(base_);
        base_ = nullptr;
        throw;
    }

    size_t k = 0;
    auto at = [&](size_t i) -> const void* { return static_cast<const char*>(base_) + (pfile.offsets[i] - data_begin); };
    const bool quant = wt != WeightType::BF16;
    auto linear = [&](int rows, int cols) {
        Linear L;
        L.w = at(k++);
        L.scales = quant ? at(k++) : nullptr;
        L.rows = rows;
        L.cols = cols;
        L.wtype = wt;
        return L;
    };
    rope_inv_freq = static_cast<const float*>(at(k++));
    tok_embeddings = linear(kVocab, kHidden);
    final_norm = static_cast<const float*>(at(k++));
    layers.resize(kLayers);
    for (auto& L : layers) {
        L.attn_norm = static_cast<const float*>(at(k++));
        L.wqkv = linear(kQkvRows, kHidden);
        L.wo = linear(kHidden, kHidden);
        L.ffn_norm = static_cast<const float*>(at(k++));
        L.w_gate_up = linear(2 * kInter, kHidden);
        L.w_down = linear(kHidden, kInter);
    }
    CLLM_CHECK(k == pfile.offsets.size(), "internal: tensor pointer assignment mismatch");
}

Weights::~Weights() {
    if (base_) {
        const cudaError_t err = cudaFree(base_);
        if (err != cudaSuccess) std::fprintf(stderr, "cudallm: cudaFree failed in ~Weights: %s\n", cudaGetErrorString(err));
    }
}

}  // namespace cudallm
