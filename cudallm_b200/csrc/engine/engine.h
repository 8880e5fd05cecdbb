// Batch-1 decode engine. Public surface of wasiqnauman/cudallm src/engine/engine.h:15-32 (create from
// a .cudallm path, step / step_debug / reset / pos), re-designed for B200: the fused opt/opt path
// runs each token as ONE persistent cooperative kernel (engine/decode_step.cu); every other option
// combination runs the reference's per-operation sequence on sm_100a kernels, optionally replayed as
// a CUDA graph. Position and token live on the device, so queued steps need no host round trip.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>

#include "common/dtype.h"
#include "engine/decode_step.h"
#include "kernels/kernels.h"
#include "model/weights.h"

namespace cudallm {

enum class MatvecImpl : int { NAIVE = 0, OPT = 1 };
enum class AttnImpl : int { NAIVE = 0, OPT = 1 };
enum class DecodePath : int { AUTO = 0, PERSISTENT = 1, PER_OP = 2 };

// Options: reference src/engine/options.h:10-17 plus the additive kv / device / path fields.
struct EngineOptions {
    MatvecImpl matvec = MatvecImpl::OPT;
    AttnImpl attn = AttnImpl::OPT;
    bool fuse = true;
    bool cuda_graph = true;
    int max_seq_len = 0;  // 0 = header value, else a multiple of 128 not above it
    int matvec_rpb = 0;   // 0 = default, else 1, 2, 4 or 8
    KvType kv = KvType::F16;
    int device = -1;  // -1 = current device
    DecodePath path = DecodePath::AUTO;
};

void validate(const EngineOptions& o, WeightType wt);  // throws ArgError

class Engine {
public:
    Engine(const std::string& path, const EngineOptions& opts);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    const ModelConfig& config() const { return weights_->config(); }
    const EngineOptions& options() const { return opts_; }
    uint64_t weight_bytes() const { return weights_->total_tensor_bytes(); }
    int max_seq() const { return max_seq_; }
    int pos() const { return host_pos_; }
    bool persistent() const { return persistent_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    void reset();
    // token >= 0: feed it; -1: feed the previous argmax (already on the device). With both outputs
    // null the call only enqueues work.
    void step(int token, float* logits_out, int* next_token_out);
    // Never graph-replayed; residuals_out: [(n_layers+1) * hidden].
    void step_debug(int token, float* residuals_out, float* logits_out, int* next_token_out);
    // Waits for queued work and reports a device-side failure.
    void synchronize();
    // Per-CTA timestamps of the persistent step (see decode_step.h kTraceSlots).
    void set_trace(bool enable);
    int trace_grid() const;
    void read_trace(unsigned long long* out, size_t count);

private:
    struct DevState {
        int token;
        int pos;
        unsigned err[2];
    };
    void enqueue_per_op(bool debug, float* residuals_out);
    void launch_linear(const Linear& L, const float* x, float* y, Epilogue ep, const float* norm_w);
    template <typename KV>
    void enqueue_layers(bool debug, float* residuals_out);
    void enqueue_persistent(int token, float* debug_res);
    void finish_sync(float* logits_out, int* next_token_out);
    void raise_if_device_error(const DevState& st);
    void free_all() noexcept;

    std::unique_ptr<Weights> weights_;
    EngineOptions opts_;
    bool persistent_ = false;
    int device_ = 0;
    int max_seq_ = 0;
    int host_pos_ = 0;
    cudaStream_t stream_ = nullptr;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
    StepParams step_params_{};

    float* x_ = nullptr;
    float* xb_ = nullptr;
    float* qkv_ = nullptr;
    float* att_ = nullptr;
    float* tmp_ = nullptr;
    float* gu_ = nullptr;
    float* act_ = nullptr;
    float* logits_ = nullptr;
    void* k_cache_ = nullptr;
    void* v_cache_ = nullptr;
    float* part_o_ = nullptr;
    float* part_ml_ = nullptr;
    float* am_v_ = nullptr;
    int* am_i_ = nullptr;
    DevState* state_ = nullptr;  // token, pos, error words
    unsigned* sync_ = nullptr;
    float* debug_res_ = nullptr;
    // Persistent step: activations exchanged between CTAs as (value, tag) words; tag of the last launch.
    unsigned long long* tagged_ = nullptr;
    size_t tagged_words_ = 0;
    unsigned step_tag_ = 0;
    unsigned long long* trace_ = nullptr;
    bool trace_on_ = false;
};

}  // namespace cudallm
