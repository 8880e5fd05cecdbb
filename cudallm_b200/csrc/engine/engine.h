// Batch-1 decode engine behind the reference's engine surface (wasiqnauman/cudallm
// src/engine/engine.h:15-32: create from a .cudallm path; step, step_debug, reset, pos).
//
// Two execution paths share the weights, the KV cache and the device-resident (token, position) pair:
//   * persistent (the default fused opt/opt configuration): each token is ONE cooperative launch of the
//     decode-step kernel (engine/decode_step.cu);
//   * per-op (every other option combination, and step_debug of them): a launch plan built once at
//     creation, one record per kernel in the reference's operation order, replayed record by record or
//     captured once as a CUDA graph.
// All device memory of the engine (activations, KV cache, scratch, control words) is one allocation
// carved into aligned regions; the weights are a second one (model/weights.h).
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "common/dtype.h"
#include "engine/decode_step.h"
#include "kernels/kernels.h"
#include "model/weights.h"

namespace cudallm {

class BatchEngine;

enum class MatvecImpl : int { NAIVE = 0, OPT = 1 };
enum class AttnImpl : int { NAIVE = 0, OPT = 1 };
enum class DecodePath : int { AUTO = 0, PERSISTENT = 1, PER_OP = 2 };

// Options of the reference (src/engine/options.h:10-17) plus the additive kv / device / path fields.
struct EngineOptions {
    MatvecImpl matvec = MatvecImpl::OPT;
    AttnImpl attn = AttnImpl::OPT;
    bool fuse = true;
    bool cuda_graph = true;
    int max_seq_len = 0;  // 0 = header value, else a positive multiple of 128 not above it
    int matvec_rpb = 0;   // 0 = default, else 1, 2, 4 or 8
    KvType kv = KvType::F16;
    int device = -1;  // -1 = current device
    DecodePath path = DecodePath::AUTO;
};

// Throws ArgError when an option (or combination) is invalid for weights of type wt.
void validate(const EngineOptions& o, WeightType wt);

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
    // token >= 0 is fed, -1 feeds the previous argmax (already on the device). With both outputs null the
    // call only enqueues work.
    void step(int token, float* logits_out, int* next_token_out);
    // Never graph-replayed; residuals_out: host [(n_layers + 1) * hidden].
    void step_debug(int token, float* residuals_out, float* logits_out, int* next_token_out);
    // Waits for queued work and reports a device-side failure.
    void synchronize();
    // Feeds tokens[0..n) at positions pos() .. pos()+n-1, as n steps would (results equal up to fp32
    // summation order), but 64 tokens per launch sequence: a batched engine (tcgen05 GEMMs, created on first
    // use with its own copy of the weights) writes this engine's KV cache directly. int8 weights have no
    // batched GEMM and step the tokens through the decode path instead. Afterwards pos() has advanced by n;
    // next_token_out / logits_out (host, or null) get the argmax and logits after tokens[n-1], and a step
    // with token -1 continues from that argmax. Synchronises.
    void prefill(const int* tokens, int n, float* logits_out, int* next_token_out);

    // Step tracing of the persistent path (decode_step.h kTraceSlots).
    void set_trace(bool enable);
    int trace_grid() const;
    void read_trace(unsigned long long* out, size_t count);
    // Validated tuning / test knobs of the persistent path, by name (ArgError when unknown or out of
    // range): "wait_limit_ns" (bound of every inter-CTA wait, 1 .. 1e10), "prefetch_tiles" (L2 prefetch
    // distance, 0 .. 1024), "whole_head_max_tiles" (attention form switch, 0 .. max_seq/64),
    // "trace_tile_op" (weight operation whose tiles the trace stamps, 0 .. 64), "stall_op" (test only: the
    // consumers of weight operation k wait for an input that is never written, so the step's waits run out
    // and it fails with StateError; -1 = off, 1 .. 64).
    void set_knob(const std::string& name, long long value);
    // Next-token rule of the persistent step: temperature 0 = greedy argmax (the default); > 0 = sampling
    // from the top_k (1..64; 0 = 64) logits with nucleus top_p (0, 1], drawn from (seed, position).
    void set_sampling(float temperature, int top_k, float top_p, unsigned long long seed);

    // Device state read back with every synchronising step: the fed/argmax token, the position and the
    // error words of the bounded in-kernel waits.
    struct DevState {
        int token;
        int pos;
        unsigned err[2];
    };

private:
    // One kernel launch of the per-op path.
    enum class Op : uint8_t { EMBED, RMSNORM, MATVEC, ROPE, KV_WRITE, ROPE_KV, ATTN, ADD, SILU_MUL, ARGMAX, SNAPSHOT };
    struct PlanStep {
        Op op;
        int layer = -1;              // KV-cache layer (ROPE / KV_WRITE / ROPE_KV / ATTN), residual slot (SNAPSHOT)
        const Linear* w = nullptr;   // MATVEC
        const float* in = nullptr;   // operand read
        float* out = nullptr;        // operand written
        const float* gain = nullptr; // RMSNorm gain (RMSNORM, or fused into MATVEC)
        Epilogue ep = Epilogue::STORE;
    };

    template <typename Fn>
    void for_each_region(Fn&& fn);
    void build_plan();
    template <typename KV>
    void run_plan(float* residuals_out);
    void run_plan_any(float* residuals_out);
    void launch_step_kernel(int token, float* debug_res);
    void collect(float* logits_out, int* next_token_out);
    void check_device_state(const DevState& st);
    void make_step_params();

    std::string path_;
    std::unique_ptr<Weights> weights_;
    std::unique_ptr<BatchEngine> prefiller_;  // made by the first prefill (bf16 / int4 weights)
    EngineOptions opts_;
    bool persistent_ = false;
    int device_ = 0;
    int max_seq_ = 0;
    int host_pos_ = 0;
    cudaStream_t stream_ = nullptr;
    cudaGraphExec_t graph_ = nullptr;
    std::vector<PlanStep> plan_;

    // Regions of the engine's single device allocation (for_each_region lists them).
    void* arena_ = nullptr;
    float* x_ = nullptr;       // residual stream [hidden]
    float* xb_ = nullptr;      // normalised input [hidden] (unfused)
    float* qkv_ = nullptr;     // [q | k | v]
    float* att_ = nullptr;     // attention output [heads * head_dim]
    float* tmp_ = nullptr;     // projection output before the residual add (unfused) [hidden]
    float* gu_ = nullptr;      // gate | up (unfused) [2 * inter]
    float* act_ = nullptr;     // SwiGLU output [inter]
    float* logits_ = nullptr;  // [vocab]
    uint16_t* k_cache_ = nullptr;  // [layers][kv heads][max_seq][head_dim], fp16 or bf16 bits
    uint16_t* v_cache_ = nullptr;
    float* part_o_ = nullptr;   // split-K attention partials [heads][max_seq / 64][head_dim]
    float* part_ml_ = nullptr;  // [heads][max_seq / 64][2]
    float* am_v_ = nullptr;     // argmax partials
    int* am_i_ = nullptr;
    unsigned long long* cand_ = nullptr;  // persistent step, sampling: [argmax slots][64] candidate keys
    DevState* state_ = nullptr;
    unsigned* sync_ = nullptr;  // persistent step: split-attention flags and the lm_head ticket
    float* debug_res_ = nullptr;  // persistent step_debug: residuals [(layers + 1) * hidden]
    unsigned long long* tagged_ = nullptr;  // persistent step: (value, tag) activation words
    size_t tagged_words_ = 0;

    StepParams step_{};
    unsigned step_tag_ = 0;
    unsigned long long* trace_ = nullptr;  // separate allocation, made when tracing is first enabled
    bool trace_on_ = false;
};

}  // namespace cudallm
