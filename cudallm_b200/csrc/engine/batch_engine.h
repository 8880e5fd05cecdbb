// Batched decode engine: up to 64 independent sequences decoded together, one token each per step, on
// one GPU. No counterpart in wasiqnauman/cudallm (its engine, src/engine/engine.h:15-65, holds one
// sequence); each row of the batch follows that engine's per-token operation sequence
// (src/engine/engine.cpp:181-237) on its own token, position and KV cache, so a row's logits match what
// the batch-1 engine computes for that sequence up to fp32 summation order. The weight matvecs become
// GEMMs on the tcgen05 tensor cores (every weight byte is read once per step for the whole batch);
// Weights: bf16, or int4 (dequantised to exact bf16 codes inside the GEMM, group scales applied to fp32
// partial sums). RMSNorm, residual adds, RoPE with the KV-cache write, SwiGLU and the logits' argmax
// partials are fused
// into the GEMM epilogues; attention runs per row. Several GPUs run one engine each on their own
// sequence groups (no collective).
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "common/dtype.h"
#include "kernels/batch.h"
#include "model/weights.h"

namespace cudallm {

struct BatchOptions {
    int n_seq = 64;       // 1..64 sequences
    int max_seq_len = 0;  // 0 = the file header's value, else a positive multiple of 128 not above it
    KvType kv = KvType::F16;
    int device = -1;         // -1 = current device
    bool cuda_graph = true;  // replay the step as a CUDA graph
    bool pdl = true;         // programmatic dependent launch between the step's kernels
    // Attention kernel: 0 = choose by size, 1 = one CTA per (KV head, sequence) streaming the whole
    // context, 2 = split over 64-token tiles and merged by a second kernel (more CTAs for few sequences).
    int attn_mode = 0;
    // Prefill engine of another engine's sequence: with both set (n_seq must be 64), the KV cache is this
    // caller-owned pair ([layers][kv heads][max_seq][64] in the cache type, one sequence) and the engine
    // only runs prefill(0, ...); it allocates no cache of its own.
    void* ext_k_cache = nullptr;
    void* ext_v_cache = nullptr;
};

class BatchEngine {
public:
    BatchEngine(const std::string& path, const BatchOptions& opts);
    ~BatchEngine();
    BatchEngine(const BatchEngine&) = delete;
    BatchEngine& operator=(const BatchEngine&) = delete;

    const ModelConfig& config() const { return weights_->config(); }
    const BatchOptions& options() const { return opts_; }
    uint64_t weight_bytes() const { return weights_->total_tensor_bytes(); }
    int n_seq() const { return opts_.n_seq; }
    int max_seq() const { return max_seq_; }
    int pos(int seq) const;
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // seq in [0, n_seq): that sequence's position back to 0; -1: every sequence.
    void reset(int seq);
    // tokens: host [n_seq], tokens[b] >= 0 is fed to sequence b, -1 feeds b's previous argmax; null = all
    // -1. next_out: host [n_seq] or null; logits_out: host [n_seq][vocab] or null. With both outputs null
    // the call does not synchronise.
    void step(const int* tokens, int* next_out, float* logits_out);
    // Prompt prefill of sequence seq: tokens[0..n) at positions pos(seq) .. pos(seq)+n-1, 64 per batched
    // step. Every row of a step is one position of that sequence (its KV cache at stride 0, position
    // increasing with the row), so the GEMMs compute 64 prompt tokens at once on the tensor cores and row b's
    // attention covers the positions up to its own (causal). Equivalent to feeding the tokens one per step
    // (up to fp32 summation order). Afterwards the sequence's position has advanced by n and its next token
    // is the argmax after tokens[n-1]; next_out (host, or null) gets it and logits_out (host [vocab], or
    // null) that step's logits. The other sequences keep their positions and previous argmax. Synchronises.
    void prefill(int seq, const int* tokens, int n, float* logits_out, int* next_out);
    // Prefill engines: the position their sequence continues from (host mirror and device word).
    void set_position(int seq, int pos);
    // Device copies of the last prefill's final logits row [vocab] and next token (valid until the next call).
    const float* last_logits() const { return last_logits_; }
    const int* last_token() const { return tok_save_ + kBatchMax; }
    // Waits for queued steps and reports a device-side failure (a timed-out wait in a GEMM).
    void synchronize();
    // Validated tuning knobs, by name (ArgError when unknown or out of range): "pdl" (0/1, programmatic
    // dependent launch between the step's kernels), "ksplit_qkv", "ksplit_wo", "ksplit_gate_up",
    // "ksplit_down" (K split = cluster size of that GEMM, 1 .. min(16, k / 64), int4 k / 128). The next step
    // captures its graph again. knob() reads them back, and "attn_stream" (1: streaming attention).
    void set_knob(const std::string& name, long long value);
    int knob(const std::string& name) const;

private:
    template <typename KV>
    void enqueue_layers(int tiles);  // tiles: 64-token attention tiles the grid covers
    void enqueue_step(int tiles);
    void free_all() noexcept;

    std::unique_ptr<Weights> weights_;
    BatchOptions opts_;
    int device_ = 0;
    int max_seq_ = 0;
    std::vector<int> host_pos_;
    cudaStream_t stream_ = nullptr;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
    int graph_tiles_ = 0;  // attention tiles the captured graph covers (split attention only)
    bool attn_stream_ = true;
    bool int4_ = false;  // int4 weights (codes re-packed at creation), else bf16

    // Per-operation K splits (cluster sizes of the GEMMs), chosen to fill the SMs.
    int ks_qkv_ = 1, ks_wo_ = 1, ks_gu_ = 1, ks_down_ = 1;
    int lm_tiles_ = 0;

    float* x_ = nullptr;              // residual stream [64][hidden] fp32
    void* pa_ = nullptr;              // activation planes [2][64][hidden] bf16: RMSNorm inputs (x * gain)
    void* pb_ = nullptr;              // activation planes [2][64][hidden] bf16: attention output
    void* act_ = nullptr;             // activation planes [2][64][inter] bf16: SwiGLU output
    float* ssq_ = nullptr;            // RMSNorm statistics: partial sums of x^2 [<= 256][64]
    float* qkv_ = nullptr;            // [64][qkv rows] (rotated q heads)
    float* logits_ = nullptr;         // [64][vocab]
    float* am_v_ = nullptr;           // per-tile argmax partials of the logits [64][vocab / 128]
    int* am_i_ = nullptr;
    void* k_cache_ = nullptr;         // [seq][layer][kv head][max_seq][64]
    void* v_cache_ = nullptr;
    float* att_o_ = nullptr;          // split attention partials [64][heads][max_seq/64][64]
    float* att_ml_ = nullptr;         // [64][heads][max_seq/64][2]
    int* tok_in_ = nullptr;           // device copy of the step's fed tokens
    int* tok_ = nullptr;              // [64] last argmax per sequence
    int* dpos_ = nullptr;             // [64] position per sequence
    unsigned* err_ = nullptr;         // device error word
    bool tok_in_fed_ = false;         // tok_in_ holds fed tokens (not all -1)
    bool ext_kv_ = false;             // prefill engine over a caller-owned cache (one sequence)
    int pf_seq_ = -1;                 // sequence a prefill step writes (-1: ordinary decode step)
    bool pf_skip_logits_ = false;     // prefill chunk before the last: no lm_head GEMM, no argmax
    int* tok_save_ = nullptr;         // [64] rows' previous argmax kept across a prefill, then [1] its token
    float* last_logits_ = nullptr;    // [vocab] logits after a prefill's last token
    std::vector<int> pf_host_;        // host staging of a prefill step's tokens and positions
};

}  // namespace cudallm
