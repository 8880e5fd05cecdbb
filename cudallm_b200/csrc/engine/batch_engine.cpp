#include "engine/batch_engine.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "common/check.h"
#include "common/device.h"
#include "kernels/batch.h"
#include "kernels/batch_ops.h"
#include "kernels/kernels.h"

namespace cudallm {

namespace {

template <typename T>
void alloc_zero(T** p, size_t count) {
    CLLM_CUDA(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
    CLLM_CUDA(cudaMemset(*p, 0, count * sizeof(T)));
}

// The attention grid of a captured step covers whole groups of this many 64-token tiles, so a graph is
// captured again only when the longest context crosses a group boundary (every 256 tokens); tiles past a
// row's context return at once.
constexpr int kTileGroup = 4;

}  // namespace

BatchEngine::BatchEngine(const std::string& path, const BatchOptions& opts) : opts_(opts) {
    const ParsedFile file = parse_cudallm(path);
    if (opts_.n_seq < 1 || opts_.n_seq > kBatchMax) throw ArgError("n_seq must be 1..64");
    if (opts_.max_seq_len < 0 || opts_.max_seq_len % 128 != 0) {
        throw ArgError("max_seq_len must be 0 or a positive multiple of 128");
    }
    if (opts_.max_seq_len > file.config.max_seq_len) throw ArgError("max_seq_len exceeds the file's max_seq_len");
    if (opts_.kv != KvType::F16 && opts_.kv != KvType::BF16) throw ArgError("kv_dtype must be 0 (fp16) or 1 (bf16)");
    if (file.config.wtype != WeightType::BF16 && file.config.wtype != WeightType::INT4) {
        throw ArgError(std::string("batched decode supports bf16 and int4 weights; the file holds ") +
                       to_string(file.config.wtype));
    }
    if (opts_.device >= 0) {
        int n = 0;
        CLLM_CUDA(cudaGetDeviceCount(&n));
        if (opts_.device >= n) throw ArgError("device ordinal out of range");
        device_ = opts_.device;
    } else {
        CLLM_CUDA(cudaGetDevice(&device_));
    }
    if (opts_.attn_mode < 0 || opts_.attn_mode > 2) throw ArgError("attention mode must be 0, 1 or 2");
    ext_kv_ = opts_.ext_k_cache != nullptr || opts_.ext_v_cache != nullptr;
    if (ext_kv_ && (opts_.ext_k_cache == nullptr || opts_.ext_v_cache == nullptr || opts_.n_seq != kBatchMax)) {
        throw ArgError("a prefill engine needs both external caches and n_seq 64");
    }
    DeviceGuard guard(device_);
    weights_ = std::make_unique<Weights>(file);
    const ModelConfig& c = weights_->config();
    max_seq_ = opts_.max_seq_len ? opts_.max_seq_len : c.max_seq_len;
    host_pos_.assign(opts_.n_seq, 0);
    try {
        CLLM_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        int sms = 0;
        CLLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_));
        const int H = c.hidden, I = c.inter, V = c.vocab, NH = c.n_heads, NKV = c.n_kv_heads, D = c.head_dim;
        const int QKV = (NH + 2 * NKV) * D;
        CLLM_CHECK(H % kGemmTileRows == 0 && H / kGemmTileRows <= 16 && I % (kGemmTileRows / 2) == 0 &&
                       QKV % kGemmTileRows == 0 && D == 64 && NH * D == H,
                   "batched decode: unsupported model shape");
        // One streaming CTA per (KV head, sequence) once that fills the SMs; fewer sequences split their
        // contexts over more CTAs.
        attn_stream_ = ext_kv_ || opts_.attn_mode == 1 || (opts_.attn_mode == 0 && opts_.n_seq * NKV >= sms);
        int4_ = c.wtype == WeightType::INT4;
        CLLM_CHECK(!int4_ || c.group_size == 128, "batched decode: int4 needs 128-column scale groups");
        auto pick = [&](int n, int k) { return int4_ ? gemm_pick_ksplit_int4(n, k) : gemm_pick_ksplit(n, k); };
        ks_qkv_ = pick(QKV, H);
        ks_wo_ = pick(H, NH * D);
        ks_gu_ = pick(2 * I, H);
        ks_down_ = pick(H, I);
        lm_tiles_ = (V + kGemmTileRows - 1) / kGemmTileRows;
        const size_t B = kBatchMax;
        alloc_zero(&x_, B * H);
        alloc_zero(reinterpret_cast<__nv_bfloat16**>(&pa_), 2 * B * H);
        alloc_zero(reinterpret_cast<__nv_bfloat16**>(&pb_), 2 * B * H);
        alloc_zero(reinterpret_cast<__nv_bfloat16**>(&act_), 2 * B * I);
        alloc_zero(&ssq_, static_cast<size_t>(16) * B);
        alloc_zero(&qkv_, B * QKV);
        alloc_zero(&logits_, B * V);
        alloc_zero(&am_v_, B * lm_tiles_);
        alloc_zero(&am_i_, B * lm_tiles_);
        if (ext_kv_) {
            k_cache_ = opts_.ext_k_cache;
            v_cache_ = opts_.ext_v_cache;
        } else {
            const size_t cache_elems = static_cast<size_t>(opts_.n_seq) * c.n_layers * NKV * max_seq_ * D;
            CLLM_CUDA(cudaMalloc(&k_cache_, cache_elems * 2));
            CLLM_CUDA(cudaMalloc(&v_cache_, cache_elems * 2));
            CLLM_CUDA(cudaMemset(k_cache_, 0, cache_elems * 2));
            CLLM_CUDA(cudaMemset(v_cache_, 0, cache_elems * 2));
        }
        alloc_zero(&tok_save_, static_cast<size_t>(kBatchMax) + 1);
        alloc_zero(&last_logits_, static_cast<size_t>(V));
        if (!attn_stream_) {
            const size_t slots = static_cast<size_t>(max_seq_ / kAttnTile);
            alloc_zero(&att_o_, B * NH * slots * D);
            alloc_zero(&att_ml_, B * NH * slots * 2);
        }
        alloc_zero(&tok_in_, B);
        alloc_zero(&tok_, B);
        alloc_zero(&dpos_, B);
        alloc_zero(&err_, 1);
        CLLM_CUDA(cudaMemset(tok_in_, 0xff, B * sizeof(int)));  // -1: feed the previous argmax
        // The gate/up matrices are re-laid out in place so that each 128-row GEMM tile holds 64 gate rows and
        // the 64 matching up rows (the SwiGLU epilogue needs both); int4 codes are also re-packed for the
        // GEMM's converters (interleave_int4_codes). This engine owns its copy of the weights.
        {
            const size_t gu_bytes = static_cast<size_t>(2) * I * row_bytes(c.wtype, H);
            void* tmp = nullptr;
            CLLM_CUDA(cudaMalloc(&tmp, gu_bytes));
            auto relayout = [&](const void* p, int row_b) {
                void* w = const_cast<void*>(p);
                interleave_gate_up_rows(w, tmp, I, row_b, stream_);
                CLLM_CUDA(cudaMemcpyAsync(w, tmp, static_cast<size_t>(2) * I * row_b, cudaMemcpyDeviceToDevice, stream_));
            };
            auto repack = [&](const Linear& L) {
                interleave_int4_codes(const_cast<void*>(L.w), static_cast<size_t>(L.rows) * L.cols / 2, stream_);
            };
            for (const LayerWeights& L : weights_->layers) {
                relayout(L.w_gate_up.w, static_cast<int>(row_bytes(c.wtype, H)));
                if (int4_) {
                    relayout(L.w_gate_up.scales, H / 128 * 2);
                    repack(L.wqkv);
                    repack(L.wo);
                    repack(L.w_gate_up);
                    repack(L.w_down);
                }
            }
            if (int4_) repack(weights_->tok_embeddings);
            CLLM_CUDA(cudaStreamSynchronize(stream_));
            CLLM_CUDA(cudaFree(tmp));
        }
        CLLM_CUDA(cudaDeviceSynchronize());
    } catch (...) {
        free_all();
        throw;
    }
}

void BatchEngine::free_all() noexcept {
    auto report = [](cudaError_t err, const char* what) {
        if (err != cudaSuccess) std::fprintf(stderr, "cudallm: %s failed in ~BatchEngine: %s\n", what, cudaGetErrorString(err));
    };
    if (graph_exec_) report(cudaGraphExecDestroy(graph_exec_), "cudaGraphExecDestroy");
    if (graph_) report(cudaGraphDestroy(graph_), "cudaGraphDestroy");
    graph_exec_ = nullptr;
    graph_ = nullptr;
    void* bufs[] = {x_,      pa_,   pb_,   act_,   ssq_,      qkv_,         logits_, am_v_, am_i_,
                    att_o_,  att_ml_, tok_in_, tok_, dpos_, err_, tok_save_, last_logits_};
    for (void* b : bufs) {
        if (b) report(cudaFree(b), "cudaFree");
    }
    if (!ext_kv_) {
        if (k_cache_) report(cudaFree(k_cache_), "cudaFree");
        if (v_cache_) report(cudaFree(v_cache_), "cudaFree");
    }
    tok_save_ = nullptr;
    last_logits_ = nullptr;
    x_ = ssq_ = qkv_ = logits_ = am_v_ = att_o_ = att_ml_ = nullptr;
    pa_ = pb_ = act_ = k_cache_ = v_cache_ = nullptr;
    am_i_ = tok_in_ = tok_ = dpos_ = nullptr;
    err_ = nullptr;
    if (stream_) report(cudaStreamDestroy(stream_), "cudaStreamDestroy");
    stream_ = nullptr;
}

BatchEngine::~BatchEngine() {
    try {
        DeviceGuard guard(device_);
        if (stream_) cudaStreamSynchronize(stream_);
        free_all();
        weights_.reset();
    } catch (const std::exception& ex) {
        std::fprintf(stderr, "cudallm: exception in ~BatchEngine: %s\n", ex.what());
    } catch (...) {
        std::fprintf(stderr, "cudallm: unknown exception in ~BatchEngine\n");
    }
}

void BatchEngine::set_knob(const std::string& name, long long value) {
    const ModelConfig& c = config();
    const int unit = int4_ ? 128 : 64;  // int4 K splits fall on 128-column scale groups
    auto in = [&](long long lo, long long hi) {
        if (value < lo || value > hi) {
            throw ArgError("knob " + name + " must be in [" + std::to_string(lo) + ", " + std::to_string(hi) + "]");
        }
    };
    if (name == "pdl") {
        in(0, 1);
        opts_.pdl = value != 0;
    } else if (name == "ksplit_qkv") {
        in(1, std::min(16, c.hidden / unit));
        ks_qkv_ = static_cast<int>(value);
    } else if (name == "ksplit_wo") {
        in(1, std::min(16, c.n_heads * c.head_dim / unit));
        ks_wo_ = static_cast<int>(value);
    } else if (name == "ksplit_gate_up") {
        in(1, std::min(16, c.hidden / unit));
        ks_gu_ = static_cast<int>(value);
    } else if (name == "ksplit_down") {
        in(1, std::min(16, c.inter / unit));
        ks_down_ = static_cast<int>(value);
    } else {
        throw ArgError("unknown knob '" + name + "' (pdl, ksplit_qkv, ksplit_wo, ksplit_gate_up, ksplit_down)");
    }
    // The captured step holds the old launch configuration: capture again at the next step.
    synchronize();
    DeviceGuard guard(device_);
    if (graph_exec_) CLLM_CUDA(cudaGraphExecDestroy(graph_exec_));
    if (graph_) CLLM_CUDA(cudaGraphDestroy(graph_));
    graph_exec_ = nullptr;
    graph_ = nullptr;
}

int BatchEngine::knob(const std::string& name) const {
    if (name == "pdl") return opts_.pdl ? 1 : 0;
    if (name == "ksplit_qkv") return ks_qkv_;
    if (name == "ksplit_wo") return ks_wo_;
    if (name == "ksplit_gate_up") return ks_gu_;
    if (name == "ksplit_down") return ks_down_;
    if (name == "attn_stream") return attn_stream_ ? 1 : 0;
    throw ArgError("unknown knob '" + name + "'");
}

int BatchEngine::pos(int seq) const {
    if (seq < 0 || seq >= opts_.n_seq) throw ArgError("pos: sequence index out of range");
    return host_pos_[seq];
}

void BatchEngine::synchronize() {
    DeviceGuard guard(device_);
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    unsigned err = 0;
    CLLM_CUDA(cudaMemcpy(&err, err_, sizeof(err), cudaMemcpyDeviceToHost));
    if (err != 0) {
        CLLM_CUDA(cudaMemset(err_, 0, sizeof(unsigned)));
        throw StateError("device: a bounded wait in the batched step gave up (flags " + std::to_string(err) +
                         "); the step's results are invalid");
    }
}

void BatchEngine::reset(int seq) {
    if (seq < -1 || seq >= opts_.n_seq) throw ArgError("reset: sequence index out of range");
    synchronize();
    DeviceGuard guard(device_);
    if (seq < 0) {
        CLLM_CUDA(cudaMemsetAsync(dpos_, 0, sizeof(int) * kBatchMax, stream_));
        std::fill(host_pos_.begin(), host_pos_.end(), 0);
    } else {
        CLLM_CUDA(cudaMemsetAsync(dpos_ + seq, 0, sizeof(int), stream_));
        host_pos_[seq] = 0;
    }
    CLLM_CUDA(cudaStreamSynchronize(stream_));
}

// Per row, the operation sequence of wasiqnauman/cudallm src/engine/engine.cpp:181-237 (RMSNorm, QKV,
// RoPE + KV write, attention, o_proj + residual, RMSNorm, gate/up + SwiGLU, down + residual; final
// RMSNorm, tied lm_head, argmax) as five launches per layer: each GEMM applies the RMSNorm of its input
// (statistics from the epilogue that produced it, gain folded into the activation planes) and fuses the
// operations that follow it into its epilogue.
template <typename KV>
void BatchEngine::enqueue_layers(int tiles) {
    const ModelConfig& c = config();
    const Weights& W = *weights_;
    const int B = opts_.n_seq, H = c.hidden, I = c.inter, V = c.vocab, NH = c.n_heads, NKV = c.n_kv_heads, D = c.head_dim;
    const int QKV = (NH + 2 * NKV) * D;
    const size_t layer_elems = static_cast<size_t>(NKV) * max_seq_ * D;
    // A prefill step points every row at sequence pf_seq_'s cache (stride 0); a decode step gives row b
    // sequence b's cache.
    const bool one_seq = pf_seq_ >= 0;
    const size_t seq_stride = one_seq ? 0 : layer_elems * c.n_layers;
    KV* kc = static_cast<KV*>(k_cache_) + (one_seq ? static_cast<size_t>(pf_seq_) * layer_elems * c.n_layers : 0);
    KV* vc = static_cast<KV*>(v_cache_) + (one_seq ? static_cast<size_t>(pf_seq_) * layer_elems * c.n_layers : 0);
    auto* pa = static_cast<__nv_bfloat16*>(pa_);
    auto* pb = static_cast<__nv_bfloat16*>(pb_);
    auto* act = static_cast<__nv_bfloat16*>(act_);
    auto gemm = [&](const Linear& L, int n, int k, const __nv_bfloat16* x, int ks, const GemmEpi& epi) {
        if (int4_) {
            launch_gemm_int4(static_cast<const uint8_t*>(L.w), static_cast<const __half*>(L.scales), n, k, x, opts_.n_seq, ks, epi,
                             err_, stream_, opts_.pdl);
        } else {
            launch_gemm(static_cast<const __nv_bfloat16*>(L.w), n, k, x, opts_.n_seq, ks, epi, err_, stream_, opts_.pdl);
        }
    };
    const bool pdl = opts_.pdl;
    const bool kv_bf16 = opts_.kv == KvType::BF16;
    cudaStream_t s = stream_;
    const int tiles_h = H / kGemmTileRows;
    // x, planes of x * attn_norm[0] and its statistics (one partial).
    launch_embed_rows(W.tok_embeddings.w, int4_ ? static_cast<const __half*>(W.tok_embeddings.scales) : nullptr, tok_in_, tok_,
                      W.layers[0].attn_norm, x_, pa, ssq_, B, H, s, pdl);
    int ssq_count = 1;
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& L = W.layers[l];
        KV* kl = kc + l * layer_elems;
        KV* vl = vc + l * layer_elems;
        GemmEpi q;
        q.kind = GemmEpilogue::QKV_ROPE;
        q.ssq_in = ssq_;
        q.ssq_count = ssq_count;
        q.norm_n = H;
        q.eps = c.rms_eps;
        q.q_out = qkv_;
        q.inv_freq = W.rope_inv_freq;
        q.k_cache = kl;
        q.v_cache = vl;
        q.seq_stride = seq_stride;
        q.pos = dpos_;
        q.nh = NH;
        q.nkv = NKV;
        q.max_seq = max_seq_;
        q.kv_bf16 = kv_bf16;
        gemm(L.wqkv, QKV, H, pa, ks_qkv_, q);
        if (attn_stream_) {
            launch_attention_rows_stream<KV>(qkv_, kl, vl, seq_stride, dpos_, pb, B, NH, NKV, max_seq_, err_, s, pdl, one_seq);
        } else {
            launch_attention_rows<KV>(qkv_, kl, vl, seq_stride, dpos_, tiles * kAttnTile, att_o_, att_ml_, pb, B, NH, NKV,
                                      max_seq_, s, pdl);
        }
        GemmEpi o;
        o.kind = GemmEpilogue::ADD;
        o.y = x_;
        o.planes = pa;
        o.gain = L.ffn_norm;
        o.ssq_out = ssq_;
        gemm(L.wo, H, NH * D, pb, ks_wo_, o);
        GemmEpi g;
        g.kind = GemmEpilogue::SWIGLU;
        g.ssq_in = ssq_;
        g.ssq_count = tiles_h;
        g.norm_n = H;
        g.eps = c.rms_eps;
        g.planes = act;
        gemm(L.w_gate_up, 2 * I, H, pa, ks_gu_, g);
        GemmEpi d;
        d.kind = GemmEpilogue::ADD;
        d.y = x_;
        d.planes = pa;
        d.gain = l + 1 < c.n_layers ? W.layers[l + 1].attn_norm : W.final_norm;
        d.ssq_out = ssq_;
        gemm(L.w_down, H, I, act, ks_down_, d);
        ssq_count = tiles_h;
    }
    if (pf_skip_logits_) return;  // a prefill chunk that is not the last needs no logits
    GemmEpi lm;
    lm.kind = GemmEpilogue::LOGITS;
    lm.ssq_in = ssq_;
    lm.ssq_count = ssq_count;
    lm.norm_n = H;
    lm.eps = c.rms_eps;
    lm.y = logits_;
    lm.am_v = am_v_;
    lm.am_i = am_i_;
    gemm(W.tok_embeddings, V, H, pa, 1, lm);
    launch_argmax_tiles(am_v_, am_i_, lm_tiles_, tok_, dpos_, B, s, pdl);
}

void BatchEngine::enqueue_step(int tiles) {
    if (opts_.kv == KvType::F16) {
        enqueue_layers<__half>(tiles);
    } else {
        enqueue_layers<__nv_bfloat16>(tiles);
    }
}

void BatchEngine::set_position(int seq, int pos) {
    CLLM_REQUIRE(seq >= 0 && seq < opts_.n_seq && pos >= 0 && pos <= max_seq_, "set_position: out of range");
    synchronize();
    DeviceGuard guard(device_);
    CLLM_CUDA(cudaMemcpy(dpos_ + seq, &pos, sizeof(int), cudaMemcpyHostToDevice));
    host_pos_[seq] = pos;
}

void BatchEngine::prefill(int seq, const int* tokens, int n, float* logits_out, int* next_out) {
    CLLM_REQUIRE(seq >= 0 && seq < (ext_kv_ ? 1 : opts_.n_seq), "prefill: sequence index out of range");
    CLLM_REQUIRE(tokens != nullptr && n >= 1, "prefill: need at least one token");
    CLLM_REQUIRE(opts_.n_seq == kBatchMax, "prefill: needs an engine of 64 rows");
    const int start = host_pos_[seq];
    if (static_cast<long long>(start) + n > max_seq_) throw StateError("prefill: the tokens do not fit in max_seq_len");
    for (int i = 0; i < n; ++i) CLLM_REQUIRE(tokens[i] >= 0 && tokens[i] < config().vocab, "prefill: token out of range");
    synchronize();
    DeviceGuard guard(device_);
    const int B = kBatchMax;
    // The rows' previous argmax (device state of every sequence) is kept aside; positions are restored from
    // the host mirror afterwards.
    CLLM_CUDA(cudaMemcpyAsync(tok_save_, tok_, sizeof(int) * B, cudaMemcpyDeviceToDevice, stream_));
    pf_host_.resize(2 * B);
    int last_row = 0;
    pf_seq_ = seq;
    try {
        for (int i0 = 0; i0 < n; i0 += B) {
            const int m = std::min(B, n - i0);
            // Row b < m: token i0+b at position start+i0+b. Rows past m repeat the last one (same token and
            // position, so they write the same cache values to the same slot).
            for (int b = 0; b < B; ++b) {
                const int i = std::min(b, m - 1);
                pf_host_[b] = tokens[i0 + i];
                pf_host_[B + b] = start + i0 + i;
            }
            CLLM_CUDA(cudaMemcpyAsync(tok_in_, pf_host_.data(), sizeof(int) * B, cudaMemcpyHostToDevice, stream_));
            CLLM_CUDA(cudaMemcpyAsync(dpos_, pf_host_.data() + B, sizeof(int) * B, cudaMemcpyHostToDevice, stream_));
            pf_skip_logits_ = i0 + m < n;
            enqueue_step(max_seq_ / kAttnTile);
            last_row = m - 1;
        }
    } catch (...) {
        pf_seq_ = -1;
        pf_skip_logits_ = false;
        throw;
    }
    pf_seq_ = -1;
    pf_skip_logits_ = false;
    const int V = config().vocab;
    CLLM_CUDA(cudaMemcpyAsync(last_logits_, logits_ + static_cast<size_t>(last_row) * V, sizeof(float) * V,
                              cudaMemcpyDeviceToDevice, stream_));
    CLLM_CUDA(cudaMemcpyAsync(tok_save_ + B, tok_ + last_row, sizeof(int), cudaMemcpyDeviceToDevice, stream_));
    CLLM_CUDA(cudaMemcpyAsync(tok_save_ + seq, tok_ + last_row, sizeof(int), cudaMemcpyDeviceToDevice, stream_));
    CLLM_CUDA(cudaMemcpyAsync(tok_, tok_save_, sizeof(int) * B, cudaMemcpyDeviceToDevice, stream_));
    host_pos_[seq] = start + n;
    std::vector<int> pos_now(B, 0);
    for (int b = 0; b < opts_.n_seq; ++b) pos_now[b] = host_pos_[b];
    CLLM_CUDA(cudaMemcpyAsync(dpos_, pos_now.data(), sizeof(int) * B, cudaMemcpyHostToDevice, stream_));
    CLLM_CUDA(cudaMemsetAsync(tok_in_, 0xff, sizeof(int) * B, stream_));  // the next step feeds argmaxes
    tok_in_fed_ = false;
    if (logits_out != nullptr) {
        CLLM_CUDA(cudaMemcpyAsync(logits_out, last_logits_, sizeof(float) * V, cudaMemcpyDeviceToHost, stream_));
    }
    int next = 0;
    CLLM_CUDA(cudaMemcpyAsync(&next, tok_save_ + B, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    synchronize();
    if (next_out != nullptr) *next_out = next;
}

void BatchEngine::step(const int* tokens, int* next_out, float* logits_out) {
    if (ext_kv_) throw StateError("step: a prefill engine only runs prefill");
    const int B = opts_.n_seq;
    int longest = 0;
    for (int b = 0; b < B; ++b) {
        if (host_pos_[b] >= max_seq_) {
            throw StateError("step: sequence " + std::to_string(b) + " is full (pos == max_seq_len); reset it");
        }
        longest = std::max(longest, host_pos_[b] + 1);
        if (tokens && (tokens[b] < -1 || tokens[b] >= config().vocab)) throw ArgError("step: token out of range");
    }
    DeviceGuard guard(device_);
    // The caller's tokens go to the device through the driver's staging copy (the host array may be reused
    // as soon as this returns); without tokens every row feeds its previous argmax.
    if (tokens) {
        CLLM_CUDA(cudaMemcpyAsync(tok_in_, tokens, sizeof(int) * B, cudaMemcpyHostToDevice, stream_));
        tok_in_fed_ = true;
    } else if (tok_in_fed_) {
        CLLM_CUDA(cudaMemsetAsync(tok_in_, 0xff, sizeof(int) * B, stream_));
        tok_in_fed_ = false;
    }
    // The split attention's grid covers the longest context (rounded up to a tile group); the streaming
    // kernel reads each row's context length on the device, so its graph never needs re-capturing.
    const int max_tiles = max_seq_ / kAttnTile;
    const int tiles = attn_stream_ ? max_tiles
                                   : std::min(max_tiles, (longest + kAttnTile * kTileGroup - 1) / (kAttnTile * kTileGroup) *
                                                             kTileGroup);
    if (opts_.cuda_graph) {
        if (!graph_exec_ || graph_tiles_ != tiles) {
            cudaGraph_t g = nullptr;
            CLLM_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            try {
                enqueue_step(tiles);
            } catch (...) {
                cudaGraph_t broken = nullptr;
                cudaStreamEndCapture(stream_, &broken);
                if (broken) cudaGraphDestroy(broken);
                throw;
            }
            CLLM_CUDA(cudaStreamEndCapture(stream_, &g));
            bool updated = false;
            if (graph_exec_) {
                cudaGraphExecUpdateResultInfo info{};
                updated = cudaGraphExecUpdate(graph_exec_, g, &info) == cudaSuccess;
                if (!updated) {
                    cudaGetLastError();  // clear the failed update's error
                    CLLM_CUDA(cudaGraphExecDestroy(graph_exec_));
                    graph_exec_ = nullptr;
                }
            }
            if (!updated) CLLM_CUDA(cudaGraphInstantiate(&graph_exec_, g, 0));
            if (graph_) CLLM_CUDA(cudaGraphDestroy(graph_));
            graph_ = g;
            graph_tiles_ = tiles;
        }
        CLLM_CUDA(cudaGraphLaunch(graph_exec_, stream_));
    } else {
        enqueue_step(tiles);
    }
    for (int b = 0; b < B; ++b) host_pos_[b] += 1;
    if (!next_out && !logits_out) return;
    if (logits_out) {
        CLLM_CUDA(cudaMemcpyAsync(logits_out, logits_, sizeof(float) * B * config().vocab, cudaMemcpyDeviceToHost, stream_));
    }
    if (next_out) CLLM_CUDA(cudaMemcpyAsync(next_out, tok_, sizeof(int) * B, cudaMemcpyDeviceToHost, stream_));
    synchronize();
}

}  // namespace cudallm
