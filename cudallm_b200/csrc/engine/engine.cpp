#include "engine/engine.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <string>
#include <type_traits>

#include "common/check.h"
#include "common/device.h"
#include "engine/batch_engine.h"
#include "kernels/batch.h"

namespace cudallm {

void validate(const EngineOptions& o, WeightType wt) {
    // Rules of the reference's option check (src/engine/engine.cpp:10-21), plus the additive fields.
    const bool rpb_ok = o.matvec_rpb == 0 || o.matvec_rpb == 1 || o.matvec_rpb == 2 || o.matvec_rpb == 4 || o.matvec_rpb == 8;
    CLLM_REQUIRE(o.matvec == MatvecImpl::NAIVE || o.matvec == MatvecImpl::OPT, "invalid matvec implementation");
    CLLM_REQUIRE(o.attn == AttnImpl::NAIVE || o.attn == AttnImpl::OPT, "invalid attention implementation");
    CLLM_REQUIRE(o.matvec == MatvecImpl::OPT || wt == WeightType::BF16, "naive matvec requires bf16 weights");
    CLLM_REQUIRE(o.matvec == MatvecImpl::OPT || !o.fuse, "naive matvec requires fuse=false");
    CLLM_REQUIRE(rpb_ok, "matvec_rpb must be one of 0, 1, 2, 4, 8");
    CLLM_REQUIRE(o.max_seq_len >= 0 && o.max_seq_len % 128 == 0, "max_seq_len must be 0 or a positive multiple of 128");
    CLLM_REQUIRE(o.kv == KvType::F16 || o.kv == KvType::BF16, "kv_dtype must be 0 (fp16) or 1 (bf16)");
    CLLM_REQUIRE(o.path != DecodePath::PERSISTENT || (o.fuse && o.matvec == MatvecImpl::OPT && o.attn == AttnImpl::OPT),
                 "the persistent decode path needs fuse=1 and opt matvec/attention");
}

namespace {

constexpr size_t kRegionAlign = 256;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;   // each inter-CTA wait of the persistent step
constexpr unsigned long long kDrainLimitNs = 1000000000ull;  // its final wait for copies still in flight
// Contexts up to this many 64-token tiles attend with one CTA per KV head; longer ones cut each head's
// context into ranges over many CTAs (the split instantiation of the step). The measured cross-over of the
// two forms on B200: ~384 tokens for bf16 / int8 weights, ~512 for int4 (whose step is shorter).
constexpr int kWholeHeadMaxTiles = 6;
constexpr int kWholeHeadMaxTilesInt4 = 8;
// L2 prefetch distance of the persistent weight stream, in tiles (ring stages of up to 16 KiB).
constexpr int kPrefetchTiles = 24;
constexpr int kTraceLmOp = 64;  // weight operation index of the lm_head

int resolve_device(int requested) {
    int dev = 0;
    if (requested < 0) {
        CLLM_CUDA(cudaGetDevice(&dev));
        return dev;
    }
    int n = 0;
    CLLM_CUDA(cudaGetDeviceCount(&n));
    CLLM_REQUIRE(requested < n, "device ordinal out of range");
    return requested;
}

}  // namespace

// Every region of the engine's device allocation, in layout order: fn(pointer member, element count).
template <typename Fn>
void Engine::for_each_region(Fn&& fn) {
    const ModelConfig& c = config();
    const size_t H = c.hidden, I = c.inter, V = c.vocab, NH = c.n_heads, NKV = c.n_kv_heads, D = c.head_dim;
    const size_t QKV = (NH + 2 * NKV) * D, slots = static_cast<size_t>(max_seq_) / kAttnTile;
    const size_t cache = static_cast<size_t>(c.n_layers) * NKV * max_seq_ * D;
    fn(state_, 1);
    fn(sync_, kSyncWords);
    fn(x_, H);
    fn(xb_, H);
    fn(qkv_, QKV);
    fn(att_, NH * D);
    fn(tmp_, H);
    fn(gu_, 2 * I);
    fn(act_, I);
    fn(logits_, V);
    fn(am_v_, kArgmaxBlocks);
    fn(am_i_, kArgmaxBlocks);
    fn(cand_, static_cast<size_t>(kArgmaxBlocks) * kMaxTopK);
    fn(part_o_, NH * slots * D);
    fn(part_ml_, NH * slots * 2);
    fn(debug_res_, (c.n_layers + 1) * H);
    fn(tagged_, tagged_words_);
    fn(k_cache_, cache);
    fn(v_cache_, cache);
}

Engine::Engine(const std::string& path, const EngineOptions& opts) : path_(path), opts_(opts) {
    // File and option errors are reported before any CUDA call.
    const ParsedFile file = parse_cudallm(path);
    validate(opts_, file.config.wtype);
    CLLM_REQUIRE(opts_.max_seq_len <= file.config.max_seq_len, "max_seq_len exceeds the file's max_seq_len");
    device_ = resolve_device(opts_.device);
    DeviceGuard on(device_);
    weights_ = std::make_unique<Weights>(file);
    const ModelConfig& c = config();
    max_seq_ = opts_.max_seq_len ? opts_.max_seq_len : c.max_seq_len;
    persistent_ = opts_.path != DecodePath::PER_OP && opts_.fuse && opts_.matvec == MatvecImpl::OPT &&
                  opts_.attn == AttnImpl::OPT;
    tagged_words_ = static_cast<size_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim + c.n_heads * c.head_dim + 2 * c.hidden +
                    c.inter;
    try {
        CLLM_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        size_t total = 0;
        for_each_region([&](auto*& p, size_t n) {
            total += (n * sizeof(*p) + kRegionAlign - 1) / kRegionAlign * kRegionAlign;
        });
        CLLM_CUDA(cudaMalloc(&arena_, total));
        // Everything starts at zero: position, token, error words, tickets, tags and the KV cache.
        CLLM_CUDA(cudaMemsetAsync(arena_, 0, total, stream_));
        size_t off = 0;
        for_each_region([&](auto*& p, size_t n) {
            p = reinterpret_cast<std::remove_reference_t<decltype(p)>>(static_cast<uint8_t*>(arena_) + off);
            off += (n * sizeof(*p) + kRegionAlign - 1) / kRegionAlign * kRegionAlign;
        });
        CLLM_CUDA(cudaStreamSynchronize(stream_));
        if (persistent_) {
            make_step_params();
        } else {
            build_plan();
        }
    } catch (...) {
        if (arena_) cudaFree(arena_);
        if (stream_) cudaStreamDestroy(stream_);
        throw;
    }
}

Engine::~Engine() {
    // Never throws: failures while releasing are reported on stderr.
    auto warn = [](cudaError_t e, const char* what) {
        if (e != cudaSuccess) std::fprintf(stderr, "cudallm: %s while destroying an engine: %s\n", what, cudaGetErrorString(e));
    };
    int prev = -1;
    if (cudaGetDevice(&prev) == cudaSuccess && prev != device_) warn(cudaSetDevice(device_), "cudaSetDevice");
    if (stream_) warn(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    if (graph_) warn(cudaGraphExecDestroy(graph_), "cudaGraphExecDestroy");
    prefiller_.reset();  // it writes this engine's cache: gone before the cache is freed
    if (trace_) warn(cudaFree(trace_), "cudaFree(trace)");
    if (arena_) warn(cudaFree(arena_), "cudaFree(arena)");
    if (stream_) warn(cudaStreamDestroy(stream_), "cudaStreamDestroy");
    weights_.reset();
    if (prev >= 0 && prev != device_) cudaSetDevice(prev);
}

// ---- persistent path ---------------------------------------------------------------------------------

void Engine::make_step_params() {
    const ModelConfig& c = config();
    const Weights& W = *weights_;
    CLLM_CHECK(decode_step_grid() <= kArgmaxBlocks, "decode step: more SMs than argmax partial slots");
    StepParams& p = step_;
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& L = W.layers[l];
        p.layers[l] = StepLayer{L.attn_norm, L.wqkv.w, L.wqkv.scales, L.wo.w, L.wo.scales,
                                L.ffn_norm,  L.w_gate_up.w, L.w_gate_up.scales, L.w_down.w, L.w_down.scales};
    }
    p.emb_w = W.tok_embeddings.w;
    p.emb_s = W.tok_embeddings.scales;
    p.final_norm = W.final_norm;
    p.inv_freq = W.rope_inv_freq;
    // The tagged activation words: q|k|v, attention output, residual after O, residual after down, SwiGLU.
    unsigned long long* t = tagged_;
    p.t_qkv = t;
    p.t_att = p.t_qkv + static_cast<size_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    p.t_xmid = p.t_att + static_cast<size_t>(c.n_heads) * c.head_dim;
    p.t_xout = p.t_xmid + c.hidden;
    p.t_act = p.t_xout + c.hidden;
    p.logits = logits_;
    p.k_cache = k_cache_;
    p.v_cache = v_cache_;
    p.part_o = part_o_;
    p.part_ml = part_ml_;
    p.am_v = am_v_;
    p.am_i = am_i_;
    p.d_token = &state_->token;
    p.d_pos = &state_->pos;
    p.sync = sync_;
    p.err = state_->err;
    p.max_seq = max_seq_;
    p.eps = c.rms_eps;
    p.group_size = c.group_size;
    p.wait_limit_ns = kWaitLimitNs;
    p.drain_limit_ns = kDrainLimitNs;
    p.prefetch_tiles = kPrefetchTiles;
    p.prefetch_mode = 3;  // bulk L2 prefetches from the prefetch warp
    p.whole_head_max_tiles = c.wtype == WeightType::INT4 ? kWholeHeadMaxTilesInt4 : kWholeHeadMaxTiles;
    p.stall_op = -1;
    p.sample_temperature = 0.f;  // greedy
    p.sample_top_k = kMaxTopK;
    p.sample_top_p = 1.f;
    p.sample_seed = 0;
    p.cand = cand_;
    CLLM_CHECK(c.vocab / decode_step_grid() >= kMaxTopK && decode_step_grid() <= kSampleMaxGrid &&
                   c.vocab / decode_step_grid() + 1 <= kSampleMaxGrid * kMaxTopK,
               "decode step: lm_head rows per CTA or grid outside the sampling bounds");
    // The persistent kernel has its own compile-time tile shape (matvec_rpb applies to the per-op kernels;
    // results do not depend on either).
    const int rows = decode_step_tile_rows(c.wtype);
    const int qkv_rows = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    p.g_qkv = make_tile_geom(c.wtype, Epilogue::STORE, qkv_rows, c.hidden, rows);
    p.g_wo = make_tile_geom(c.wtype, Epilogue::ADD, c.hidden, c.hidden, rows);
    p.g_gu = make_tile_geom(c.wtype, Epilogue::SWIGLU, 2 * c.inter, c.hidden, rows);
    p.g_down = make_tile_geom(c.wtype, Epilogue::ADD, c.hidden, c.inter, rows, kDownSegBytes);
    p.g_lm = make_tile_geom(c.wtype, Epilogue::STORE, c.vocab, c.hidden, rows);
    set_knob("trace_tile_op", kTraceLmOp);
}

void Engine::set_sampling(float temperature, int top_k, float top_p, unsigned long long seed) {
    CLLM_REQUIRE(std::isfinite(temperature) && temperature >= 0.f, "temperature must be finite and >= 0 (0 = greedy)");
    CLLM_REQUIRE(top_k >= 0 && top_k <= kMaxTopK, "top_k must be in [0, 64] (0 = 64)");
    CLLM_REQUIRE(top_p > 0.f && top_p <= 1.f, "top_p must be in (0, 1]");
    CLLM_REQUIRE(temperature == 0.f || persistent_, "sampling needs the persistent decode path");
    step_.sample_temperature = temperature;
    step_.sample_top_k = top_k == 0 ? kMaxTopK : top_k;
    step_.sample_top_p = top_p;
    step_.sample_seed = seed;
}

void Engine::set_knob(const std::string& name, long long value) {
    CLLM_REQUIRE(persistent_, "debug knobs apply to the persistent decode path only");
    auto in = [&](long long lo, long long hi) {
        if (value < lo || value > hi) {
            throw ArgError("knob " + name + " must be in [" + std::to_string(lo) + ", " + std::to_string(hi) + "]");
        }
    };
    if (name == "wait_limit_ns") {
        in(1, 10000000000ll);
        step_.wait_limit_ns = static_cast<unsigned long long>(value);
    } else if (name == "prefetch_tiles") {
        in(0, 1024);
        step_.prefetch_tiles = static_cast<int>(value);
    } else if (name == "whole_head_max_tiles") {
        in(0, max_seq_ / kAttnTile);
        step_.whole_head_max_tiles = static_cast<int>(value);
    } else if (name == "trace_tile_op") {
        in(0, kTraceLmOp);
        // Global index (in CTA 0's tile stream) of the first tile of that weight operation: CTA 0 owns rows
        // [0, rows / grid) of every operation.
        const int grid = decode_step_grid();
        const TileGeom* per_layer[4] = {&step_.g_qkv, &step_.g_wo, &step_.g_gu, &step_.g_down};
        int t0 = 0;
        for (int o = 0; o < value; ++o) {
            const TileGeom& g = *per_layer[o % 4];
            t0 += (g.out_rows / grid + g.rows_per_tile - 1) / g.rows_per_tile * g.n_seg;
        }
        step_.trace_t0 = t0;
    } else if (name == "stall_op") {
        in(-1, kTraceLmOp);
        CLLM_REQUIRE(value != 0, "knob stall_op: weight operation 0 reads the embedding row, which has no wait");
        step_.stall_op = static_cast<int>(value);
    } else {
        throw ArgError("unknown knob '" + name + "' (wait_limit_ns, prefetch_tiles, whole_head_max_tiles, trace_tile_op, stall_op)");
    }
}

void Engine::launch_step_kernel(int token, float* debug_res) {
    // Each launch tags its activations with a fresh number (24 bits of the tag); before the number would
    // repeat the words are cleared, so no value of an earlier launch can match.
    if (++step_tag_ >= (1u << 24)) {
        CLLM_CUDA(cudaMemsetAsync(tagged_, 0, tagged_words_ * sizeof(unsigned long long), stream_));
        step_tag_ = 1;
    }
    StepParams p = step_;
    p.step_tag = step_tag_;
    p.token_override = token;
    p.debug_res = debug_res;
    p.trace = trace_on_ ? trace_ : nullptr;
    // The step's context is host_pos_ + 1 tokens (the host mirror is exact for the persistent path).
    const int tiles = (host_pos_ + 1 + kAttnTile - 1) / kAttnTile;
    launch_decode_step(p, config().wtype, opts_.kv, tiles > p.whole_head_max_tiles, stream_);
}

void Engine::set_trace(bool enable) {
    CLLM_REQUIRE(persistent_, "tracing needs the persistent decode path");
    DeviceGuard on(device_);
    if (enable && trace_ == nullptr) {
        const size_t bytes = trace_words(decode_step_grid()) * sizeof(unsigned long long);
        CLLM_CUDA(cudaMalloc(&trace_, bytes));
        CLLM_CUDA(cudaMemset(trace_, 0, bytes));
    }
    trace_on_ = enable;
}

int Engine::trace_grid() const { return decode_step_grid(); }

void Engine::read_trace(unsigned long long* out, size_t count) {
    if (trace_ == nullptr) throw StateError("tracing was never enabled");
    const size_t n = trace_words(decode_step_grid());
    CLLM_REQUIRE(count >= n, "read_trace: output buffer too small");
    synchronize();
    DeviceGuard on(device_);
    CLLM_CUDA(cudaMemcpy(out, trace_, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
}

// ---- per-op path -------------------------------------------------------------------------------------

// The plan follows the reference's per-token sequence (src/engine/engine.cpp:181-237): the fused form
// folds RMSNorm into the projections' prologue, the residual add / SwiGLU into their epilogues and RoPE
// into the KV write; the unfused form runs each as its own kernel. SNAPSHOT records only act in step_debug.
void Engine::build_plan() {
    const ModelConfig& c = config();
    const Weights& W = *weights_;
    const bool fused = opts_.fuse;
    auto add = [&](PlanStep s) { plan_.push_back(s); };
    add({Op::EMBED, -1, nullptr, nullptr, x_});
    add({Op::SNAPSHOT, 0, nullptr, x_});
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& L = W.layers[l];
        if (fused) {
            add({Op::MATVEC, l, &L.wqkv, x_, qkv_, L.attn_norm, Epilogue::STORE});
            add({Op::ROPE_KV, l, nullptr, nullptr, qkv_});
            add({Op::ATTN, l, nullptr, qkv_, att_});
            add({Op::MATVEC, l, &L.wo, att_, x_, nullptr, Epilogue::ADD});
            add({Op::MATVEC, l, &L.w_gate_up, x_, act_, L.ffn_norm, Epilogue::SWIGLU});
            add({Op::MATVEC, l, &L.w_down, act_, x_, nullptr, Epilogue::ADD});
        } else {
            add({Op::RMSNORM, l, nullptr, x_, xb_, L.attn_norm});
            add({Op::MATVEC, l, &L.wqkv, xb_, qkv_});
            add({Op::ROPE, l, nullptr, nullptr, qkv_});
            add({Op::KV_WRITE, l, nullptr, qkv_});
            add({Op::ATTN, l, nullptr, qkv_, att_});
            add({Op::MATVEC, l, &L.wo, att_, tmp_});
            add({Op::ADD, l, nullptr, tmp_, x_});
            add({Op::RMSNORM, l, nullptr, x_, xb_, L.ffn_norm});
            add({Op::MATVEC, l, &L.w_gate_up, xb_, gu_});
            add({Op::SILU_MUL, l, nullptr, gu_, act_});
            add({Op::MATVEC, l, &L.w_down, act_, tmp_});
            add({Op::ADD, l, nullptr, tmp_, x_});
        }
        add({Op::SNAPSHOT, l + 1, nullptr, x_});
    }
    if (fused) {
        add({Op::MATVEC, -1, &W.tok_embeddings, x_, logits_, W.final_norm, Epilogue::STORE});
    } else {
        add({Op::RMSNORM, -1, nullptr, x_, xb_, W.final_norm});
        add({Op::MATVEC, -1, &W.tok_embeddings, xb_, logits_});
    }
    add({Op::ARGMAX, -1, nullptr, logits_});
    for (const PlanStep& s : plan_) {
        CLLM_CHECK(s.op != Op::MATVEC || static_cast<const void*>(s.in) != static_cast<const void*>(s.out),
                   "launch plan: a projection reads and writes the same buffer");
        CLLM_CHECK(s.op != Op::MATVEC || opts_.matvec == MatvecImpl::OPT || (s.ep == Epilogue::STORE && s.gain == nullptr),
                   "launch plan: the naive matvec has no epilogue or fused norm");
    }
}

// Enqueues the plan on the engine's stream. residuals_out (host) != null: SNAPSHOT records copy x there.
template <typename KV>
void Engine::run_plan(float* residuals_out) {
    const ModelConfig& c = config();
    const int H = c.hidden, NH = c.n_heads, NKV = c.n_kv_heads, D = c.head_dim;
    const size_t layer_elems = static_cast<size_t>(NKV) * max_seq_ * D;
    const int* d_pos = &state_->pos;
    int* d_tok = &state_->token;
    for (const PlanStep& s : plan_) {
        KV* kl = reinterpret_cast<KV*>(k_cache_) + (s.layer < 0 ? 0 : s.layer * layer_elems);
        KV* vl = reinterpret_cast<KV*>(v_cache_) + (s.layer < 0 ? 0 : s.layer * layer_elems);
        switch (s.op) {
            case Op::EMBED: launch_embedding(weights_->tok_embeddings, d_tok, s.out, H, c.group_size, stream_); break;
            case Op::RMSNORM: launch_rmsnorm(s.in, s.gain, c.rms_eps, s.out, H, stream_); break;
            case Op::MATVEC: {
                MatvecArgs a;
                a.w = s.w->w;
                a.scales = s.w->scales;
                a.x = s.in;
                a.norm_w = s.gain;
                a.eps = c.rms_eps;
                a.y = s.out;
                a.rows = s.w->rows;
                a.cols = s.w->cols;
                if (opts_.matvec == MatvecImpl::NAIVE) {
                    launch_matvec_naive(a, stream_);
                } else {
                    launch_matvec_stream(s.w->wtype, s.ep, s.gain != nullptr, a, opts_.matvec_rpb, stream_, state_->err);
                }
                break;
            }
            case Op::ROPE: launch_rope_inplace<KV>(s.out, weights_->rope_inv_freq, d_pos, NH, NKV, D, stream_); break;
            case Op::KV_WRITE: launch_kv_write<KV>(s.in, kl, vl, d_pos, NH, NKV, D, max_seq_, stream_); break;
            case Op::ROPE_KV:
                launch_rope_kv_fused<KV>(s.out, weights_->rope_inv_freq, kl, vl, d_pos, NH, NKV, D, max_seq_, stream_);
                break;
            case Op::ATTN:
                if (opts_.attn == AttnImpl::NAIVE) {
                    launch_attention_naive<KV>(s.in, kl, vl, d_pos, s.out, NH, NKV, D, max_seq_, stream_);
                } else {
                    launch_attention_split<KV>(s.in, kl, vl, d_pos, part_o_, part_ml_, s.out, NH, NKV, D, max_seq_, stream_);
                }
                break;
            case Op::ADD: launch_add_inplace(s.out, s.in, H, stream_); break;
            case Op::SILU_MUL: launch_silu_mul(s.in, s.out, c.inter, stream_); break;
            case Op::ARGMAX: launch_argmax(s.in, c.vocab, am_v_, am_i_, d_tok, &state_->pos, stream_); break;
            case Op::SNAPSHOT:
                if (residuals_out != nullptr) {
                    CLLM_CUDA(cudaMemcpyAsync(residuals_out + static_cast<size_t>(s.layer) * H, s.in, sizeof(float) * H,
                                              cudaMemcpyDeviceToHost, stream_));
                }
                break;
        }
    }
}

void Engine::run_plan_any(float* residuals_out) {
    if (opts_.kv == KvType::F16) {
        run_plan<__half>(residuals_out);
    } else {
        run_plan<__nv_bfloat16>(residuals_out);
    }
}

// ---- stepping ------------------------------------------------------------------------------------------

void Engine::check_device_state(const DevState& st) {
    if (st.err[0] == 0) return;
    // A bounded in-kernel wait gave up. The failed step (and any queued after it, which abort at once) left
    // the device position where it was: take the host mirror from it, clear the error words and the
    // persistent step's tickets, and report; the engine stays usable.
    CLLM_CUDA(cudaMemsetAsync(state_->err, 0, sizeof(st.err), stream_));
    CLLM_CUDA(cudaMemsetAsync(sync_, 0, kSyncWords * sizeof(unsigned), stream_));
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    host_pos_ = st.pos;
    throw StateError("device: a bounded inter-block wait gave up (flags " + std::to_string(st.err[0]) + ", wait id " +
                     std::to_string(st.err[1]) + "); the step's results are invalid and its position was not taken");
}

void Engine::collect(float* logits_out, int* next_token_out) {
    DevState st{};
    CLLM_CUDA(cudaMemcpyAsync(&st, state_, sizeof(st), cudaMemcpyDeviceToHost, stream_));
    if (logits_out != nullptr) {
        CLLM_CUDA(cudaMemcpyAsync(logits_out, logits_, sizeof(float) * config().vocab, cudaMemcpyDeviceToHost, stream_));
    }
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    check_device_state(st);
    if (next_token_out != nullptr) *next_token_out = st.token;
}

void Engine::synchronize() {
    DeviceGuard on(device_);
    collect(nullptr, nullptr);
}

void Engine::reset() {
    DeviceGuard on(device_);
    synchronize();
    CLLM_CUDA(cudaMemsetAsync(&state_->pos, 0, sizeof(int), stream_));
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    host_pos_ = 0;
}

void Engine::step(int token, float* logits_out, int* next_token_out) {
    if (host_pos_ >= max_seq_) throw StateError("step: sequence is full (pos == max_seq_len); call reset()");
    CLLM_REQUIRE(token >= -1 && token < config().vocab, "step: token out of range");
    DeviceGuard on(device_);
    if (persistent_) {
        launch_step_kernel(token, nullptr);
    } else {
        if (token >= 0) launch_set_token(&state_->token, token, stream_);
        if (!opts_.cuda_graph) {
            run_plan_any(nullptr);
        } else {
            if (graph_ == nullptr) {
                // Capture the plan once; replays read the position and token from the device.
                cudaGraph_t g = nullptr;
                CLLM_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
                try {
                    run_plan_any(nullptr);
                } catch (...) {
                    cudaStreamEndCapture(stream_, &g);
                    if (g) cudaGraphDestroy(g);
                    throw;
                }
                CLLM_CUDA(cudaStreamEndCapture(stream_, &g));
                const cudaError_t inst = cudaGraphInstantiate(&graph_, g, 0);
                cudaGraphDestroy(g);
                CLLM_CUDA(inst);
            }
            CLLM_CUDA(cudaGraphLaunch(graph_, stream_));
        }
    }
    ++host_pos_;
    if (logits_out != nullptr || next_token_out != nullptr) collect(logits_out, next_token_out);
}

void Engine::step_debug(int token, float* residuals_out, float* logits_out, int* next_token_out) {
    if (host_pos_ >= max_seq_) throw StateError("step_debug: sequence is full (pos == max_seq_len); call reset()");
    CLLM_REQUIRE(token >= -1 && token < config().vocab, "step_debug: token out of range");
    CLLM_REQUIRE(residuals_out != nullptr, "step_debug: residuals_out is null");
    DeviceGuard on(device_);
    if (persistent_) {
        launch_step_kernel(token, debug_res_);
        const size_t n = static_cast<size_t>(config().n_layers + 1) * config().hidden;
        CLLM_CUDA(cudaMemcpyAsync(residuals_out, debug_res_, n * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    } else {
        if (token >= 0) launch_set_token(&state_->token, token, stream_);
        run_plan_any(residuals_out);
    }
    ++host_pos_;
    collect(logits_out, next_token_out);
}

}  // namespace cudallm

namespace cudallm {

void Engine::prefill(const int* tokens, int n, float* logits_out, int* next_token_out) {
    CLLM_REQUIRE(tokens != nullptr && n >= 1, "prefill: need at least one token");
    for (int i = 0; i < n; ++i) CLLM_REQUIRE(tokens[i] >= 0 && tokens[i] < config().vocab, "prefill: token out of range");
    if (static_cast<long long>(host_pos_) + n > max_seq_) throw StateError("prefill: the tokens do not fit in max_seq_len");
    DeviceGuard on(device_);
    collect(nullptr, nullptr);  // earlier steps done (and their failures reported)
    if (config().wtype == WeightType::INT8) {
        for (int i = 0; i < n; ++i) step(tokens[i], nullptr, nullptr);
        collect(logits_out, next_token_out);
        return;
    }
    if (!prefiller_) {
        BatchOptions o;
        o.n_seq = kBatchMax;
        o.max_seq_len = max_seq_;
        o.kv = opts_.kv;
        o.device = device_;
        o.cuda_graph = false;
        o.ext_k_cache = k_cache_;
        o.ext_v_cache = v_cache_;
        prefiller_ = std::make_unique<BatchEngine>(path_, o);
    }
    prefiller_->set_position(0, host_pos_);
    prefiller_->prefill(0, tokens, n, nullptr, nullptr);  // synchronises its own stream
    const int pos = host_pos_ + n;
    CLLM_CUDA(cudaMemcpyAsync(logits_, prefiller_->last_logits(), sizeof(float) * config().vocab, cudaMemcpyDeviceToDevice,
                              stream_));
    CLLM_CUDA(cudaMemcpyAsync(&state_->token, prefiller_->last_token(), sizeof(int), cudaMemcpyDeviceToDevice, stream_));
    CLLM_CUDA(cudaMemcpyAsync(&state_->pos, &pos, sizeof(int), cudaMemcpyHostToDevice, stream_));
    host_pos_ = pos;
    collect(logits_out, next_token_out);
}

}  // namespace cudallm
