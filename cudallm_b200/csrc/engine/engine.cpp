#include "engine/engine.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "common/check.h"
#include "common/device.h"

namespace cudallm {

void validate(const EngineOptions& o, WeightType wt) {
    // Rules of wasiqnauman/cudallm src/engine/engine.cpp:10-21, plus the additive fields.
    if (o.matvec != MatvecImpl::NAIVE && o.matvec != MatvecImpl::OPT) throw ArgError("invalid matvec implementation");
    if (o.attn != AttnImpl::NAIVE && o.attn != AttnImpl::OPT) throw ArgError("invalid attention implementation");
    if (o.matvec == MatvecImpl::NAIVE) {
        if (wt != WeightType::BF16) throw ArgError("naive matvec requires bf16 weights");
        if (o.fuse) throw ArgError("naive matvec requires fuse=false");
    }
    if (o.matvec_rpb != 0 && o.matvec_rpb != 1 && o.matvec_rpb != 2 && o.matvec_rpb != 4 && o.matvec_rpb != 8) {
        throw ArgError("matvec_rpb must be one of 0, 1, 2, 4, 8");
    }
    if (o.max_seq_len < 0 || o.max_seq_len % 128 != 0) throw ArgError("max_seq_len must be 0 or a positive multiple of 128");
    if (o.kv != KvType::F16 && o.kv != KvType::BF16) throw ArgError("kv_dtype must be 0 (fp16) or 1 (bf16)");
    if (o.path == DecodePath::PERSISTENT &&
        !(o.fuse && o.matvec == MatvecImpl::OPT && o.attn == AttnImpl::OPT)) {
        throw ArgError("the persistent decode path needs fuse=1 and opt matvec/attention");
    }
}

namespace {

template <typename T>
void alloc(T** p, size_t count) {
    CLLM_CUDA(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
}

constexpr unsigned long long kStepWaitLimitNs = 1000000000ull;  // 1 s per inter-CTA wait
// Contexts up to this many 64-token tiles use the whole-head attention (one CTA per KV head); longer ones
// spread (head, tile) items over all CTAs. CUDALLM_WHOLE_HEAD_MAX_TILES overrides it.
constexpr int kDefaultWholeHeadMaxTiles = 2;
// L2 prefetch distance (tiles per SM) of the persistent step; CUDALLM_PREFETCH_TILES overrides it. 24 tiles
// of 16 KiB for bf16 / int8; int4 tiles hold 2 rows (1-8 KiB), so the same byte distance is ~8x the tiles.
constexpr int kDefaultPrefetchTiles = 24;
constexpr int kDefaultPrefetchTilesInt4 = 192;

}  // namespace

Engine::Engine(const std::string& path, const EngineOptions& opts) : opts_(opts) {
    // File and option errors are reported before any CUDA call (as the reference's loader does).
    const ParsedFile file = parse_cudallm(path);
    validate(opts_, file.config.wtype);
    if (opts_.max_seq_len > file.config.max_seq_len) throw ArgError("max_seq_len exceeds the file's max_seq_len");
    if (opts_.device >= 0) {
        int n = 0;
        CLLM_CUDA(cudaGetDeviceCount(&n));
        if (opts_.device >= n) throw ArgError("device ordinal out of range");
        device_ = opts_.device;
    } else {
        CLLM_CUDA(cudaGetDevice(&device_));
    }
    DeviceGuard guard(device_);
    weights_ = std::make_unique<Weights>(file);
    const ModelConfig& c = weights_->config();
    max_seq_ = opts_.max_seq_len ? opts_.max_seq_len : c.max_seq_len;
    persistent_ = opts_.path != DecodePath::PER_OP && opts_.fuse && opts_.matvec == MatvecImpl::OPT &&
                  opts_.attn == AttnImpl::OPT;
    try {
        CLLM_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        const size_t H = c.hidden, I = c.inter, V = c.vocab, S = max_seq_, KV = c.n_kv_heads, D = c.head_dim, NH = c.n_heads;
        alloc(&x_, H);
        alloc(&xb_, H);
        alloc(&qkv_, (NH + 2 * KV) * D);
        alloc(&att_, NH * D);
        alloc(&tmp_, H);
        alloc(&gu_, 2 * I);
        alloc(&act_, I);
        alloc(&logits_, V);
        const size_t cache_elems = static_cast<size_t>(c.n_layers) * KV * S * D;
        CLLM_CUDA(cudaMalloc(&k_cache_, cache_elems * 2));
        CLLM_CUDA(cudaMalloc(&v_cache_, cache_elems * 2));
        alloc(&part_o_, NH * (S / kAttnTile) * D);
        alloc(&part_ml_, NH * (S / kAttnTile) * 2);
        alloc(&am_v_, kArgmaxBlocks);
        alloc(&am_i_, kArgmaxBlocks);
        alloc(&state_, 1);
        alloc(&sync_, kSyncWords);
        alloc(&debug_res_, static_cast<size_t>(c.n_layers + 1) * H);
        tagged_words_ = (NH + 2 * KV) * D + NH * D + 2 * H + I;
        alloc(&tagged_, tagged_words_);
        CLLM_CUDA(cudaMemset(tagged_, 0, tagged_words_ * sizeof(unsigned long long)));
        CLLM_CUDA(cudaMemset(state_, 0, sizeof(DevState)));
        CLLM_CUDA(cudaMemset(sync_, 0, kSyncWords * sizeof(unsigned)));
        CLLM_CUDA(cudaMemset(k_cache_, 0, cache_elems * 2));
        CLLM_CUDA(cudaMemset(v_cache_, 0, cache_elems * 2));
        CLLM_CUDA(cudaDeviceSynchronize());

        if (persistent_) {
            CLLM_CHECK(decode_step_grid() <= kArgmaxBlocks, "decode step: more SMs than argmax partial slots");
            StepParams& p = step_params_;
            const Weights& W = *weights_;
            for (int l = 0; l < c.n_layers; ++l) {
                const LayerWeights& L = W.layers[l];
                p.layers[l] = {L.attn_norm, L.wqkv.w, L.wqkv.scales, L.wo.w, L.wo.scales,
                               L.ffn_norm,  L.w_gate_up.w, L.w_gate_up.scales, L.w_down.w, L.w_down.scales};
            }
            p.emb_w = W.tok_embeddings.w;
            p.emb_s = W.tok_embeddings.scales;
            p.final_norm = W.final_norm;
            p.inv_freq = W.rope_inv_freq;
            p.t_qkv = tagged_;
            p.t_att = p.t_qkv + (NH + 2 * KV) * D;
            p.t_xmid = p.t_att + NH * D;
            p.t_xout = p.t_xmid + H;
            p.t_act = p.t_xout + H;
            p.step_tag = 0;
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
            p.debug_res = nullptr;
            p.trace = nullptr;
            p.token_override = -1;
            p.max_seq = max_seq_;
            p.eps = c.rms_eps;
            p.group_size = c.group_size;
            p.wait_limit_ns = kStepWaitLimitNs;
            p.prefetch_tiles = c.wtype == WeightType::INT4 ? kDefaultPrefetchTilesInt4 : kDefaultPrefetchTiles;
            if (const char* env = std::getenv("CUDALLM_PREFETCH_TILES")) p.prefetch_tiles = std::max(0, std::atoi(env));
            p.prefetch_mode = 3;  // bulk L2 prefetches from the prefetch warp
            if (const char* env = std::getenv("CUDALLM_PREFETCH_MODE")) p.prefetch_mode = std::atoi(env);
            p.whole_head_max_tiles = kDefaultWholeHeadMaxTiles;
            if (const char* env = std::getenv("CUDALLM_WHOLE_HEAD_MAX_TILES")) p.whole_head_max_tiles = std::atoi(env);
            int trace_op = 64;  // lm_head; CUDALLM_TRACE_TILE_OP picks the weight operation whose tiles are stamped first
            if (const char* env = std::getenv("CUDALLM_TRACE_TILE_OP")) trace_op = std::atoi(env);
            // The persistent kernel is compiled for its own tile shape (decode_step_tile_rows; matvec_rpb
            // selects the tile rows of the per-op kernels only; results do not depend on it).
            const int rpb = decode_step_tile_rows(c.wtype);
            p.g_qkv = make_tile_geom(c.wtype, Epilogue::STORE, (c.n_heads + 2 * c.n_kv_heads) * c.head_dim, c.hidden, rpb);
            p.g_wo = make_tile_geom(c.wtype, Epilogue::ADD, c.hidden, c.hidden, rpb);
            p.g_gu = make_tile_geom(c.wtype, Epilogue::SWIGLU, 2 * c.inter, c.hidden, rpb);
            p.g_down = make_tile_geom(c.wtype, Epilogue::ADD, c.hidden, c.inter, rpb);
            p.g_lm = make_tile_geom(c.wtype, Epilogue::STORE, c.vocab, c.hidden, rpb);
            // Global index (in CTA 0's tile stream) of the first tile of weight operation trace_op: CTA 0 owns
            // rows [0, rows / grid) of every operation.
            const int grid = decode_step_grid();
            const TileGeom* per_layer[4] = {&p.g_qkv, &p.g_wo, &p.g_gu, &p.g_down};
            int t0 = 0;
            for (int o = 0; o < std::min(std::max(trace_op, 0), 64); ++o) {
                const TileGeom& g = *per_layer[o % 4];
                const int rows = g.out_rows / grid;
                t0 += (rows + g.rows_per_tile - 1) / g.rows_per_tile * g.n_seg;
            }
            p.trace_t0 = t0;
        }
    } catch (...) {
        free_all();
        throw;
    }
}

void Engine::free_all() noexcept {
    auto report = [](cudaError_t err, const char* what) {
        if (err != cudaSuccess) std::fprintf(stderr, "cudallm: %s failed in ~Engine: %s\n", what, cudaGetErrorString(err));
    };
    if (graph_exec_) report(cudaGraphExecDestroy(graph_exec_), "cudaGraphExecDestroy");
    if (graph_) report(cudaGraphDestroy(graph_), "cudaGraphDestroy");
    graph_exec_ = nullptr;
    graph_ = nullptr;
    void* bufs[] = {x_,      xb_,      qkv_,  att_,  tmp_,   gu_,   act_,       logits_, k_cache_,
                    v_cache_, part_o_, part_ml_, am_v_, am_i_, state_, sync_, debug_res_, tagged_, trace_};
    for (void* b : bufs) {
        if (b) report(cudaFree(b), "cudaFree");
    }
    x_ = xb_ = qkv_ = att_ = tmp_ = gu_ = act_ = logits_ = part_o_ = part_ml_ = am_v_ = debug_res_ = nullptr;
    k_cache_ = v_cache_ = nullptr;
    am_i_ = nullptr;
    trace_ = nullptr;
    tagged_ = nullptr;
    state_ = nullptr;
    sync_ = nullptr;
    if (stream_) report(cudaStreamDestroy(stream_), "cudaStreamDestroy");
    stream_ = nullptr;
}

Engine::~Engine() {
    try {
        DeviceGuard guard(device_);
        if (stream_) cudaStreamSynchronize(stream_);
        free_all();
        weights_.reset();
    } catch (const std::exception& ex) {
        std::fprintf(stderr, "cudallm: exception in ~Engine: %s\n", ex.what());
    } catch (...) {
        std::fprintf(stderr, "cudallm: unknown exception in ~Engine\n");
    }
}

void Engine::raise_if_device_error(const DevState& st) {
    if (st.err[0] == 0) return;
    // Leave the engine usable: clear the error words and the step's dependency counters.
    CLLM_CUDA(cudaMemsetAsync(state_->err, 0, sizeof(st.err), stream_));
    CLLM_CUDA(cudaMemsetAsync(sync_, 0, kSyncWords * sizeof(unsigned), stream_));
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    throw StateError("device: a bounded inter-block wait gave up (flags " + std::to_string(st.err[0]) + ", wait id " +
                     std::to_string(st.err[1]) + "); the step's results are invalid");
}

void Engine::synchronize() {
    DeviceGuard guard(device_);
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    DevState st{};
    CLLM_CUDA(cudaMemcpy(&st, state_, sizeof(st), cudaMemcpyDeviceToHost));
    raise_if_device_error(st);
}

void Engine::reset() {
    DeviceGuard guard(device_);
    synchronize();
    CLLM_CUDA(cudaMemsetAsync(&state_->pos, 0, sizeof(int), stream_));
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    host_pos_ = 0;
}

void Engine::finish_sync(float* logits_out, int* next_token_out) {
    DevState st{};
    CLLM_CUDA(cudaMemcpyAsync(&st, state_, sizeof(st), cudaMemcpyDeviceToHost, stream_));
    if (logits_out) {
        CLLM_CUDA(cudaMemcpyAsync(logits_out, logits_, sizeof(float) * config().vocab, cudaMemcpyDeviceToHost, stream_));
    }
    CLLM_CUDA(cudaStreamSynchronize(stream_));
    raise_if_device_error(st);
    if (next_token_out) *next_token_out = st.token;
}

void Engine::set_trace(bool enable) {
    if (!persistent_) throw ArgError("tracing needs the persistent decode path");
    DeviceGuard guard(device_);
    if (enable && !trace_) {
        const size_t n = trace_words(decode_step_grid());
        CLLM_CUDA(cudaMalloc(&trace_, n * sizeof(unsigned long long)));
        CLLM_CUDA(cudaMemset(trace_, 0, n * sizeof(unsigned long long)));
    }
    trace_on_ = enable;
}

int Engine::trace_grid() const { return decode_step_grid(); }

void Engine::read_trace(unsigned long long* out, size_t count) {
    if (!trace_) throw StateError("tracing was never enabled");
    const size_t n = trace_words(decode_step_grid());
    if (count < n) throw ArgError("read_trace: output buffer too small");
    synchronize();
    DeviceGuard guard(device_);
    CLLM_CUDA(cudaMemcpy(out, trace_, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
}

void Engine::enqueue_persistent(int token, float* debug_res) {
    StepParams p = step_params_;
    // Each launch tags its activations with a fresh step number (24 bits in the tag); before it would
    // repeat, the words are cleared so no value of an earlier launch can match.
    if (++step_tag_ >= (1u << 24)) {
        CLLM_CUDA(cudaMemsetAsync(tagged_, 0, tagged_words_ * sizeof(unsigned long long), stream_));
        step_tag_ = 1;
    }
    p.step_tag = step_tag_;
    p.token_override = token;
    p.debug_res = debug_res;
    p.trace = trace_on_ ? trace_ : nullptr;
    launch_decode_step(p, config().wtype, opts_.kv, stream_);
}

void Engine::step(int token, float* logits_out, int* next_token_out) {
    if (host_pos_ >= max_seq_) throw StateError("step: sequence is full (pos == max_seq_len); call reset()");
    if (token < -1 || token >= config().vocab) throw ArgError("step: token out of range");
    DeviceGuard guard(device_);
    if (persistent_) {
        enqueue_persistent(token, nullptr);
    } else {
        if (token >= 0) launch_set_token(&state_->token, token, stream_);
        if (opts_.cuda_graph) {
            if (!graph_exec_) {
                CLLM_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
                try {
                    enqueue_per_op(false, nullptr);
                } catch (...) {
                    cudaGraph_t broken = nullptr;
                    cudaStreamEndCapture(stream_, &broken);
                    if (broken) cudaGraphDestroy(broken);
                    throw;
                }
                CLLM_CUDA(cudaStreamEndCapture(stream_, &graph_));
                CLLM_CUDA(cudaGraphInstantiate(&graph_exec_, graph_, 0));
            }
            CLLM_CUDA(cudaGraphLaunch(graph_exec_, stream_));
        } else {
            enqueue_per_op(false, nullptr);
        }
    }
    host_pos_ += 1;
    if (logits_out || next_token_out) finish_sync(logits_out, next_token_out);
}

void Engine::step_debug(int token, float* residuals_out, float* logits_out, int* next_token_out) {
    if (host_pos_ >= max_seq_) throw StateError("step_debug: sequence is full (pos == max_seq_len); call reset()");
    if (token < -1 || token >= config().vocab) throw ArgError("step_debug: token out of range");
    if (!residuals_out) throw ArgError("step_debug: residuals_out is null");
    DeviceGuard guard(device_);
    const ModelConfig& c = config();
    if (persistent_) {
        enqueue_persistent(token, debug_res_);
        CLLM_CUDA(cudaMemcpyAsync(residuals_out, debug_res_, sizeof(float) * (c.n_layers + 1) * c.hidden,
                                  cudaMemcpyDeviceToHost, stream_));
    } else {
        if (token >= 0) launch_set_token(&state_->token, token, stream_);
        enqueue_per_op(true, residuals_out);
    }
    host_pos_ += 1;
    finish_sync(logits_out, next_token_out);
}

void Engine::launch_linear(const Linear& L, const float* x, float* y, Epilogue ep, const float* norm_w) {
    CLLM_CHECK(static_cast<const void*>(x) != static_cast<const void*>(y), "launch_linear: input and output alias");
    MatvecArgs a;
    a.w = L.w;
    a.scales = L.scales;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = config().rms_eps;
    a.y = y;
    a.rows = L.rows;
    a.cols = L.cols;
    if (opts_.matvec == MatvecImpl::NAIVE) {
        CLLM_CHECK(ep == Epilogue::STORE && norm_w == nullptr, "launch_linear: naive matvec supports STORE only, no fused norm");
        launch_matvec_naive(a, stream_);
    } else {
        launch_matvec_stream(L.wtype, ep, norm_w != nullptr, a, opts_.matvec_rpb, stream_, state_->err);
    }
}

void Engine::enqueue_per_op(bool debug, float* residuals_out) {
    if (opts_.kv == KvType::F16) {
        enqueue_layers<__half>(debug, residuals_out);
    } else {
        enqueue_layers<__nv_bfloat16>(debug, residuals_out);
    }
}

// The operation sequence of wasiqnauman/cudallm src/engine/engine.cpp:181-237 (fused and unfused).
template <typename KV>
void Engine::enqueue_layers(bool debug, float* residuals_out) {
    const ModelConfig& c = config();
    const Weights& W = *weights_;
    const int H = c.hidden, NH = c.n_heads, NKV = c.n_kv_heads, D = c.head_dim;
    const size_t layer_elems = static_cast<size_t>(NKV) * max_seq_ * D;
    KV* kc = static_cast<KV*>(k_cache_);
    KV* vc = static_cast<KV*>(v_cache_);
    const int* d_pos = &state_->pos;
    auto snapshot = [&](int k) {
        if (!debug) return;
        CLLM_CUDA(cudaMemcpyAsync(residuals_out + static_cast<size_t>(k) * H, x_, sizeof(float) * H, cudaMemcpyDeviceToHost,
                                  stream_));
    };
    auto attention = [&](int l) {
        const KV* kl = kc + l * layer_elems;
        const KV* vl = vc + l * layer_elems;
        if (opts_.attn == AttnImpl::NAIVE) {
            launch_attention_naive<KV>(qkv_, kl, vl, d_pos, att_, NH, NKV, D, max_seq_, stream_);
        } else {
            launch_attention_split<KV>(qkv_, kl, vl, d_pos, part_o_, part_ml_, att_, NH, NKV, D, max_seq_, stream_);
        }
    };
    launch_embedding(W.tok_embeddings, &state_->token, x_, H, c.group_size, stream_);
    snapshot(0);
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerWeights& L = W.layers[l];
        KV* kl = kc + l * layer_elems;
        KV* vl = vc + l * layer_elems;
        if (!opts_.fuse) {
            launch_rmsnorm(x_, L.attn_norm, c.rms_eps, xb_, H, stream_);
            launch_linear(L.wqkv, xb_, qkv_, Epilogue::STORE, nullptr);
            launch_rope_inplace<KV>(qkv_, W.rope_inv_freq, d_pos, NH, NKV, D, stream_);
            launch_kv_write<KV>(qkv_, kl, vl, d_pos, NH, NKV, D, max_seq_, stream_);
            attention(l);
            launch_linear(L.wo, att_, tmp_, Epilogue::STORE, nullptr);
            launch_add_inplace(x_, tmp_, H, stream_);
            launch_rmsnorm(x_, L.ffn_norm, c.rms_eps, xb_, H, stream_);
            launch_linear(L.w_gate_up, xb_, gu_, Epilogue::STORE, nullptr);
            launch_silu_mul(gu_, act_, c.inter, stream_);
            launch_linear(L.w_down, act_, tmp_, Epilogue::STORE, nullptr);
            launch_add_inplace(x_, tmp_, H, stream_);
        } else {
            launch_linear(L.wqkv, x_, qkv_, Epilogue::STORE, L.attn_norm);
            launch_rope_kv_fused<KV>(qkv_, W.rope_inv_freq, kl, vl, d_pos, NH, NKV, D, max_seq_, stream_);
            attention(l);
            launch_linear(L.wo, att_, x_, Epilogue::ADD, nullptr);
            launch_linear(L.w_gate_up, x_, act_, Epilogue::SWIGLU, L.ffn_norm);
            launch_linear(L.w_down, act_, x_, Epilogue::ADD, nullptr);
        }
        snapshot(l + 1);
    }
    if (!opts_.fuse) {
        launch_rmsnorm(x_, W.final_norm, c.rms_eps, xb_, H, stream_);
        launch_linear(W.tok_embeddings, xb_, logits_, Epilogue::STORE, nullptr);
    } else {
        launch_linear(W.tok_embeddings, x_, logits_, Epilogue::STORE, W.final_norm);
    }
    launch_argmax(logits_, c.vocab, am_v_, am_i_, &state_->token, &state_->pos, stream_);
}

}  // namespace cudallm
