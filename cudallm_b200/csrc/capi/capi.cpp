// The extern "C" boundary of libcudallm.so (include/cudallm.h).
//
// Symbols, argument meaning, return codes and ownership follow wasiqnauman/cudallm's C ABI
// (include/cudallm/cudallm.h:1-62); the plumbing behind them is this library's own:
//   * every library error is a cudallm::Error that carries its return code (common/check.h); the two
//     wrappers below (`invoke` for code-returning entry points, `answer` for value-returning ones) turn an
//     exception into a code plus the thread-local message read by cudallm_last_error();
//   * handles carry a tag word checked on every call, so a NULL or destroyed handle is reported as
//     INVALID_ARG instead of being dereferenced;
//   * the single-kernel test hooks stage all their device buffers as slices of ONE allocation
//     (HookStage), upload every input, launch on the legacy default stream, synchronise once and copy the
//     outputs back.
#include "cudallm.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "common/check.h"
#include "engine/batch_engine.h"
#include "engine/engine.h"
#include "kernels/batch.h"
#include "kernels/kernels.h"

namespace {
constexpr uint64_t kEngineTag = 0x62316d6c6c647563ull;  // "cudllm1b"
constexpr uint64_t kBatchTag = 0x6863746162647563ull;   // "cudbatch"
constexpr uint64_t kDeadTag = 0;
}  // namespace

struct cudallm_engine {
    uint64_t tag = kEngineTag;
    std::unique_ptr<cudallm::Engine> impl;
};

struct cudallm_batch {
    uint64_t tag = kBatchTag;
    std::unique_ptr<cudallm::BatchEngine> impl;
};

namespace cudallm {
namespace {

std::string& last_message() {
    thread_local std::string msg;
    return msg;
}

int fail(Status s, const char* what) {
    last_message() = what ? what : "";
    return static_cast<int>(s);
}

int report(const std::exception& ex) {
    if (const auto* e = dynamic_cast<const Error*>(&ex)) return fail(e->status(), e->what());
    if (dynamic_cast<const std::bad_alloc*>(&ex)) return fail(Status::INTERNAL, "host memory allocation failed");
    return fail(Status::INTERNAL, ex.what());
}

// Runs an entry point's body; returns CUDALLM_OK or the code of what it threw.
template <typename Body>
int invoke(Body&& body) noexcept {
    try {
        body();
        return CUDALLM_OK;
    } catch (const std::exception& ex) {
        return report(ex);
    } catch (...) {
        return fail(Status::INTERNAL, "unknown exception");
    }
}

// Runs a value-returning entry point; on failure records the message and returns `fallback`.
template <typename T, typename Body>
T answer(T fallback, Body&& body) noexcept {
    try {
        return body();
    } catch (const std::exception& ex) {
        report(ex);
    } catch (...) {
        fail(Status::INTERNAL, "unknown exception");
    }
    return fallback;
}

Engine& engine_of(cudallm_engine* h, const char* fn) {
    if (h == nullptr || h->tag != kEngineTag || !h->impl) throw ArgError(std::string(fn) + ": null or destroyed engine");
    return *h->impl;
}

BatchEngine& batch_of(cudallm_batch* h, const char* fn) {
    if (h == nullptr || h->tag != kBatchTag || !h->impl) throw ArgError(std::string(fn) + ": null or destroyed batch engine");
    return *h->impl;
}

void describe(const ModelConfig& c, int max_seq, uint64_t bytes, cudallm_config_info* out) {
    *out = cudallm_config_info{};
    out->weight_dtype = static_cast<int>(c.wtype);
    out->hidden = c.hidden;
    out->inter = c.inter;
    out->n_layers = c.n_layers;
    out->n_heads = c.n_heads;
    out->n_kv_heads = c.n_kv_heads;
    out->head_dim = c.head_dim;
    out->vocab = c.vocab;
    out->max_seq_len = max_seq;
    out->group_size = c.group_size;
    out->rms_eps = c.rms_eps;
    out->weight_bytes = bytes;
}

EngineOptions engine_options(const cudallm_options& o, const cudallm_options_ex* ex) {
    CLLM_REQUIRE(o.matvec_impl == 0 || o.matvec_impl == 1, "matvec_impl must be 0 (naive) or 1 (opt)");
    CLLM_REQUIRE(o.attn_impl == 0 || o.attn_impl == 1, "attn_impl must be 0 (naive) or 1 (opt)");
    EngineOptions r;
    r.matvec = o.matvec_impl ? MatvecImpl::OPT : MatvecImpl::NAIVE;
    r.attn = o.attn_impl ? AttnImpl::OPT : AttnImpl::NAIVE;
    r.fuse = o.fuse != 0;
    r.cuda_graph = o.cuda_graph != 0;
    r.max_seq_len = o.max_seq_len;
    r.matvec_rpb = o.matvec_rpb;
    if (ex != nullptr) {
        CLLM_REQUIRE(ex->struct_size == static_cast<int>(sizeof(cudallm_options_ex)),
                     "cudallm_options_ex.struct_size must be sizeof(cudallm_options_ex)");
        CLLM_REQUIRE(ex->kv_dtype == CUDALLM_KV_FP16 || ex->kv_dtype == CUDALLM_KV_BF16, "kv_dtype must be 0 (fp16) or 1 (bf16)");
        CLLM_REQUIRE(ex->path >= CUDALLM_PATH_AUTO && ex->path <= CUDALLM_PATH_PER_OP, "path must be 0 (auto), 1 or 2");
        CLLM_REQUIRE(ex->device >= -1, "device must be -1 (current) or an ordinal");
        r.kv = ex->kv_dtype == CUDALLM_KV_BF16 ? KvType::BF16 : KvType::F16;
        r.device = ex->device;
        r.path = static_cast<DecodePath>(ex->path);
    }
    return r;
}

// Device staging of one test-hook call. The call declares its buffers first (slice), then stage()
// makes one allocation, zero-fills what asked for it and uploads every input; after the launch, finish()
// synchronises, surfaces a failed in-kernel wait and downloads every output.
class HookStage {
public:
    HookStage() = default;
    HookStage(const HookStage&) = delete;
    HookStage& operator=(const HookStage&) = delete;
    ~HookStage() {
        if (base_ != nullptr) cudaFree(base_);
    }

    int slice(size_t bytes, const void* host_in = nullptr, void* host_out = nullptr, bool zero = false) {
        CLLM_CHECK(base_ == nullptr, "HookStage: slice after stage()");
        const size_t off = total_;
        total_ += (std::max<size_t>(bytes, 1) + 255) & ~size_t{255};
        slices_.push_back({off, bytes, host_in, host_out, zero});
        return static_cast<int>(slices_.size()) - 1;
    }

    void stage() {
        CLLM_CUDA(cudaMalloc(&base_, total_));
        for (const Slice& s : slices_) {
            if (s.zero) CLLM_CUDA(cudaMemsetAsync(base_ + s.off, 0, s.bytes, 0));
            if (s.in != nullptr && s.bytes) CLLM_CUDA(cudaMemcpyAsync(base_ + s.off, s.in, s.bytes, cudaMemcpyHostToDevice, 0));
        }
    }

    template <typename T>
    T* dev(int id) const {
        return reinterpret_cast<T*>(base_ + slices_[id].off);
    }

    void finish() {
        CLLM_CUDA(cudaGetLastError());
        CLLM_CUDA(cudaDeviceSynchronize());
        check_kernel_error();
        for (const Slice& s : slices_) {
            if (s.out != nullptr && s.bytes) CLLM_CUDA(cudaMemcpy(s.out, base_ + s.off, s.bytes, cudaMemcpyDeviceToHost));
        }
    }

private:
    struct Slice {
        size_t off, bytes;
        const void* in;
        void* out;
        bool zero;
    };
    std::vector<Slice> slices_;
    size_t total_ = 0;
    uint8_t* base_ = nullptr;
};

WeightType hook_weight_type(int code) {
    switch (code) {
        case 1: return WeightType::BF16;
        case 3: return WeightType::INT8;
        case 4: return WeightType::INT4;
        default: throw ArgError("weight_dtype must be 1 (bf16), 3 (int8) or 4 (int4)");
    }
}

size_t fp16_cache_bytes(int nkv, int max_seq, int hd) { return sizeof(__half) * static_cast<size_t>(nkv) * max_seq * hd; }

}  // namespace

// For entry points defined in other source files: records ex for cudallm_last_error, returns its code.
int capi_report(const std::exception& ex) { return report(ex); }

}  // namespace cudallm

using cudallm::answer;
using cudallm::invoke;

extern "C" {

const char* cudallm_last_error(void) { return cudallm::last_message().c_str(); }

void cudallm_default_options(cudallm_options* out) {
    if (out != nullptr) *out = cudallm_options{1, 1, 1, 1, 0, 0};
}

void cudallm_default_options_ex(cudallm_options_ex* out) {
    if (out == nullptr) return;
    *out = cudallm_options_ex{};
    out->struct_size = sizeof(cudallm_options_ex);
    out->kv_dtype = CUDALLM_KV_FP16;
    out->device = -1;
    out->path = CUDALLM_PATH_AUTO;
}

int cudallm_create_ex(const char* path, const cudallm_options* opts, const cudallm_options_ex* ex, cudallm_engine** out) {
    if (out != nullptr) *out = nullptr;
    return invoke([&] {
        CLLM_REQUIRE(path != nullptr && opts != nullptr && out != nullptr, "cudallm_create: path, opts and out must be non-null");
        auto h = std::make_unique<cudallm_engine>();
        h->impl = std::make_unique<cudallm::Engine>(path, cudallm::engine_options(*opts, ex));
        *out = h.release();
    });
}

int cudallm_create(const char* path, const cudallm_options* opts, cudallm_engine** out) {
    return cudallm_create_ex(path, opts, nullptr, out);
}

void cudallm_destroy(cudallm_engine* e) {
    if (e == nullptr || e->tag != kEngineTag) return;
    e->tag = kDeadTag;
    delete e;
}

int cudallm_get_config(cudallm_engine* e, cudallm_config_info* out) {
    return invoke([&] {
        cudallm::Engine& eng = cudallm::engine_of(e, "cudallm_get_config");
        CLLM_REQUIRE(out != nullptr, "cudallm_get_config: out is null");
        cudallm::describe(eng.config(), eng.max_seq(), eng.weight_bytes(), out);
    });
}

int cudallm_reset(cudallm_engine* e) { return invoke([&] { cudallm::engine_of(e, "cudallm_reset").reset(); }); }

int cudallm_pos(cudallm_engine* e) {
    return answer(-1, [&] { return cudallm::engine_of(e, "cudallm_pos").pos(); });
}

int cudallm_step(cudallm_engine* e, int token, float* logits_out, int* next_token_out) {
    return invoke([&] { cudallm::engine_of(e, "cudallm_step").step(token, logits_out, next_token_out); });
}

int cudallm_step_debug(cudallm_engine* e, int token, float* residuals_out, float* logits_out, int* next_token_out) {
    return invoke([&] {
        cudallm::engine_of(e, "cudallm_step_debug").step_debug(token, residuals_out, logits_out, next_token_out);
    });
}

int cudallm_synchronize(cudallm_engine* e) {
    return invoke([&] { cudallm::engine_of(e, "cudallm_synchronize").synchronize(); });
}

int cudallm_prefill(cudallm_engine* e, const int* tokens, int n, float* logits_out, int* next_token_out) {
    return invoke([&] { cudallm::engine_of(e, "cudallm_prefill").prefill(tokens, n, logits_out, next_token_out); });
}

int cudallm_engine_path(cudallm_engine* e) {
    return answer(-1, [&] {
        return cudallm::engine_of(e, "cudallm_engine_path").persistent() ? CUDALLM_PATH_PERSISTENT : CUDALLM_PATH_PER_OP;
    });
}

void* cudallm_engine_stream(cudallm_engine* e) {
    return answer<void*>(nullptr, [&] { return static_cast<void*>(cudallm::engine_of(e, "cudallm_engine_stream").stream()); });
}

int cudallm_engine_device(cudallm_engine* e) {
    return answer(-1, [&] { return cudallm::engine_of(e, "cudallm_engine_device").device(); });
}

int cudallm_debug_trace(cudallm_engine* e, int enable) {
    return invoke([&] { cudallm::engine_of(e, "cudallm_debug_trace").set_trace(enable != 0); });
}

int cudallm_debug_read_trace(cudallm_engine* e, unsigned long long* out, unsigned long long count, int* grid_out,
                             int* slots_out) {
    return invoke([&] {
        cudallm::Engine& eng = cudallm::engine_of(e, "cudallm_debug_read_trace");
        CLLM_REQUIRE(out != nullptr, "cudallm_debug_read_trace: out is null");
        eng.read_trace(out, static_cast<size_t>(count));
        if (grid_out != nullptr) *grid_out = eng.trace_grid();
        if (slots_out != nullptr) *slots_out = cudallm::kTraceSlots;
    });
}

int cudallm_debug_set(cudallm_engine* e, const char* knob, long long value) {
    return invoke([&] {
        cudallm::Engine& eng = cudallm::engine_of(e, "cudallm_debug_set");
        CLLM_REQUIRE(knob != nullptr, "cudallm_debug_set: knob is null");
        eng.set_knob(knob, value);
    });
}

int cudallm_set_sampling(cudallm_engine* e, float temperature, int top_k, float top_p, unsigned long long seed) {
    return invoke([&] { cudallm::engine_of(e, "cudallm_set_sampling").set_sampling(temperature, top_k, top_p, seed); });
}

// ---- single-kernel test hooks ----

int cudallm_kernel_matvec(int impl, int weight_dtype, int epilogue, int fuse_norm, int rpb, const void* w,
                          unsigned long long w_bytes, const void* scales, unsigned long long scales_bytes, const float* x,
                          const float* norm_w, float eps, float* y, int rows, int cols) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(w != nullptr && x != nullptr && y != nullptr && w_bytes > 0, "cudallm_kernel_matvec: null argument");
        CLLM_REQUIRE(rows > 0 && cols > 0, "cudallm_kernel_matvec: rows and cols must be positive");
        CLLM_REQUIRE(impl == 0 || impl == 1, "cudallm_kernel_matvec: impl must be 0 or 1");
        CLLM_REQUIRE(epilogue >= 0 && epilogue <= 2, "cudallm_kernel_matvec: epilogue must be 0, 1 or 2");
        CLLM_REQUIRE(rpb == 0 || rpb == 1 || rpb == 2 || rpb == 4 || rpb == 8, "cudallm_kernel_matvec: rpb must be 0, 1, 2, 4 or 8");
        const WeightType wt = hook_weight_type(weight_dtype);
        CLLM_REQUIRE(impl == 1 || (wt == WeightType::BF16 && epilogue == 0 && !fuse_norm),
                     "cudallm_kernel_matvec: naive requires bf16, STORE and no fused norm");
        CLLM_REQUIRE(!fuse_norm || norm_w != nullptr, "cudallm_kernel_matvec: fuse_norm needs norm_w");
        CLLM_REQUIRE(wt == WeightType::BF16 || (scales != nullptr && scales_bytes > 0),
                     "cudallm_kernel_matvec: quantized weights need scales");
        CLLM_REQUIRE(w_bytes >= static_cast<unsigned long long>(rows) * row_bytes(wt, static_cast<uint64_t>(cols)),
                     "cudallm_kernel_matvec: w_bytes smaller than rows x row bytes");
        if (wt == WeightType::INT8) CLLM_REQUIRE(scales_bytes >= 4ull * rows, "cudallm_kernel_matvec: int8 scales need rows floats");
        if (wt == WeightType::INT4) {
            CLLM_REQUIRE(cols % 128 == 0 && scales_bytes >= 2ull * rows * (cols / 128),
                         "cudallm_kernel_matvec: int4 scales need rows x cols/128 halves");
        }
        const Epilogue ep = static_cast<Epilogue>(epilogue);
        const int outs = ep == Epilogue::SWIGLU ? rows / 2 : rows;
        HookStage st;
        const int sw = st.slice(w_bytes, w);
        const int ss = scales != nullptr ? st.slice(scales_bytes, scales) : -1;
        const int sx = st.slice(sizeof(float) * cols, x);
        const int sn = fuse_norm ? st.slice(sizeof(float) * cols, norm_w) : -1;
        const int sy = st.slice(sizeof(float) * outs, y, y);  // ADD accumulates into the caller's y
        st.stage();
        MatvecArgs a;
        a.w = st.dev<void>(sw);
        a.scales = ss >= 0 ? st.dev<void>(ss) : nullptr;
        a.x = st.dev<float>(sx);
        a.norm_w = sn >= 0 ? st.dev<float>(sn) : nullptr;
        a.eps = eps;
        a.y = st.dev<float>(sy);
        a.rows = rows;
        a.cols = cols;
        if (impl == 0) {
            launch_matvec_naive(a, 0);
        } else {
            launch_matvec_stream(wt, ep, fuse_norm != 0, a, rpb, 0);
        }
        st.finish();
    });
}

int cudallm_kernel_rmsnorm(const float* x, const float* w, float eps, float* y, int n) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(x != nullptr && w != nullptr && y != nullptr && n > 0, "cudallm_kernel_rmsnorm: bad argument");
        HookStage st;
        const size_t b = sizeof(float) * n;
        const int sx = st.slice(b, x), sw = st.slice(b, w), sy = st.slice(b, nullptr, y);
        st.stage();
        launch_rmsnorm(st.dev<float>(sx), st.dev<float>(sw), eps, st.dev<float>(sy), n, 0);
        st.finish();
    });
}

int cudallm_kernel_rope_kv(int fused, float* qkv, const float* inv_freq, int pos, unsigned short* k_cache,
                           unsigned short* v_cache, int nh, int nkv, int hd, int max_seq) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(qkv != nullptr && inv_freq != nullptr && k_cache != nullptr && v_cache != nullptr,
                     "cudallm_kernel_rope_kv: null argument");
        CLLM_REQUIRE(nh > 0 && nkv > 0 && hd > 0 && max_seq > 0 && pos >= 0 && pos < max_seq,
                     "cudallm_kernel_rope_kv: bad dimensions (need pos in [0, max_seq))");
        HookStage st;
        const size_t cache = fp16_cache_bytes(nkv, max_seq, hd);
        const int sq = st.slice(sizeof(float) * (nh + 2 * nkv) * hd, qkv, qkv);
        const int sf = st.slice(sizeof(float) * hd / 2, inv_freq);
        const int sk = st.slice(cache, k_cache, k_cache);
        const int sv = st.slice(cache, v_cache, v_cache);
        const int sp = st.slice(sizeof(int), &pos);
        st.stage();
        float* dq = st.dev<float>(sq);
        __half* dk = st.dev<__half>(sk);
        __half* dv = st.dev<__half>(sv);
        const int* dp = st.dev<int>(sp);
        if (fused) {
            launch_rope_kv_fused<__half>(dq, st.dev<float>(sf), dk, dv, dp, nh, nkv, hd, max_seq, 0);
        } else {
            launch_rope_inplace<__half>(dq, st.dev<float>(sf), dp, nh, nkv, hd, 0);
            launch_kv_write<__half>(dq, dk, dv, dp, nh, nkv, hd, max_seq, 0);
        }
        st.finish();
    });
}

int cudallm_kernel_attention(int impl, const float* q, const unsigned short* k_cache, const unsigned short* v_cache, int ctx,
                             float* out, int nh, int nkv, int hd, int max_seq) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(q != nullptr && k_cache != nullptr && v_cache != nullptr && out != nullptr,
                     "cudallm_kernel_attention: null argument");
        CLLM_REQUIRE(impl == 0 || impl == 1, "cudallm_kernel_attention: impl must be 0 or 1");
        CLLM_REQUIRE(nh > 0 && nkv > 0 && hd > 0 && max_seq > 0 && ctx >= 1 && ctx <= max_seq,
                     "cudallm_kernel_attention: bad dimensions (need ctx in [1, max_seq])");
        if (impl == 1) {
            CLLM_REQUIRE(max_seq % kAttnAbiChunk == 0, "cudallm_kernel_attention: opt needs max_seq % 128 == 0");
            CLLM_REQUIRE(nh == 4 * nkv && hd == 64, "cudallm_kernel_attention: opt needs nh == 4*nkv and hd == 64");
        }
        const int last = ctx - 1;  // the kernels read the position of the newest cached token
        const size_t slots = static_cast<size_t>(max_seq) / kAttnTile;
        const size_t qb = sizeof(float) * nh * hd;
        HookStage st;
        const int sq = st.slice(qb, q);
        const int sk = st.slice(fp16_cache_bytes(nkv, max_seq, hd), k_cache);
        const int sv = st.slice(fp16_cache_bytes(nkv, max_seq, hd), v_cache);
        const int sp = st.slice(sizeof(int), &last);
        const int so = st.slice(qb, nullptr, out);
        const int spo = impl == 1 ? st.slice(sizeof(float) * nh * slots * hd) : -1;
        const int spm = impl == 1 ? st.slice(sizeof(float) * nh * slots * 2) : -1;
        st.stage();
        const auto* dk = st.dev<const __half>(sk);
        const auto* dv = st.dev<const __half>(sv);
        if (impl == 0) {
            launch_attention_naive<__half>(st.dev<float>(sq), dk, dv, st.dev<int>(sp), st.dev<float>(so), nh, nkv, hd, max_seq, 0);
        } else {
            launch_attention_split<__half>(st.dev<float>(sq), dk, dv, st.dev<int>(sp), st.dev<float>(spo), st.dev<float>(spm),
                                           st.dev<float>(so), nh, nkv, hd, max_seq, 0);
        }
        st.finish();
    });
}

int cudallm_kernel_silu_mul(const float* gu, float* act, int inter) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(gu != nullptr && act != nullptr && inter > 0, "cudallm_kernel_silu_mul: bad argument");
        HookStage st;
        const int sg = st.slice(sizeof(float) * 2 * inter, gu), sa = st.slice(sizeof(float) * inter, nullptr, act);
        st.stage();
        launch_silu_mul(st.dev<float>(sg), st.dev<float>(sa), inter, 0);
        st.finish();
    });
}

int cudallm_kernel_argmax(const float* logits, int n, int* out_idx) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(logits != nullptr && out_idx != nullptr && n > 0, "cudallm_kernel_argmax: bad argument");
        HookStage st;
        const int sl = st.slice(sizeof(float) * n, logits);
        const int sv = st.slice(sizeof(float) * kArgmaxBlocks), si = st.slice(sizeof(int) * kArgmaxBlocks);
        const int stok = st.slice(sizeof(int), nullptr, out_idx, true);
        const int spos = st.slice(sizeof(int), nullptr, nullptr, true);
        st.stage();
        launch_argmax(st.dev<float>(sl), n, st.dev<float>(sv), st.dev<int>(si), st.dev<int>(stok), st.dev<int>(spos), 0);
        st.finish();
    });
}

// ---- batched decode ----

void cudallm_default_batch_options(cudallm_batch_options* out) {
    if (out == nullptr) return;
    *out = cudallm_batch_options{};
    out->struct_size = sizeof(cudallm_batch_options);
    out->n_seq = cudallm::kBatchMax;
    out->kv_dtype = CUDALLM_KV_FP16;
    out->device = -1;
    out->cuda_graph = 1;
}

int cudallm_batch_create(const char* path, const cudallm_batch_options* opts, cudallm_batch** out) {
    if (out != nullptr) *out = nullptr;
    return invoke([&] {
        CLLM_REQUIRE(path != nullptr && opts != nullptr && out != nullptr, "cudallm_batch_create: path, opts and out must be non-null");
        CLLM_REQUIRE(opts->struct_size == static_cast<int>(sizeof(cudallm_batch_options)),
                     "cudallm_batch_create: struct_size must be sizeof(cudallm_batch_options)");
        CLLM_REQUIRE(opts->kv_dtype == CUDALLM_KV_FP16 || opts->kv_dtype == CUDALLM_KV_BF16, "kv_dtype must be 0 (fp16) or 1 (bf16)");
        cudallm::BatchOptions o;
        o.n_seq = opts->n_seq;
        o.max_seq_len = opts->max_seq_len;
        o.kv = opts->kv_dtype == CUDALLM_KV_BF16 ? cudallm::KvType::BF16 : cudallm::KvType::F16;
        o.device = opts->device;
        o.cuda_graph = opts->cuda_graph != 0;
        o.attn_mode = opts->attn_mode;
        auto h = std::make_unique<cudallm_batch>();
        h->impl = std::make_unique<cudallm::BatchEngine>(path, o);
        *out = h.release();
    });
}

void cudallm_batch_destroy(cudallm_batch* e) {
    if (e == nullptr || e->tag != kBatchTag) return;
    e->tag = kDeadTag;
    delete e;
}

int cudallm_batch_get_config(cudallm_batch* e, cudallm_config_info* out) {
    return invoke([&] {
        cudallm::BatchEngine& eng = cudallm::batch_of(e, "cudallm_batch_get_config");
        CLLM_REQUIRE(out != nullptr, "cudallm_batch_get_config: out is null");
        cudallm::describe(eng.config(), eng.max_seq(), eng.weight_bytes(), out);
    });
}

int cudallm_batch_reset(cudallm_batch* e, int seq) {
    return invoke([&] { cudallm::batch_of(e, "cudallm_batch_reset").reset(seq); });
}

int cudallm_batch_pos(cudallm_batch* e, int seq) {
    return answer(-1, [&] {
        cudallm::BatchEngine& eng = cudallm::batch_of(e, "cudallm_batch_pos");
        CLLM_REQUIRE(seq >= 0 && seq < eng.n_seq(), "cudallm_batch_pos: sequence index out of range");
        return eng.pos(seq);
    });
}

int cudallm_batch_step(cudallm_batch* e, const int* tokens, int* next_out, float* logits_out) {
    return invoke([&] { cudallm::batch_of(e, "cudallm_batch_step").step(tokens, next_out, logits_out); });
}

int cudallm_batch_synchronize(cudallm_batch* e) {
    return invoke([&] { cudallm::batch_of(e, "cudallm_batch_synchronize").synchronize(); });
}

int cudallm_batch_prefill(cudallm_batch* e, int seq, const int* tokens, int n, float* logits_out, int* next_token_out) {
    return invoke([&] { cudallm::batch_of(e, "cudallm_batch_prefill").prefill(seq, tokens, n, logits_out, next_token_out); });
}

void* cudallm_batch_stream(cudallm_batch* e) {
    return answer<void*>(nullptr, [&] { return static_cast<void*>(cudallm::batch_of(e, "cudallm_batch_stream").stream()); });
}

int cudallm_batch_debug_set(cudallm_batch* e, const char* knob, long long value) {
    return invoke([&] {
        cudallm::BatchEngine& eng = cudallm::batch_of(e, "cudallm_batch_debug_set");
        CLLM_REQUIRE(knob != nullptr, "cudallm_batch_debug_set: knob is null");
        eng.set_knob(knob, value);
    });
}

int cudallm_batch_debug_get(cudallm_batch* e, const char* knob, long long* value_out) {
    return invoke([&] {
        cudallm::BatchEngine& eng = cudallm::batch_of(e, "cudallm_batch_debug_get");
        CLLM_REQUIRE(knob != nullptr && value_out != nullptr, "cudallm_batch_debug_get: null argument");
        *value_out = eng.knob(knob);
    });
}

int cudallm_kernel_gemm(const unsigned short* w, const unsigned short* x, const unsigned short* x_lo, float* y, int n, int k,
                        int batch, int ksplit, int epilogue) {
    using namespace cudallm;
    return invoke([&] {
        CLLM_REQUIRE(w != nullptr && x != nullptr && y != nullptr, "cudallm_kernel_gemm: null argument");
        CLLM_REQUIRE(n > 0 && k >= 64 && k % 64 == 0 && batch >= 1 && batch <= kBatchMax && ksplit >= 1 &&
                         ksplit <= std::min(16, k / 64),
                     "cudallm_kernel_gemm: bad shape (batch 1..64, k a multiple of 64, ksplit <= min(16, k / 64))");
        CLLM_REQUIRE(epilogue >= 0 && epilogue <= 2, "cudallm_kernel_gemm: epilogue must be 0, 1 or 2");
        CLLM_REQUIRE(epilogue != 2 || n % 128 == 0, "cudallm_kernel_gemm: SWIGLU needs n % 128 == 0");
        const size_t wb = static_cast<size_t>(n) * k * 2;
        const size_t xb = static_cast<size_t>(batch) * k * 2;
        const size_t plane = static_cast<size_t>(kBatchMax) * k * 2;  // one bf16 activation plane [64][k]
        const size_t yb = static_cast<size_t>(batch) * (epilogue == 2 ? n / 2 : n) * sizeof(float);
        HookStage st;
        const int sw = st.slice(wb, w);
        const int sx = st.slice(2 * plane, nullptr, nullptr, true);  // [hi plane | lo plane], unused rows zero
        const int sy = st.slice(yb, y, y);                           // ADD accumulates into y
        const int se = st.slice(sizeof(unsigned), nullptr, nullptr, true);
        const int swi = epilogue == 2 ? st.slice(wb) : -1;
        st.stage();
        uint8_t* planes = st.dev<uint8_t>(sx);
        CLLM_CUDA(cudaMemcpyAsync(planes, x, xb, cudaMemcpyHostToDevice, 0));
        if (x_lo != nullptr) CLLM_CUDA(cudaMemcpyAsync(planes + plane, x_lo, xb, cudaMemcpyHostToDevice, 0));
        const __nv_bfloat16* wdev = st.dev<__nv_bfloat16>(sw);
        if (epilogue == 2) {
            // The SwiGLU epilogue reads gate/up rows interleaved per 128-row tile (the batched engine's layout).
            interleave_gate_up(wdev, st.dev<__nv_bfloat16>(swi), n / 2, k, 0);
            wdev = st.dev<__nv_bfloat16>(swi);
        }
        GemmEpi epi;
        epi.kind = static_cast<GemmEpilogue>(epilogue);
        epi.y = st.dev<float>(sy);
        launch_gemm(wdev, n, k, reinterpret_cast<const __nv_bfloat16*>(planes), batch, ksplit, epi, st.dev<unsigned>(se), 0);
        unsigned gave_up = 0;
        st.finish();
        CLLM_CUDA(cudaMemcpy(&gave_up, st.dev<unsigned>(se), sizeof(gave_up), cudaMemcpyDeviceToHost));
        if (gave_up != 0) throw StateError("cudallm_kernel_gemm: a bounded wait in the GEMM gave up; y is invalid");
    });
}

}  // extern "C"
