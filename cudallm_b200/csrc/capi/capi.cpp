// extern "C" boundary. Same symbols, argument meaning, validation and error-code mapping as
// wasiqnauman/cudallm src/capi/cudallm_capi.cpp:1-318 (see include/cudallm.h for the per-symbol
// citations); no exception crosses the ABI.
#include "cudallm.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "common/check.h"
#include "engine/batch_engine.h"
#include "engine/engine.h"
#include "kernels/batch.h"
#include "kernels/kernels.h"

struct cudallm_engine {
    cudallm::Engine* impl;
};

struct cudallm_batch {
    cudallm::BatchEngine* impl;
};

namespace {

thread_local std::string g_last_error;

void set_error(const char* msg) { g_last_error = msg ? msg : ""; }

int error_code(const std::exception& ex) {
    if (dynamic_cast<const cudallm::ArgError*>(&ex)) return CUDALLM_ERR_INVALID_ARG;
    if (dynamic_cast<const cudallm::FormatError*>(&ex)) return CUDALLM_ERR_FORMAT;
    if (dynamic_cast<const cudallm::IoError*>(&ex)) return CUDALLM_ERR_IO;
    if (dynamic_cast<const cudallm::StateError*>(&ex)) return CUDALLM_ERR_STATE;
    if (std::strstr(ex.what(), "CUDA")) return CUDALLM_ERR_CUDA;
    return CUDALLM_ERR_INTERNAL;
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return CUDALLM_OK;
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return error_code(ex);
    } catch (...) {
        set_error("unknown exception");
        return CUDALLM_ERR_INTERNAL;
    }
}

void require(bool cond, const char* msg) {
    if (!cond) throw cudallm::ArgError(msg);
}

// Device buffer that lives for one test-hook call.
class DevBuf {
public:
    explicit DevBuf(size_t bytes) {
        if (bytes) CLLM_CUDA(cudaMalloc(&p_, bytes));
    }
    ~DevBuf() {
        if (p_) cudaFree(p_);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    template <typename T>
    T* as() const {
        return static_cast<T*>(p_);
    }
    void upload(const void* src, size_t bytes) { CLLM_CUDA(cudaMemcpy(p_, src, bytes, cudaMemcpyHostToDevice)); }
    void download(void* dst, size_t bytes) const { CLLM_CUDA(cudaMemcpy(dst, p_, bytes, cudaMemcpyDeviceToHost)); }

private:
    void* p_ = nullptr;
};

void sync_and_check() {
    CLLM_CUDA(cudaGetLastError());
    CLLM_CUDA(cudaDeviceSynchronize());
    cudallm::check_kernel_error();
}

cudallm::WeightType to_weight_type(int code) {
    require(code == 1 || code == 3 || code == 4, "weight_dtype must be 1 (bf16), 3 (int8) or 4 (int4)");
    return static_cast<cudallm::WeightType>(code);
}

cudallm::EngineOptions to_options(const cudallm_options* opts, const cudallm_options_ex* ex) {
    require(opts->matvec_impl == 0 || opts->matvec_impl == 1, "matvec_impl must be 0 or 1");
    require(opts->attn_impl == 0 || opts->attn_impl == 1, "attn_impl must be 0 or 1");
    cudallm::EngineOptions o;
    o.matvec = static_cast<cudallm::MatvecImpl>(opts->matvec_impl);
    o.attn = static_cast<cudallm::AttnImpl>(opts->attn_impl);
    o.fuse = opts->fuse != 0;
    o.cuda_graph = opts->cuda_graph != 0;
    o.max_seq_len = opts->max_seq_len;
    o.matvec_rpb = opts->matvec_rpb;
    if (ex) {
        require(ex->struct_size == static_cast<int>(sizeof(cudallm_options_ex)), "cudallm_options_ex: bad struct_size");
        require(ex->kv_dtype == CUDALLM_KV_FP16 || ex->kv_dtype == CUDALLM_KV_BF16, "kv_dtype must be 0 (fp16) or 1 (bf16)");
        require(ex->path >= CUDALLM_PATH_AUTO && ex->path <= CUDALLM_PATH_PER_OP, "path must be 0, 1 or 2");
        require(ex->device >= -1, "device must be >= -1");
        o.kv = static_cast<cudallm::KvType>(ex->kv_dtype);
        o.device = ex->device;
        o.path = static_cast<cudallm::DecodePath>(ex->path);
    }
    return o;
}

}  // namespace

namespace cudallm {
// Records ex for cudallm_last_error and returns its code; for entry points in other source files.
int capi_report(const std::exception& ex) {
    set_error(ex.what());
    return error_code(ex);
}
}  // namespace cudallm

extern "C" {

const char* cudallm_last_error(void) { return g_last_error.c_str(); }

void cudallm_default_options(cudallm_options* out) {
    if (!out) return;
    out->matvec_impl = 1;
    out->attn_impl = 1;
    out->fuse = 1;
    out->cuda_graph = 1;
    out->max_seq_len = 0;
    out->matvec_rpb = 0;
}

void cudallm_default_options_ex(cudallm_options_ex* out) {
    if (!out) return;
    std::memset(out, 0, sizeof(*out));
    out->struct_size = sizeof(cudallm_options_ex);
    out->kv_dtype = CUDALLM_KV_FP16;
    out->device = -1;
    out->path = CUDALLM_PATH_AUTO;
}

int cudallm_create_ex(const char* path, const cudallm_options* opts, const cudallm_options_ex* ex, cudallm_engine** out) {
    return guarded([&] {
        require(path && opts && out, "cudallm_create: null argument");
        *out = nullptr;
        const cudallm::EngineOptions o = to_options(opts, ex);
        auto* e = new cudallm_engine{nullptr};
        try {
            e->impl = new cudallm::Engine(path, o);
        } catch (...) {
            delete e;
            throw;
        }
        *out = e;
    });
}

int cudallm_create(const char* path, const cudallm_options* opts, cudallm_engine** out) {
    return cudallm_create_ex(path, opts, nullptr, out);
}

void cudallm_destroy(cudallm_engine* e) {
    if (!e) return;
    delete e->impl;
    delete e;
}

int cudallm_get_config(cudallm_engine* e, cudallm_config_info* out) {
    return guarded([&] {
        require(e && e->impl && out, "cudallm_get_config: null argument");
        const cudallm::ModelConfig& c = e->impl->config();
        out->weight_dtype = static_cast<int>(c.wtype);
        out->hidden = c.hidden;
        out->inter = c.inter;
        out->n_layers = c.n_layers;
        out->n_heads = c.n_heads;
        out->n_kv_heads = c.n_kv_heads;
        out->head_dim = c.head_dim;
        out->vocab = c.vocab;
        out->max_seq_len = e->impl->max_seq();
        out->group_size = c.group_size;
        out->rms_eps = c.rms_eps;
        out->weight_bytes = e->impl->weight_bytes();
    });
}

int cudallm_reset(cudallm_engine* e) {
    return guarded([&] {
        require(e && e->impl, "cudallm_reset: null engine");
        e->impl->reset();
    });
}

int cudallm_pos(cudallm_engine* e) {
    if (!e || !e->impl) {
        set_error("cudallm_pos: null engine");
        return -1;
    }
    return e->impl->pos();
}

int cudallm_step(cudallm_engine* e, int token, float* logits_out, int* next_token_out) {
    return guarded([&] {
        require(e && e->impl, "cudallm_step: null engine");
        require(token >= -1, "cudallm_step: token must be >= -1");
        e->impl->step(token, logits_out, next_token_out);
    });
}

int cudallm_step_debug(cudallm_engine* e, int token, float* residuals_out, float* logits_out, int* next_token_out) {
    return guarded([&] {
        require(e && e->impl, "cudallm_step_debug: null engine");
        require(token >= -1, "cudallm_step_debug: token must be >= -1");
        require(residuals_out, "cudallm_step_debug: residuals_out is null");
        e->impl->step_debug(token, residuals_out, logits_out, next_token_out);
    });
}

int cudallm_synchronize(cudallm_engine* e) {
    return guarded([&] {
        require(e && e->impl, "cudallm_synchronize: null engine");
        e->impl->synchronize();
    });
}

int cudallm_engine_path(cudallm_engine* e) {
    if (!e || !e->impl) {
        set_error("cudallm_engine_path: null engine");
        return -1;
    }
    return e->impl->persistent() ? CUDALLM_PATH_PERSISTENT : CUDALLM_PATH_PER_OP;
}

void* cudallm_engine_stream(cudallm_engine* e) {
    if (!e || !e->impl) {
        set_error("cudallm_engine_stream: null engine");
        return nullptr;
    }
    return static_cast<void*>(e->impl->stream());
}

int cudallm_engine_device(cudallm_engine* e) {
    if (!e || !e->impl) {
        set_error("cudallm_engine_device: null engine");
        return -1;
    }
    return e->impl->device();
}

int cudallm_debug_trace(cudallm_engine* e, int enable) {
    return guarded([&] {
        require(e && e->impl, "cudallm_debug_trace: null engine");
        e->impl->set_trace(enable != 0);
    });
}

int cudallm_debug_read_trace(cudallm_engine* e, unsigned long long* out, unsigned long long count, int* grid_out,
                             int* slots_out) {
    return guarded([&] {
        require(e && e->impl && out, "cudallm_debug_read_trace: null argument");
        e->impl->read_trace(out, static_cast<size_t>(count));
        if (grid_out) *grid_out = e->impl->trace_grid();
        if (slots_out) *slots_out = cudallm::kTraceSlots;
    });
}

int cudallm_kernel_matvec(int impl, int weight_dtype, int epilogue, int fuse_norm, int rpb, const void* w,
                          unsigned long long w_bytes, const void* scales, unsigned long long scales_bytes, const float* x,
                          const float* norm_w, float eps, float* y, int rows, int cols) {
    return guarded([&] {
        require(w && x && y && w_bytes > 0, "cudallm_kernel_matvec: null argument");
        require(rows > 0 && cols > 0, "cudallm_kernel_matvec: bad shape");
        require(impl == 0 || impl == 1, "cudallm_kernel_matvec: impl must be 0 or 1");
        require(epilogue >= 0 && epilogue <= 2, "cudallm_kernel_matvec: bad epilogue");
        require(rpb == 0 || rpb == 1 || rpb == 2 || rpb == 4 || rpb == 8, "cudallm_kernel_matvec: rpb must be 0, 1, 2, 4 or 8");
        const cudallm::WeightType wt = to_weight_type(weight_dtype);
        const auto ep = static_cast<cudallm::Epilogue>(epilogue);
        if (impl == 0) {
            require(weight_dtype == 1 && epilogue == 0 && fuse_norm == 0,
                    "cudallm_kernel_matvec: naive requires bf16, STORE and no fused norm");
        }
        if (fuse_norm) require(norm_w != nullptr, "cudallm_kernel_matvec: fuse_norm needs norm_w");
        if (wt != cudallm::WeightType::BF16) {
            require(scales && scales_bytes > 0, "cudallm_kernel_matvec: quantized weights need scales");
        }
        require(w_bytes >= static_cast<unsigned long long>(rows) * cudallm::row_bytes(wt, static_cast<uint64_t>(cols)),
                "cudallm_kernel_matvec: w_bytes smaller than rows x row bytes");
        if (wt == cudallm::WeightType::INT8) {
            require(scales_bytes >= 4ull * rows, "cudallm_kernel_matvec: int8 scales need rows floats");
        } else if (wt == cudallm::WeightType::INT4) {
            require(cols % 128 == 0 && scales_bytes >= 2ull * rows * (cols / 128),
                    "cudallm_kernel_matvec: int4 scales need rows x cols/128 halves");
        }
        const int out_rows = (ep == cudallm::Epilogue::SWIGLU) ? rows / 2 : rows;
        DevBuf dw(w_bytes), ds(scales ? scales_bytes : 0), dx(sizeof(float) * cols), dn(fuse_norm ? sizeof(float) * cols : 0),
            dy(sizeof(float) * out_rows);
        dw.upload(w, w_bytes);
        if (scales) ds.upload(scales, scales_bytes);
        dx.upload(x, sizeof(float) * cols);
        if (fuse_norm) dn.upload(norm_w, sizeof(float) * cols);
        dy.upload(y, sizeof(float) * out_rows);
        cudallm::MatvecArgs a;
        a.w = dw.as<void>();
        a.scales = scales ? ds.as<void>() : nullptr;
        a.x = dx.as<float>();
        a.norm_w = fuse_norm ? dn.as<float>() : nullptr;
        a.eps = eps;
        a.y = dy.as<float>();
        a.rows = rows;
        a.cols = cols;
        if (impl == 0) {
            cudallm::launch_matvec_naive(a, 0);
        } else {
            cudallm::launch_matvec_stream(wt, ep, fuse_norm != 0, a, rpb, 0);
        }
        sync_and_check();
        dy.download(y, sizeof(float) * out_rows);
    });
}

int cudallm_kernel_rmsnorm(const float* x, const float* w, float eps, float* y, int n) {
    return guarded([&] {
        require(x && w && y && n > 0, "cudallm_kernel_rmsnorm: bad argument");
        const size_t bytes = sizeof(float) * n;
        DevBuf dx(bytes), dw(bytes), dy(bytes);
        dx.upload(x, bytes);
        dw.upload(w, bytes);
        cudallm::launch_rmsnorm(dx.as<float>(), dw.as<float>(), eps, dy.as<float>(), n, 0);
        sync_and_check();
        dy.download(y, bytes);
    });
}

int cudallm_kernel_rope_kv(int fused, float* qkv, const float* inv_freq, int pos, unsigned short* k_cache,
                           unsigned short* v_cache, int nh, int nkv, int hd, int max_seq) {
    return guarded([&] {
        require(qkv && inv_freq && k_cache && v_cache, "cudallm_kernel_rope_kv: null argument");
        require(nh > 0 && nkv > 0 && hd > 0 && max_seq > 0 && pos >= 0 && pos < max_seq,
                "cudallm_kernel_rope_kv: bad dimensions");
        const size_t qkv_bytes = sizeof(float) * (nh + 2 * nkv) * hd;
        const size_t cache_bytes = sizeof(__half) * static_cast<size_t>(nkv) * max_seq * hd;
        DevBuf dqkv(qkv_bytes), dinv(sizeof(float) * hd / 2), dk(cache_bytes), dv(cache_bytes), dpos(sizeof(int));
        dqkv.upload(qkv, qkv_bytes);
        dinv.upload(inv_freq, sizeof(float) * hd / 2);
        dk.upload(k_cache, cache_bytes);
        dv.upload(v_cache, cache_bytes);
        dpos.upload(&pos, sizeof(int));
        if (fused) {
            cudallm::launch_rope_kv_fused<__half>(dqkv.as<float>(), dinv.as<float>(), dk.as<__half>(), dv.as<__half>(),
                                                  dpos.as<int>(), nh, nkv, hd, max_seq, 0);
        } else {
            cudallm::launch_rope_inplace<__half>(dqkv.as<float>(), dinv.as<float>(), dpos.as<int>(), nh, nkv, hd, 0);
            cudallm::launch_kv_write<__half>(dqkv.as<float>(), dk.as<__half>(), dv.as<__half>(), dpos.as<int>(), nh, nkv, hd,
                                             max_seq, 0);
        }
        sync_and_check();
        dqkv.download(qkv, qkv_bytes);
        dk.download(k_cache, cache_bytes);
        dv.download(v_cache, cache_bytes);
    });
}

int cudallm_kernel_attention(int impl, const float* q, const unsigned short* k_cache, const unsigned short* v_cache, int ctx,
                             float* out, int nh, int nkv, int hd, int max_seq) {
    return guarded([&] {
        require(q && k_cache && v_cache && out, "cudallm_kernel_attention: null argument");
        require(impl == 0 || impl == 1, "cudallm_kernel_attention: impl must be 0 or 1");
        require(nh > 0 && nkv > 0 && hd > 0 && max_seq > 0 && ctx >= 1 && ctx <= max_seq,
                "cudallm_kernel_attention: bad dimensions");
        if (impl == 1) {
            require(max_seq % cudallm::kAttnAbiChunk == 0, "cudallm_kernel_attention: opt needs max_seq % 128 == 0");
            require(nh == 4 * nkv && hd == 64, "cudallm_kernel_attention: opt needs nh == 4*nkv and hd == 64");
        }
        const size_t q_bytes = sizeof(float) * nh * hd;
        const size_t cache_bytes = sizeof(__half) * static_cast<size_t>(nkv) * max_seq * hd;
        const int pos = ctx - 1;
        const size_t n_slots = static_cast<size_t>(max_seq) / cudallm::kAttnTile;
        DevBuf dq(q_bytes), dk(cache_bytes), dv(cache_bytes), dpos(sizeof(int)), dout(q_bytes),
            dpo(impl == 1 ? sizeof(float) * nh * n_slots * hd : 0), dpml(impl == 1 ? sizeof(float) * nh * n_slots * 2 : 0);
        dq.upload(q, q_bytes);
        dk.upload(k_cache, cache_bytes);
        dv.upload(v_cache, cache_bytes);
        dpos.upload(&pos, sizeof(int));
        if (impl == 0) {
            cudallm::launch_attention_naive<__half>(dq.as<float>(), dk.as<__half>(), dv.as<__half>(), dpos.as<int>(),
                                                    dout.as<float>(), nh, nkv, hd, max_seq, 0);
        } else {
            cudallm::launch_attention_split<__half>(dq.as<float>(), dk.as<__half>(), dv.as<__half>(), dpos.as<int>(),
                                                    dpo.as<float>(), dpml.as<float>(), dout.as<float>(), nh, nkv, hd, max_seq, 0);
        }
        sync_and_check();
        dout.download(out, q_bytes);
    });
}

int cudallm_kernel_silu_mul(const float* gu, float* act, int inter) {
    return guarded([&] {
        require(gu && act && inter > 0, "cudallm_kernel_silu_mul: bad argument");
        DevBuf dgu(sizeof(float) * 2 * inter), dact(sizeof(float) * inter);
        dgu.upload(gu, sizeof(float) * 2 * inter);
        cudallm::launch_silu_mul(dgu.as<float>(), dact.as<float>(), inter, 0);
        sync_and_check();
        dact.download(act, sizeof(float) * inter);
    });
}

int cudallm_kernel_argmax(const float* logits, int n, int* out_idx) {
    return guarded([&] {
        require(logits && out_idx && n > 0, "cudallm_kernel_argmax: bad argument");
        DevBuf dl(sizeof(float) * n), dpv(sizeof(float) * cudallm::kArgmaxBlocks), dpi(sizeof(int) * cudallm::kArgmaxBlocks),
            dtok(sizeof(int)), dpos(sizeof(int));
        dl.upload(logits, sizeof(float) * n);
        const int zero = 0;
        dtok.upload(&zero, sizeof(int));
        dpos.upload(&zero, sizeof(int));
        cudallm::launch_argmax(dl.as<float>(), n, dpv.as<float>(), dpi.as<int>(), dtok.as<int>(), dpos.as<int>(), 0);
        sync_and_check();
        dtok.download(out_idx, sizeof(int));
    });
}

void cudallm_default_batch_options(cudallm_batch_options* out) {
    if (!out) return;
    std::memset(out, 0, sizeof(*out));
    out->struct_size = sizeof(cudallm_batch_options);
    out->n_seq = cudallm::kBatchMax;
    out->kv_dtype = CUDALLM_KV_FP16;
    out->device = -1;
    out->cuda_graph = 1;
}

int cudallm_batch_create(const char* path, const cudallm_batch_options* opts, cudallm_batch** out) {
    return guarded([&] {
        require(out != nullptr, "cudallm_batch_create: null argument");
        *out = nullptr;
        require(path && opts, "cudallm_batch_create: null argument");
        require(opts->struct_size == static_cast<int>(sizeof(cudallm_batch_options)),
                "cudallm_batch_create: struct_size must be sizeof(cudallm_batch_options)");
        cudallm::BatchOptions o;
        o.n_seq = opts->n_seq;
        o.max_seq_len = opts->max_seq_len;
        o.kv = static_cast<cudallm::KvType>(opts->kv_dtype);
        o.device = opts->device;
        o.cuda_graph = opts->cuda_graph != 0;
        auto* e = new cudallm_batch{nullptr};
        try {
            e->impl = new cudallm::BatchEngine(path, o);
        } catch (...) {
            delete e;
            throw;
        }
        *out = e;
    });
}

void cudallm_batch_destroy(cudallm_batch* e) {
    if (!e) return;
    delete e->impl;
    delete e;
}

int cudallm_batch_get_config(cudallm_batch* e, cudallm_config_info* out) {
    return guarded([&] {
        require(e && e->impl && out, "cudallm_batch_get_config: null argument");
        const cudallm::ModelConfig& c = e->impl->config();
        out->weight_dtype = static_cast<int>(c.wtype);
        out->hidden = c.hidden;
        out->inter = c.inter;
        out->n_layers = c.n_layers;
        out->n_heads = c.n_heads;
        out->n_kv_heads = c.n_kv_heads;
        out->head_dim = c.head_dim;
        out->vocab = c.vocab;
        out->max_seq_len = e->impl->max_seq();
        out->group_size = c.group_size;
        out->rms_eps = c.rms_eps;
        out->weight_bytes = e->impl->weight_bytes();
    });
}

int cudallm_batch_reset(cudallm_batch* e, int seq) {
    return guarded([&] {
        require(e && e->impl, "cudallm_batch_reset: null engine");
        e->impl->reset(seq);
    });
}

int cudallm_batch_pos(cudallm_batch* e, int seq) {
    if (!e || !e->impl || seq < 0 || seq >= e->impl->n_seq()) {
        set_error("cudallm_batch_pos: null engine or sequence index out of range");
        return -1;
    }
    return e->impl->pos(seq);
}

int cudallm_batch_step(cudallm_batch* e, const int* tokens, int* next_out, float* logits_out) {
    return guarded([&] {
        require(e && e->impl, "cudallm_batch_step: null engine");
        e->impl->step(tokens, next_out, logits_out);
    });
}

int cudallm_batch_synchronize(cudallm_batch* e) {
    return guarded([&] {
        require(e && e->impl, "cudallm_batch_synchronize: null engine");
        e->impl->synchronize();
    });
}

void* cudallm_batch_stream(cudallm_batch* e) {
    if (!e || !e->impl) {
        set_error("cudallm_batch_stream: null engine");
        return nullptr;
    }
    return static_cast<void*>(e->impl->stream());
}

int cudallm_kernel_gemm(const unsigned short* w, const unsigned short* x, const unsigned short* x_lo, float* y, int n, int k,
                        int batch, int ksplit, int epilogue) {
    return guarded([&] {
        require(w && x && y, "cudallm_kernel_gemm: null argument");
        require(n > 0 && k >= 64 && k % 64 == 0 && batch >= 1 && batch <= cudallm::kBatchMax && ksplit >= 1 &&
                    ksplit <= std::min(16, k / 64),
                "cudallm_kernel_gemm: bad shape (batch 1..64, k a multiple of 64, ksplit <= min(16, k / 64))");
        require(epilogue >= 0 && epilogue <= 2 && (epilogue != 2 || n % 2 == 0), "cudallm_kernel_gemm: bad epilogue");
        const size_t wb = static_cast<size_t>(n) * k * 2, xb = static_cast<size_t>(batch) * k * 2;
        const size_t plane = static_cast<size_t>(cudallm::kBatchMax) * k * 2;
        const int n_out = epilogue == 2 ? n / 2 : n;
        const size_t yb = static_cast<size_t>(batch) * n_out * sizeof(float);
        DevBuf dw(wb), dx(2 * plane), dy(yb), derr(sizeof(unsigned));
        dw.upload(w, wb);
        // Activation planes [2][64][k]: x in the hi plane, x_lo (or zeros) in the lo plane, unused rows zero.
        CLLM_CUDA(cudaMemset(dx.as<void>(), 0, 2 * plane));
        CLLM_CUDA(cudaMemcpy(dx.as<void>(), x, xb, cudaMemcpyHostToDevice));
        if (x_lo) CLLM_CUDA(cudaMemcpy(dx.as<uint8_t>() + plane, x_lo, xb, cudaMemcpyHostToDevice));
        dy.upload(y, yb);  // ADD accumulates into y
        CLLM_CUDA(cudaMemset(derr.as<void>(), 0, sizeof(unsigned)));
        cudallm::GemmEpi epi;
        epi.kind = static_cast<cudallm::GemmEpilogue>(epilogue);
        epi.y = dy.as<float>();
        const __nv_bfloat16* wdev = dw.as<__nv_bfloat16>();
        DevBuf dwi(epilogue == 2 ? wb : 0);
        if (epilogue == 2) {
            // The SwiGLU epilogue takes gate/up rows interleaved per 128-row tile, as the batched engine
            // lays them out.
            require(n % 128 == 0, "cudallm_kernel_gemm: SWIGLU needs n % 128 == 0");
            cudallm::interleave_gate_up(wdev, dwi.as<__nv_bfloat16>(), n / 2, k, 0);
            wdev = dwi.as<__nv_bfloat16>();
        }
        cudallm::launch_gemm(wdev, n, k, dx.as<__nv_bfloat16>(), batch, ksplit, epi, derr.as<unsigned>(), 0);
        sync_and_check();
        unsigned e = 0;
        derr.download(&e, sizeof(e));
        if (e != 0) throw cudallm::StateError("cudallm_kernel_gemm: a bounded wait in the GEMM gave up");
        dy.download(y, yb);
    });
}

}  // extern "C"
