/*
 * cudallm.h: C ABI of the B200 (sm_100a) Llama-3.2-1B decode engine.
 *
 * Drop-in replacement for wasiqnauman/cudallm's include/cudallm/cudallm.h:1-62. Every symbol, struct
 * layout, return code and ownership rule of that header is kept, so its ctypes wrapper
 * (python/cudallm/engine.py:39-66) and its tests bind this library unchanged when CUDALLM_LIB points
 * at it. Entry points after the "additive" marker are new and change none of the originals.
 *
 * Conventions (reference src/capi/cudallm_capi.cpp:24-44): every entry point returns a CUDALLM_*
 * code (except destroy / default_options / pos / last_error); no C++ exception crosses the ABI;
 * the message of the last failure on the calling thread is returned by cudallm_last_error().
 * One engine per thread; engines own all device memory, callers own all host buffers.
 */
#ifndef CUDALLM_B200_CUDALLM_H
#define CUDALLM_B200_CUDALLM_H

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes: reference include/cudallm/cudallm.h:8-14. */
#define CUDALLM_OK 0
#define CUDALLM_ERR_INVALID_ARG 1
#define CUDALLM_ERR_IO 2
#define CUDALLM_ERR_FORMAT 3
#define CUDALLM_ERR_CUDA 4
#define CUDALLM_ERR_STATE 5
#define CUDALLM_ERR_INTERNAL 6

typedef struct cudallm_engine cudallm_engine;

/* Engine options, 24 bytes: reference include/cudallm/cudallm.h:18-25.
 * matvec_impl/attn_impl: 0 naive, 1 opt. fuse: 1 selects the fused decode path (the persistent
 * decode-step kernel when matvec and attention are both opt). cuda_graph: replay the step as a CUDA
 * graph. max_seq_len: 0 = the file header's value, else a positive multiple of 128 not above it.
 * matvec_rpb: 0 = default, else 1, 2, 4 or 8 = the most weight rows a consumer warp takes per tile. */
typedef struct {
    int matvec_impl;
    int attn_impl;
    int fuse;
    int cuda_graph;
    int max_seq_len;
    int matvec_rpb;
} cudallm_options;

/* Model description: reference include/cudallm/cudallm.h:27-32. weight_bytes = sum of the nbytes of
 * every tensor in the file, each counted once (the bytes one decode step streams). */
typedef struct {
    int weight_dtype; /* 1 bf16, 3 int8, 4 int4 */
    int hidden, inter, n_layers, n_heads, n_kv_heads, head_dim, vocab, max_seq_len, group_size;
    float rms_eps;
    unsigned long long weight_bytes;
} cudallm_config_info;

/* Replaces reference cudallm.h:34 (thread-local message of the last failure). */
const char* cudallm_last_error(void);
/* Replaces reference cudallm.h:35: fills opt, opt, fuse 1, graph 1, 0, 0. */
void cudallm_default_options(cudallm_options* out);
/* Replaces reference cudallm.h:36: loads a .cudallm file; *out = NULL on failure. */
int cudallm_create(const char* path, const cudallm_options* opts, cudallm_engine** out);
/* Replaces reference cudallm.h:37; NULL-safe. */
void cudallm_destroy(cudallm_engine* e);
/* Replaces reference cudallm.h:38. */
int cudallm_get_config(cudallm_engine* e, cudallm_config_info* out);
/* Replaces reference cudallm.h:39: position back to 0 (KV contents are overwritten as it advances). */
int cudallm_reset(cudallm_engine* e);
/* Replaces reference cudallm.h:40: host mirror of the position; -1 for a NULL engine. */
int cudallm_pos(cudallm_engine* e);
/* Replaces reference cudallm.h:41. token >= 0 is fed; -1 feeds the previous step's device argmax.
 * logits_out: host [vocab] or NULL; next_token_out: host or NULL. With both NULL the call does not
 * synchronise (steps queue asynchronously on the engine's stream). */
int cudallm_step(cudallm_engine* e, int token, float* logits_out, int* next_token_out);
/* Replaces reference cudallm.h:42. Never uses a CUDA graph; residuals_out: host [(n_layers+1)*hidden],
 * the residual stream after the embedding and after each layer. */
int cudallm_step_debug(cudallm_engine* e, int token, float* residuals_out, float* logits_out, int* next_token_out);

/* ---- single-kernel test hooks: host pointers in/out; each call allocates, uploads, runs on the
 * default stream, synchronises, downloads and frees (reference cudallm.h:44-56, cudallm_capi.cpp:179-316). */

/* Replaces reference cudallm.h:45-48. impl 0 naive (bf16, STORE, no norm), 1 opt. weight_dtype 1/3/4;
 * epilogue 0 STORE, 1 ADD (y += W x), 2 SWIGLU (y[r] = silu(g_r) u_r, rows/2 outputs). */
int cudallm_kernel_matvec(int impl, int weight_dtype, int epilogue, int fuse_norm, int rpb,
                          const void* w, unsigned long long w_bytes, const void* scales, unsigned long long scales_bytes,
                          const float* x, const float* norm_w, float eps,
                          float* y /* in/out (ADD reads it) */, int rows, int cols);
/* Replaces reference cudallm.h:49. */
int cudallm_kernel_rmsnorm(const float* x, const float* w, float eps, float* y, int n);
/* Replaces reference cudallm.h:50-52. Caches are fp16 bits [nkv][max_seq][hd]. */
int cudallm_kernel_rope_kv(int fused, float* qkv /* in/out */, const float* inv_freq, int pos,
                           unsigned short* k_cache, unsigned short* v_cache, int nh, int nkv, int hd, int max_seq);
/* Replaces reference cudallm.h:53-54. impl 1 requires max_seq % 128 == 0, nh == 4*nkv, hd == 64. */
int cudallm_kernel_attention(int impl, const float* q, const unsigned short* k_cache, const unsigned short* v_cache,
                             int ctx, float* out, int nh, int nkv, int hd, int max_seq);
/* Replaces reference cudallm.h:55. */
int cudallm_kernel_silu_mul(const float* gu, float* act, int inter);
/* Replaces reference cudallm.h:56. Lowest index wins ties. */
int cudallm_kernel_argmax(const float* logits, int n, int* out_idx);

/* ================================ additive (no counterpart in the reference ABI) ================ */

#define CUDALLM_KV_FP16 0
#define CUDALLM_KV_BF16 1

#define CUDALLM_PATH_AUTO 0       /* persistent decode-step kernel when fuse=1 and both impls are opt */
#define CUDALLM_PATH_PERSISTENT 1 /* force the persistent decode-step kernel (needs fuse=1, opt/opt) */
#define CUDALLM_PATH_PER_OP 2     /* one kernel per operation, as the reference sequences them */

/* Extended creation options. struct_size must be sizeof(cudallm_options_ex). */
typedef struct {
    int struct_size;
    int kv_dtype; /* CUDALLM_KV_FP16 (reference default, engine.cpp:51-52) or CUDALLM_KV_BF16 */
    int device;   /* CUDA device ordinal; -1 = the calling thread's current device */
    int path;     /* CUDALLM_PATH_* */
    int reserved[4];
} cudallm_options_ex;

/* Fills kv fp16, device -1, path auto. */
void cudallm_default_options_ex(cudallm_options_ex* out);
/* cudallm_create with extended options (ex may be NULL = defaults). */
int cudallm_create_ex(const char* path, const cudallm_options* opts, const cudallm_options_ex* ex, cudallm_engine** out);
/* Waits for every queued step; reports a device-side failure (e.g. a timed-out inter-block wait). */
int cudallm_synchronize(cudallm_engine* e);
/* Prompt prefill: feeds tokens[0..n) (host) at positions pos .. pos+n-1, with the results of n calls of
 * cudallm_step(e, tokens[i], NULL, NULL) up to fp32 summation order, 64 tokens per batched tensor-core step
 * (a batched engine with its own copy of the weights is created on the first call and writes this engine's
 * KV cache; int8 weights step the tokens through the decode path). Afterwards cudallm_pos advanced by n,
 * *next_token_out (or NULL) is the argmax after tokens[n-1], logits_out (host [vocab], or NULL) its logits,
 * and cudallm_step(e, -1, ...) continues from that argmax. n must fit in max_seq_len (else STATE).
 * Synchronises. No counterpart in the reference, which feeds prompts one cudallm_step at a time. */
int cudallm_prefill(cudallm_engine* e, const int* tokens, int n, float* logits_out, int* next_token_out);
/* Which decode path the engine runs: CUDALLM_PATH_PERSISTENT or CUDALLM_PATH_PER_OP. */
int cudallm_engine_path(cudallm_engine* e);
/* The engine's CUDA stream (a cudaStream_t) and device, so callers can order or time work against the
 * steps it enqueues; NULL / -1 for a NULL engine. */
void* cudallm_engine_stream(cudallm_engine* e);
int cudallm_engine_device(cudallm_engine* e);
/* Step tracing (persistent path only): enable = 1 makes every following step record, per CTA, the
 * %globaltimer value (ns) at each operation's dependency-wait begin / end, its end, and when the
 * producer warp starts streaming its weights; 0 turns it off. */
int cudallm_debug_trace(cudallm_engine* e, int enable);
/* Copies the last traced step: grid x slots per-CTA values followed by 256 x 5 stamps of 256 consecutive
 * tiles of CTA 0 (from the first tile of the weight operation the "trace_tile_op" knob names, by default the
 * lm_head); count >= grid*slots + 1280. *grid_out, *slots_out get the shape. Waits for queued work. */
int cudallm_debug_read_trace(cudallm_engine* e, unsigned long long* out, unsigned long long count, int* grid_out,
                             int* slots_out);
/* Sets a tuning or test knob of the persistent decode path by name; CUDALLM_ERR_INVALID_ARG for an unknown
 * name, a value out of range, or a per-op engine. Knobs: "wait_limit_ns" (bound of every inter-block wait of
 * the step, 1 .. 1e10; default 1e9; a step whose wait runs out returns CUDALLM_ERR_STATE and leaves the
 * position unchanged), "prefetch_tiles" (L2 prefetch distance of the weight stream, 0 .. 1024),
 * "whole_head_max_tiles" (contexts up to this many 64-token tiles attend with one block per KV head, longer
 * ones split each head's context over many blocks, 0 .. max_seq_len/64; default 6, int4 weights 8), "trace_tile_op" (weight operation whose tiles the trace stamps, 0 .. 64),
 * "stall_op" (for tests of the failure path: the blocks computing weight operation k, 1 .. 64, wait for an
 * input that is never written, so every such wait runs out after wait_limit_ns and the step fails with
 * CUDALLM_ERR_STATE; -1 = off, the default). */
int cudallm_debug_set(cudallm_engine* e, const char* knob, long long value);

/* Next-token rule of the following steps (no counterpart in the reference, which decodes greedily:
 * src/kernels/argmax.cu). temperature 0 (the default) = argmax, lowest index on ties. temperature > 0 =
 * sampling: the top_k largest logits (1 .. 64; 0 = 64; ties to the lower index) are weighted by
 * exp((logit - max) / temperature); the nucleus is the shortest prefix of them, in descending order, whose
 * weight reaches top_p (0 < top_p <= 1) of their total; the token is drawn from it with a uniform number
 * that depends only on (seed, position), so a rerun reproduces the tokens. The `next` output of
 * cudallm_step and the token fed by cudallm_step(e, -1, ...) are the drawn token; logits are unchanged.
 * Persistent decode path only (INVALID_ARG on a per-op engine with temperature > 0). */
int cudallm_set_sampling(cudallm_engine* e, float temperature, int top_k, float top_p, unsigned long long seed);

/* ---- batched decode (no counterpart in the reference, whose engine holds one sequence): up to 64
 * independent sequences decoded together on one GPU, one token each per step; every row runs the
 * reference engine's per-token sequence (src/engine/engine.cpp:181-237) on its own token, position and KV
 * cache, with the weight matvecs as tensor-core GEMMs (bf16 or int4 weights). Several GPUs: one batch engine per
 * device (device field), each on its own sequences; no communication between them. */
typedef struct cudallm_batch cudallm_batch;

typedef struct {
    int struct_size; /* sizeof(cudallm_batch_options) */
    int n_seq;       /* 1..64 */
    int max_seq_len; /* 0 = the file header's value, else a positive multiple of 128 not above it */
    int kv_dtype;    /* CUDALLM_KV_FP16 or CUDALLM_KV_BF16 */
    int device;      /* CUDA device ordinal; -1 = the calling thread's current device */
    int cuda_graph;  /* 1: replay the step as a CUDA graph */
    int attn_mode;   /* 0 choose by size; 1 one block per (KV head, sequence) streaming the context;
                        2 split over 64-token tiles, merged by a second kernel */
    int reserved[3];
} cudallm_batch_options;

/* Fills n_seq 64, max_seq_len 0, kv fp16, device -1, cuda_graph 1, attn_mode 0. */
void cudallm_default_batch_options(cudallm_batch_options* out);
/* Loads a .cudallm file (bf16 or int4 weights; int8 returns INVALID_ARG) for n_seq sequences; *out = NULL on failure. */
int cudallm_batch_create(const char* path, const cudallm_batch_options* opts, cudallm_batch** out);
/* NULL-safe. */
void cudallm_batch_destroy(cudallm_batch* e);
/* As cudallm_get_config; max_seq_len is the engine's. */
int cudallm_batch_get_config(cudallm_batch* e, cudallm_config_info* out);
/* seq in [0, n_seq): that sequence's position back to 0; seq = -1: every sequence. */
int cudallm_batch_reset(cudallm_batch* e, int seq);
/* Host mirror of sequence seq's position; -1 for a NULL engine or an index out of range. */
int cudallm_batch_pos(cudallm_batch* e, int seq);
/* One decode step of every sequence. tokens: host [n_seq], tokens[b] >= 0 is fed to sequence b, -1 feeds
 * b's previous argmax; NULL = all -1. next_out: host [n_seq] (each row's argmax, lowest index on ties) or
 * NULL; logits_out: host [n_seq][vocab] or NULL. With both outputs NULL the call does not synchronise.
 * Every sequence must have room (pos < max_seq_len), else CUDALLM_ERR_STATE and nothing runs. */
int cudallm_batch_step(cudallm_batch* e, const int* tokens, int* next_out, float* logits_out);
/* Waits for every queued step; reports a device-side failure. */
int cudallm_batch_synchronize(cudallm_batch* e);
/* Prompt prefill of sequence seq (engines of n_seq 64): tokens[0..n) at that sequence's positions pos ..
 * pos+n-1, 64 per batched step, every row of a step one position of that sequence. The other sequences keep
 * their positions and previous argmax. next_token_out / logits_out (host, or NULL) as in cudallm_prefill.
 * Synchronises. */
int cudallm_batch_prefill(cudallm_batch* e, int seq, const int* tokens, int n, float* logits_out, int* next_token_out);
/* The engine's CUDA stream (a cudaStream_t); NULL for a NULL engine. */
void* cudallm_batch_stream(cudallm_batch* e);
/* Tuning knobs of the batched step by name (CUDALLM_ERR_INVALID_ARG when unknown or out of range): "pdl"
 * (0/1: programmatic dependent launch between the step's kernels), "ksplit_qkv", "ksplit_wo",
 * "ksplit_gate_up", "ksplit_down" (K split of that GEMM, 1 .. min(16, k/64); int4 k/128). The next step
 * captures its graph again. _get reads them back, and "attn_stream" (1 = streaming attention in use). */
int cudallm_batch_debug_set(cudallm_batch* e, const char* knob, long long value);
int cudallm_batch_debug_get(cudallm_batch* e, const char* knob, long long* value_out);

/* Test hook of the batched path (no counterpart in the reference): tensor-core GEMM y[b][j] (+)= sum_k
 * (x[b][k] + x_lo[b][k]) * w[j][k] for b < batch (1..64), w [n][k], x and x_lo [batch][k] bf16 bits (x_lo
 * may be NULL = zeros; the engine passes an fp32 activation as its bf16 rounding plus the bf16 rounding of
 * the remainder), fp32 result, the 64-column K chunks split evenly over `ksplit` CTA rows (k a multiple of
 * 64, ksplit <= k / 64). epilogue 0 stores, 1 adds to y, 2 applies SwiGLU (y is [batch][n/2]: silu(gate) *
 * up, gate rows first). Host pointers; allocates, runs on the default stream and synchronises like the
 * other hooks. */
int cudallm_kernel_gemm(const unsigned short* w, const unsigned short* x, const unsigned short* x_lo, float* y, int n, int k,
                        int batch, int ksplit, int epilogue);

/* No counterpart in the reference. Split-K decode attention (the kernels behind
 * cudallm_kernel_attention impl 1) for callers that cannot allocate device memory: code whose device
 * memory is owned by another runtime's pool, or loops that must not enter the driver's allocator.
 * Every argument is caller-owned DEVICE memory: q [nh*hd] fp32, k_cache / v_cache [nkv][max_seq][hd]
 * fp16 bits (16-byte aligned), out [nh*hd] fp32; ctx in [1, max_seq]; stream a cudaStream_t (NULL = the
 * legacy default stream). The call only enqueues work on stream; it allocates nothing. The split-K
 * partials live in one fixed device array of 1.03 MiB that every GPU loading the library holds until
 * exit, so nh <= 32 and max_seq <= 8192 (and nh == 4*nkv, hd == 64, max_seq % 128 == 0); larger sizes
 * return CUDALLM_ERR_INVALID_ARG. All calls share that array and it keeps the last call's contents, so
 * calls whose GPU work overlaps (other streams or threads, same device) race: order them on one stream.
 * The first call on each device, with that device current, looks up the array's device address
 * (cudaGetSymbolAddress) and keeps it for the life of the process; make that first call before any stream
 * capture that includes this function. A cudaDeviceReset of that device invalidates the kept address:
 * call this function no more on a device that was reset while the library stayed loaded. */
int cudallm_attention_noalloc(const float* q, const unsigned short* k_cache, const unsigned short* v_cache, int ctx,
                              float* out, int nh, int nkv, int hd, int max_seq, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CUDALLM_B200_CUDALLM_H */
