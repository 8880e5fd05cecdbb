// Per-row kernels of the batched decode step (kernels/batch_ops.cu): row b = sequence b. GEMM operands are
// written as activation planes [2][kBatchMax][n] bf16 (hi, lo; see launch_gemm_bf16). pdl: launch with the
// programmatic-dependent-launch attribute (every kernel here waits for its predecessor before reading).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace cudallm {

// Row b's token t = tok_in[b] when >= 0, else tok[b] (the previous argmax); x[b][:] = embedding row t
// (bf16 weights, or with emb_scales int4 codes re-packed by interleave_int4_codes and fp16 group scales),
// planes of x[b][j] * gain[j] and ssq[b] = sum_j x[b][j]^2 (the first RMSNorm's input and statistics, ssq
// as one [1][64] partial).
void launch_embed_rows(const void* emb, const __half* emb_scales, const int* tok_in, const int* tok, const float* gain,
                       float* x, __nv_bfloat16* planes, float* ssq, int batch, int hidden, cudaStream_t stream,
                       bool pdl = false);
// tok[b] = the best of the per-tile argmax partials am_v / am_i [batch][n_tiles] of row b (lowest index on
// ties), pos[b] += 1.
void launch_argmax_tiles(const float* am_v, const int* am_i, int n_tiles, int* tok, int* pos, int batch, cudaStream_t stream,
                         bool pdl = false);
// out planes of rmsnorm(x[b][:]) * w.
void launch_rmsnorm_rows(const float* x, const float* w, float eps, __nv_bfloat16* out, int batch, int n, cudaStream_t stream,
                         bool pdl = false);
// Rotates the q heads of every row in place and writes the rotated k and the v of row b into sequence b's
// cache ([nkv][max_seq][hd] at k_cache + b * seq_stride) at position pos[b].
template <typename KV>
void launch_rope_kv_rows(float* qkv, const float* inv_freq, KV* k_cache, KV* v_cache, size_t seq_stride, const int* pos,
                         int batch, int nh, int nkv, int hd, int max_seq, cudaStream_t stream, bool pdl = false);
// Split-K GQA attention of every row over its own context (pos[b] + 1 tokens; max_ctx >= the largest sets
// the grid): out = attention output planes [2][kBatchMax][nh * 64]. Partials: [batch][nh][max_seq/64][64]
// and [...][2].
template <typename KV>
void launch_attention_rows(const float* qkv, const KV* k_cache, const KV* v_cache, size_t seq_stride, const int* pos,
                           int max_ctx, float* part_o, float* part_ml, __nv_bfloat16* out, int batch, int nh, int nkv,
                           int max_seq, cudaStream_t stream, bool pdl = false);
// The same attention as launch_attention_rows, one CTA per (KV head, row) streaming the row's whole
// context through shared memory (bulk async copies); no partials. err: device word, bit 1 set if a
// bounded wait for a copy gave up. Caches 16-byte aligned. one_seq: every row is one position of the same
// sequence (seq_stride 0, positions increasing from row 0: a prefill chunk), so a row reads the keys and
// values its predecessors in the chunk wrote in this step.
template <typename KV>
void launch_attention_rows_stream(const float* qkv, const KV* k_cache, const KV* v_cache, size_t seq_stride, const int* pos,
                                  __nv_bfloat16* out, int batch, int nh, int nkv, int max_seq, unsigned* err,
                                  cudaStream_t stream, bool pdl = false, bool one_seq = false);
// tok[b] = argmax of logits row b (lowest index on ties), pos[b] += 1. Each row is split over
// kArgmaxSplit blocks; scratch_v / scratch_i hold [batch][kArgmaxSplit] slice results and ticket [batch]
// counters that must be zero before the first launch (each launch leaves them zero).
constexpr int kArgmaxSplit = 16;
void launch_argmax_rows(const float* logits, int n, float* scratch_v, int* scratch_i, unsigned* ticket, int* tok, int* pos,
                        int batch, cudaStream_t stream, bool pdl = false);

}  // namespace cudallm
