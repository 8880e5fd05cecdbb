// Batched decode: tensor-core GEMM with fused epilogues, and the per-row kernels around it (batch of
// independent sequences, one row per sequence).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace cudallm {

constexpr int kBatchMax = 64;
constexpr int kGemmTileRows = 128;  // weight rows per CTA

enum class GemmEpilogue : int { STORE = 0, ADD = 1, SWIGLU = 2, QKV_ROPE = 3, LOGITS = 4 };

// What a fused GEMM does with s[b][j] = sum_k x[b][k] * w[j][k] (all K splits added, in split order).
// Every output of row b is first multiplied by inv_rms[b] = 1 / sqrt(sum_i ssq_in[i][b] / norm_n + eps)
// (i < ssq_count, summed in order) when ssq_in is set: the RMSNorm of the GEMM input, whose gain was
// already applied when the activation planes were written.
struct GemmEpi {
    GemmEpilogue kind = GemmEpilogue::STORE;
    const float* ssq_in = nullptr;  // [ssq_count][64], ssq_count <= 16
    int ssq_count = 0;
    int norm_n = 0;
    float eps = 0.f;
    // STORE / LOGITS: y[b][j] = v. ADD: y[b][j] += v (the residual stream). SWIGLU: y[b][f] (optional) =
    // silu(gate) * up for the f-th output (the weight rows interleaved by interleave_gate_up).
    float* y = nullptr;
    // ADD: planes of y_new[b][j] * gain[j] (the next RMSNorm's input); SWIGLU: planes of the outputs.
    // Activation planes are [2][64][cols] bf16: hi = bf16(v), lo = bf16(v - hi).
    __nv_bfloat16* planes = nullptr;
    const float* gain = nullptr;
    // ADD: partial sums of y_new^2 per row, one per 128-row tile: [n_tiles][64] (at most 16 tiles feed a
    // later ssq_in).
    float* ssq_out = nullptr;
    // QKV_ROPE: rows are [q heads | k heads | v heads] x 64 dims. q heads are rotated and stored in q_out
    // ([b][(nh + 2 nkv) * 64], q part only); k heads are rotated, v heads copied, both rounded to the cache
    // type and written to row b's cache (k_cache / v_cache + b * seq_stride, [nkv][max_seq][64]) at pos[b].
    float* q_out = nullptr;
    const float* inv_freq = nullptr;
    void* k_cache = nullptr;
    void* v_cache = nullptr;
    size_t seq_stride = 0;
    const int* pos = nullptr;
    int nh = 0, nkv = 0, max_seq = 0;
    bool kv_bf16 = false;
    // LOGITS: per 128-row tile t, the largest scaled output of row b and its index (lowest on ties):
    // am_v / am_i [64][n_tiles].
    float* am_v = nullptr;
    int* am_i = nullptr;
};

// K split for an n x k GEMM: the most grid rows (up to 16) that keep every SM busy with one CTA and
// that the device can hold as clusters (the CTAs of one 128-row tile form a cluster and add their
// partial sums through distributed shared memory).
int gemm_pick_ksplit(int n, int k);

// Fused batched GEMM: w [n][k] bf16 row-major (for SWIGLU in the interleaved gate/up layout); x the
// activation planes [2][kBatchMax][k] (rows >= batch ignored); batch 1..64; k % 64 == 0; 1 <= ksplit <=
// min(16, k / 64); LOGITS needs ksplit 1. err: device word, bit 0 set if a bounded wait gave up. pdl:
// programmatic dependent launch (the weight stream starts before the previous kernel ends).
void launch_gemm(const __nv_bfloat16* w, int n, int k, const __nv_bfloat16* x, int batch, int ksplit, const GemmEpi& epi,
                 unsigned* err, cudaStream_t stream, bool pdl = false);

// The same GEMM over int4 weights in the .cudallm layout (codes [n][k/2], two per byte, value (u - 8) *
// scale; fp16 scales [n][k/128]) after interleave_int4_codes has re-packed the codes. k % 128 == 0,
// ksplit <= min(16, k / 128) (K splits fall on 128-column groups).
void launch_gemm_int4(const uint8_t* codes, const __half* scales, int n, int k, const __nv_bfloat16* x, int batch, int ksplit,
                      const GemmEpi& epi, unsigned* err, cudaStream_t stream, bool pdl = false);
int gemm_pick_ksplit_int4(int n, int k);

// In place, every 32-bit word of int4 codes: byte j = columns (2j, 2j+1) -> byte j = columns (j, j+4)
// of the word's 8 columns (low nibble first). launch_gemm_int4 and the batched embedding read this form.
void interleave_int4_codes(void* codes, size_t bytes, cudaStream_t stream);

// dst = the gate/up matrix [2 * inter][k] (gate rows, then up rows) with rows reordered so that every
// 128-row tile t holds gate rows 64t..64t+63 followed by up rows 64t..64t+63 (inter % 64 == 0).
void interleave_gate_up(const __nv_bfloat16* src, __nv_bfloat16* dst, int inter, int k, cudaStream_t stream);
// The same row order for any per-row data of row_bytes bytes (a multiple of 16): int4 codes, group scales.
void interleave_gate_up_rows(const void* src, void* dst, int inter, int row_bytes, cudaStream_t stream);

}  // namespace cudallm
