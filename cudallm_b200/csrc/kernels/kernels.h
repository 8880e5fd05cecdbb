// Host launchers for the per-operation sm_100a kernels. Counterpart of wasiqnauman/cudallm
// src/kernels/kernels.h:13-44 (same operations, same device-side position/token convention so every
// launch can be captured in a CUDA graph). All launchers validate their arguments and throw.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "common/dtype.h"
#include "model/weights.h"

namespace cudallm {

enum class Epilogue : int { STORE = 0, ADD = 1, SWIGLU = 2 };

// Split-K attention granularity of the reference ABI (cudallm_kernel_attention impl=1 requires
// max_seq % 128 == 0); the kernels themselves split the context into kAttnTile-token chunks.
constexpr int kAttnAbiChunk = 128;
constexpr int kAttnTile = 64;
constexpr int kArgmaxBlocks = 296;  // 2 x 148 SMs

// Weight tiles are streamed through shared memory in stages of this size.
constexpr int kStageBytes = 16 * 1024;
constexpr int kMaxTileRows = 16;

struct MatvecArgs {
    const void* w = nullptr;
    const void* scales = nullptr;
    const float* x = nullptr;
    const float* norm_w = nullptr;  // fused RMSNorm gain, or null
    float eps = 0.f;
    float* y = nullptr;
    int rows = 0, cols = 0;
};

// Tile shape of one weight operation (host-computed, identical in every kernel that streams it).
struct TileGeom {
    int out_rows;   // outputs (rows/2 for SWIGLU)
    int cols;
    int row_bytes;  // bytes of one stored row
    int seg_bytes;  // bytes of the row segment one tile holds (divides row_bytes, multiple of 512)
    int n_seg;      // row_bytes / seg_bytes
    int rows_per_tile;
    int halves;     // 2 for SWIGLU (gate rows then up rows in one stage), else 1
};
// seg_cap > 0 caps the row segment of a tile at that many bytes (a multiple of 512), so that a tile holds
// more rows of a long row.
TileGeom make_tile_geom(WeightType wt, Epilogue ep, int rows, int cols, int rpb, int seg_cap = 0);

int num_sms();
int default_rpb(WeightType w);

void launch_embedding(const Linear& emb, const int* d_token, float* x, int hidden, int group_size, cudaStream_t);
void launch_rmsnorm(const float* x, const float* w, float eps, float* y, int n, cudaStream_t);
void launch_matvec_naive(const MatvecArgs&, cudaStream_t);
// err: device word that receives a nonzero code if a bounded in-kernel wait gives up (null = the
// process-wide word checked by check_kernel_error()).
void launch_matvec_stream(WeightType, Epilogue, bool fuse_norm, const MatvecArgs&, int rpb, cudaStream_t,
                          unsigned* err = nullptr);
// Reads and clears the process-wide kernel error word; throws StateError if a wait gave up.
void check_kernel_error();

template <typename KV>
void launch_rope_inplace(float* qkv, const float* inv_freq, const int* d_pos, int nh, int nkv, int hd, cudaStream_t);
template <typename KV>
void launch_kv_write(const float* qkv, KV* k_cache_l, KV* v_cache_l, const int* d_pos, int nh, int nkv, int hd, int max_seq,
                     cudaStream_t);
template <typename KV>
void launch_rope_kv_fused(float* qkv, const float* inv_freq, KV* k_cache_l, KV* v_cache_l, const int* d_pos, int nh, int nkv,
                          int hd, int max_seq, cudaStream_t);
template <typename KV>
void launch_attention_naive(const float* q, const KV* k_l, const KV* v_l, const int* d_pos, float* out, int nh, int nkv,
                            int hd, int max_seq, cudaStream_t);
// Split-K GQA attention: partials [nh][max_seq/kAttnTile][hd] and [nh][max_seq/kAttnTile][2].
template <typename KV>
void launch_attention_split(const float* q, const KV* k_l, const KV* v_l, const int* d_pos, float* part_o, float* part_ml,
                            float* out, int nh, int nkv, int hd, int max_seq, cudaStream_t);

void launch_add_inplace(float* x, const float* y, int n, cudaStream_t);
void launch_silu_mul(const float* gu, float* act, int inter, cudaStream_t);
void launch_set_token(int* d_token, int token, cudaStream_t);
// Deterministic argmax (lowest index on ties); writes *d_token and increments *d_pos.
void launch_argmax(const float* logits, int n, float* part_v, int* part_i, int* d_token, int* d_pos, cudaStream_t);

// HBM bandwidth probes (kernels/hbm_probe.cu). sink: probe_grid() * 256 words for the plain probes,
// num_sms() * 256 for the bulk read; err: a device word set when a bounded wait of the bulk read gave up.
int probe_grid();
void launch_bw_read(const uint4* src, size_t n_uint4, unsigned* sink, int grid, cudaStream_t);
void launch_bw_write(uint4* dst, size_t n_uint4, int grid, cudaStream_t);
void launch_bw_copy(const uint4* src, uint4* dst, size_t n_uint4, int grid, cudaStream_t);
size_t bulk_probe_chunk_bytes();
void launch_bw_bulk_read(const void* src, size_t bytes, unsigned* sink, unsigned* err, cudaStream_t);
// Bulk copies of `bytes` (re-read `reps` times) through a 12-stage ring per SM with per-stage producer lanes
// and 8 consumer warps; returns the bytes one launch moves. sink: num_sms() * 256 words.
size_t launch_bw_bulk_ring(const void* src, size_t bytes, int reps, unsigned* sink, unsigned* err, cudaStream_t);

}  // namespace cudallm
