// Persistent decode-step kernel: one cooperative launch computes a whole Llama-3.2-1B token step
// (embedding -> 16 x [QKV, RoPE + KV write + split-K GQA attention, O proj + residual, RMSNorm +
// gate/up + SwiGLU, down + residual] -> final RMSNorm + tied lm_head -> argmax) on one CTA per SM.
// It replaces the 116-launch graph of wasiqnauman/cudallm src/engine/engine.cpp:181-237 for the
// fused opt/opt path.
//
// Inside the kernel, warp 0 of every CTA streams that CTA's share of every weight matrix, in use
// order, through a ring of shared-memory stages with bulk (TMA) copies, and prefetches the head of
// the next operation into L2; it never waits for activations, so HBM keeps streaming while the 8
// consumer warps wait on inter-CTA dependencies. Dependencies are monotonic per-step counters in
// global memory (release add / acquire load), every wait is bounded by a wall-clock limit after
// which the kernel records an error code and exits cleanly, and the last CTA to finish the lm_head
// reduces the argmax, advances the device position and zeroes the counters for the next step.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common/dtype.h"
#include "kernels/kernels.h"
#include "kernels/sampling.cuh"

namespace cudallm {

// Most weight rows in one tile (one ring stage) of the persistent kernel. bf16 / int8 tiles are one consumer
// warp's work. int4 stages are shared: a 16 KiB stage holds 16 rows of a 2048-column matrix and each of the
// 8 consumer warps takes 2 of them (the down projection: 4 rows of 8192 columns, one per warp, two warp
// groups alternating stages), so the ring keeps full 16 KiB stages in flight while every warp has work
// even in the small operations.
__host__ __device__ constexpr int decode_step_tile_rows(WeightType) { return kMaxTileRows; }
// Longest row segment of the down projection's tiles (K = 8192). At 16 KiB every type keeps whole rows
// (bf16: 1 row per stage, int8: 2, int4: 4). Shorter segments (more rows per stage, each input column read
// from shared memory serving more rows) were measured slower: a warp then walks a row group's segments in
// sequence and fewer warps share the operation.
constexpr int kDownSegBytes = 16384;

struct StepLayer {
    const float* attn_norm;
    const void* wqkv;
    const void* sqkv;
    const void* wo;
    const void* so;
    const float* ffn_norm;
    const void* wgu;
    const void* sgu;
    const void* wdown;
    const void* sdown;
};

constexpr int kStepLayers = 16;
// Largest grid whose lm_head candidates the persistent step's last CTA can hold when sampling.
constexpr int kSampleMaxGrid = 160;

// Trace layout per CTA: operation k (layer l: 5l + {0 qkv, 1 attention, 2 o-proj, 3 gate/up, 4 down};
// 80 lm_head; 81 step end) has kTraceStamps slots: 0 dependency wait begins, 1 wait ends, 2 operation
// ends, 3 producer starts issuing its tiles, 4 input vector staged, 5 consumer warp 0 done with its
// first tile (3-5: weight operations only); slot 3 of entry 81 holds the CTA's SM id.
constexpr int kTraceOps = 82;
constexpr int kTraceStamps = 6;
constexpr int kTraceSlots = kTraceOps * kTraceStamps;
// After the per-CTA slots: kTraceTiles tiles of CTA 0's tile stream starting at global tile index
// StepParams::trace_t0, 5 stamps each: producer issues the copy, consumer starts waiting for it, the data
// is there, consumer is done with the tile, the prefetch warp has issued its L2 prefetch.
constexpr int kTraceTiles = 256;
constexpr int kTraceTileStamps = 5;
inline constexpr size_t trace_words(int grid) {
    return static_cast<size_t>(grid) * kTraceSlots + kTraceTiles * kTraceTileStamps;
}

// Device error word layout (err[0] = flags, err[1] = id of the first wait that gave up).
constexpr unsigned kErrWaitTimeout = 1u;
constexpr unsigned kErrAborted = 2u;

// Attention past whole_head_max_tiles: every KV head's context is cut into S <= kAttnMaxSplits ranges of
// 128-token passes, one CTA per (head, range), and one further CTA per head merges the S partials
// (O[64], M, L per query head, in part_o / part_ml at slot = range) in range order. A range CTA publishes
// its partials by a release store of this step's tag into its flag word (sync[kSyncFlags + 32 h + range]);
// the merging CTA acquires the S flags, then reads the partials.
constexpr int kAttnMaxSplits = 17;

// Words the step uses (zeroed at creation, after an error and by the step itself at its end): the split
// attention's per-(KV head, range) flags and the lm_head ticket. Activations between operations
// are synchronised through their tags, not counters.
constexpr int kSyncFlags = 0, kSyncLm = 8 * 32, kSyncWords = 512;

struct StepParams {
    StepLayer layers[kStepLayers];
    const void* emb_w;
    const void* emb_s;
    const float* final_norm;
    const float* inv_freq;
    // Activations exchanged between CTAs, each element a (value, tag) word: tag = step << 8 | layer << 3 |
    // kind (decode_step.cu), so a reader polls the data itself instead of a counter.
    unsigned long long* t_qkv;   // [3072] q | k | v projections
    unsigned long long* t_att;   // [2048] attention output
    unsigned long long* t_xmid;  // [2048] residual after the O projection
    unsigned long long* t_xout;  // [2048] residual after the down projection
    unsigned long long* t_act;   // [8192] SwiGLU output
    unsigned step_tag;           // this launch's step number (1 .. 2^24 - 1)
    float* logits;  // [128256]
    void* k_cache;  // [16][8][max_seq][64]
    void* v_cache;
    float* part_o;   // [32][max_seq/64][64]
    float* part_ml;  // [32][max_seq/64][2]
    float* am_v;     // [grid]
    int* am_i;       // [grid]
    int* d_token;
    int* d_pos;
    unsigned* sync;  // [kSyncWords]
    unsigned* err;   // [2]
    float* debug_res;  // [(16+1)][2048] or null
    unsigned long long* trace;  // [grid][kTraceSlots] %globaltimer stamps, or null
    int token_override;  // >= 0: feed this token instead of *d_token
    int max_seq;
    float eps;
    int group_size;
    unsigned long long wait_limit_ns;   // bound of every dependency wait (error + clean exit after it)
    unsigned long long drain_limit_ns;  // bound of the producer's final wait for its copies in flight
    int prefetch_tiles;  // L2 prefetch distance of the weight stream, in tiles beyond the copies
    int prefetch_mode;   // 0 none, 2 prefetch warp (load/store-unit prefetch instructions), 3 same warp, bulk prefetches
    int whole_head_max_tiles;  // contexts up to this many 64-token tiles use one CTA per KV head for attention
    int trace_t0;        // first stamped tile (global index in CTA 0's tile stream)
    int stall_op;        // test only, -1 = off: the consumers of weight operation k (k >= 1) wait for an input
                         // tag that nothing writes, so every CTA's wait runs out after wait_limit_ns
    // Next-token choice: temperature 0 = greedy (argmax, the reference's rule); > 0 = sampling from the top
    // sample_top_k (1..64) logits, nucleus sample_top_p, draw sample_seed at the current position. cand:
    // [grid][64] candidate keys (each CTA's top k), used only when sampling.
    float sample_temperature;  // (sampling needs grid <= kSampleMaxGrid and <= kSampleMaxGrid * 64 rows per CTA)
    float sample_top_p;
    int sample_top_k;
    unsigned long long sample_seed;
    unsigned long long* cand;
    TileGeom g_qkv, g_wo, g_gu, g_down, g_lm;
};

// Shared memory bytes of one CTA of the persistent kernel.
int decode_step_smem_bytes();
// Prepares (once per device) and launches one step on `stream` as a cooperative launch with one CTA
// per SM. Throws if the device cannot hold the grid. split: launch the instantiation whose attention cuts
// a context into ranges over many CTAs (for contexts past whole_head_max_tiles tiles); the other gives each
// KV head one CTA. Both compute every context length correctly; the choice only affects speed.
void launch_decode_step(const StepParams& p, WeightType wt, KvType kv, bool split, cudaStream_t stream);
// Grid size the launch uses (the number of SMs).
int decode_step_grid();

}  // namespace cudallm
