// Persistent decode-step kernel (see decode_step.h for the design). Operation order and arithmetic
// follow wasiqnauman/cudallm src/engine/engine.cpp:181-237 (fused path) and
// python/cudallm/reference.py:123-158; the work decomposition is this engine's own.
#include "engine/decode_step.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>

#include "common/check.h"
#include "kernels/attention_core.cuh"
#include "kernels/matvec_core.cuh"
#include "kernels/ptx.cuh"

namespace cudallm {

namespace {

constexpr int kCw = 8;             // consumer warps
constexpr int kCt = 32 * kCw;      // consumer threads
constexpr int kThreads = 32 + kCt; // + one producer warp
constexpr int kStages = 11;
constexpr int kMaxK = 8192;
constexpr int kPrefetchBytes = 192 * 1024;
constexpr int kOpsPerLayer = 4;
constexpr int kWeightOps = kStepLayers * kOpsPerLayer + 1;  // + tied lm_head
constexpr int kH = 2048, kNh = 32, kNkv = 8;

enum OpKind : int { kQkv = 0, kWo = 1, kGu = 2, kDown = 3, kLm = 4 };

struct Flags {
    int abort;
    int ok;
    int role;
    int pad;
};

// Shared-memory layout (byte offsets).
constexpr int kOffBars = 0;
constexpr int kOffFlags = 256;
constexpr int kOffRed = 384;
constexpr int kOffCs = 512;
constexpr int kOffScratch = 768;
constexpr int kOffAm = kOffScratch + kCw * 32 * 4;  // 1792
constexpr int kOffXc = 2048;
constexpr int kOffXp = 3072;
constexpr int kOffRing = kOffXp + kMaxK * 4;  // 35840
constexpr int kSmemBytes = kOffRing + kStages * kStageBytes;
static_assert(2 * kStages * 8 <= kOffFlags, "barriers overflow");
static_assert(kOffAm + kCw * 8 <= kOffXc, "argmax scratch overflow");
static_assert(kOffXc + (kMaxK / 32) * 4 <= kOffXp, "chunk sums overflow");
static_assert(sizeof(AttSmem<__half>) <= kMaxK * 4, "attention scratch must fit in the vector area");
static_assert(kOffRing % 128 == 0, "ring alignment");

struct WOp {
    const uint8_t* w;
    const void* s;
    TileGeom g;
};

__device__ __forceinline__ WOp weight_op(const StepParams& p, int o) {
    if (o == kWeightOps - 1) return {static_cast<const uint8_t*>(p.emb_w), p.emb_s, p.g_lm};
    const StepLayer& L = p.layers[o / kOpsPerLayer];
    switch (o % kOpsPerLayer) {
        case kQkv: return {static_cast<const uint8_t*>(L.wqkv), L.sqkv, p.g_qkv};
        case kWo: return {static_cast<const uint8_t*>(L.wo), L.so, p.g_wo};
        case kGu: return {static_cast<const uint8_t*>(L.wgu), L.sgu, p.g_gu};
        default: return {static_cast<const uint8_t*>(L.wdown), L.sdown, p.g_down};
    }
}

__device__ __forceinline__ void split_rows(int n, int& lo, int& hi) {
    lo = static_cast<int>(static_cast<long long>(blockIdx.x) * n / gridDim.x);
    hi = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * n / gridDim.x);
}

__device__ __forceinline__ int op_tiles(const TileGeom& g, int lo, int hi) {
    const int R = g.rows_per_tile;
    return ((hi - lo + R - 1) / R) * g.n_seg;
}

__device__ __forceinline__ void fail(const StepParams& p, volatile Flags* fl, unsigned code, unsigned id) {
    fl->abort = 1;
    atomicOr(p.err, code);
    atomicCAS(p.err + 1, 0u, id);
}

// Bounded spin until *ctr >= target (acquire). Gives up on timeout or when another CTA reported an
// error; returns false then.
__device__ bool spin_until(const StepParams& p, const unsigned* ctr, unsigned target, volatile Flags* fl, unsigned id) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (ld_acquire_gpu(ctr) >= target) return true;
        if ((it & 31) == 0) {
            if (*reinterpret_cast<volatile unsigned*>(p.err) != 0) {
                fl->abort = 1;
                return false;
            }
            const uint64_t t = global_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > p.wait_limit_ns) {
                fail(p, fl, kErrWaitTimeout, id);
                return false;
            }
        }
        __nanosleep(64);
    }
}

// Bounded wait on an mbarrier phase; also gives up when the CTA aborts (check_abort).
__device__ bool wait_bar(const StepParams& p, uint64_t* bar, uint32_t parity, volatile Flags* fl, bool check_abort,
                         unsigned id) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (check_abort && fl->abort) return false;
            const uint64_t t = global_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > p.wait_limit_ns) {
                fail(p, fl, kErrWaitTimeout, id);
                return false;
            }
        }
    }
}

__device__ void prefetch_head(const StepParams& p, int o) {
    const WOp op = weight_op(p, o);
    int lo, hi;
    split_rows(op.g.out_rows, lo, hi);
    const size_t slice = static_cast<size_t>(hi - lo) * op.g.row_bytes;
    const size_t want = min(slice, static_cast<size_t>(kPrefetchBytes / op.g.halves));
    for (int h = 0; h < op.g.halves; ++h) {
        const uint8_t* base = op.w + (static_cast<size_t>(lo) + static_cast<size_t>(h) * op.g.out_rows) * op.g.row_bytes;
        for (size_t off = 0; off < want; off += 32768) {
            bulk_prefetch_l2(base + off, static_cast<uint32_t>(min(static_cast<size_t>(32768), want - off)));
        }
    }
}

__device__ __forceinline__ void issue_tile(const WOp& op, int lo, int hi, int i, uint8_t* dst, uint64_t* bar, uint64_t pol) {
    const TileGeom& g = op.g;
    const int grp = i / g.n_seg, sg = i % g.n_seg;
    const int r0 = lo + grp * g.rows_per_tile;
    const int nr = min(g.rows_per_tile, hi - r0);
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nr * g.seg_bytes * g.halves));
    for (int h = 0; h < g.halves; ++h) {
        const size_t row = static_cast<size_t>(r0) + static_cast<size_t>(h) * g.out_rows;
        if (g.n_seg == 1) {
            bulk_load(dst + h * nr * g.seg_bytes, op.w + row * g.row_bytes, static_cast<uint32_t>(nr * g.row_bytes), bar, pol);
        } else {
            for (int r = 0; r < nr; ++r) {
                bulk_load(dst + (h * nr + r) * g.seg_bytes, op.w + (row + r) * g.row_bytes + static_cast<size_t>(sg) * g.seg_bytes,
                          static_cast<uint32_t>(g.seg_bytes), bar, pol);
            }
        }
    }
}

// Warp 0, lane 0: streams every tile of the step in order.
__device__ void run_producer(const StepParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty, volatile Flags* fl) {
    const uint64_t pol = l2_policy_evict_first();
    int t = 0;
    bool stop = false;
    prefetch_head(p, 0);
    for (int o = 0; o < kWeightOps && !stop; ++o) {
        if (o + 1 < kWeightOps) prefetch_head(p, o + 1);
        const WOp op = weight_op(p, o);
        int lo, hi;
        split_rows(op.g.out_rows, lo, hi);
        const int nt = op_tiles(op.g, lo, hi);
        for (int i = 0; i < nt; ++i) {
            const int s = t % kStages, k = t / kStages;
            if (k > 0 && !wait_bar(p, &empty[s], (k - 1) & 1, fl, true, 1000u + o)) {
                stop = true;
                break;
            }
            issue_tile(op, lo, hi, i, ring + s * kStageBytes, &full[s], pol);
            ++t;
        }
    }
    // Every issued copy lands before the CTA may exit.
    for (int u = max(0, t - kStages); u < t; ++u) wait_bar(p, &full[u % kStages], (u / kStages) & 1, fl, false, 2000u);
}

template <WeightType WT>
__device__ __forceinline__ float emb_value(const StepParams& p, int tok, int j) {
    if constexpr (WT == WeightType::BF16) {
        return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(p.emb_w) + static_cast<size_t>(tok) * kH + j))
                               << 16);
    } else if constexpr (WT == WeightType::INT8) {
        return static_cast<float>(__ldg(static_cast<const int8_t*>(p.emb_w) + static_cast<size_t>(tok) * kH + j)) *
               __ldg(static_cast<const float*>(p.emb_s) + tok);
    } else {
        const uint8_t b = __ldg(static_cast<const uint8_t*>(p.emb_w) + static_cast<size_t>(tok) * (kH / 2) + j / 2);
        const int q = ((j & 1) ? (b >> 4) : (b & 0x0F)) - 8;
        return static_cast<float>(q) *
               __half2float(__ldg(static_cast<const __half*>(p.emb_s) + static_cast<size_t>(tok) * (kH / p.group_size) +
                                  j / p.group_size));
    }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

struct ConsumerCtx {
    const StepParams* p;
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    volatile Flags* fl;
    float* xp;
    float* xc;
    float* red;
    float* scratch;
    int tid, cw, lane;
    int t_base;  // global tile index of the current operation's first tile
};

__device__ __forceinline__ void csync() { named_barrier(1, kCt); }

// Waits (thread 0) for a dependency; all consumer threads learn the outcome.
__device__ __forceinline__ bool dep_wait(ConsumerCtx& c, const unsigned* ctr, unsigned target, unsigned id) {
    if (c.tid == 0) c.fl->ok = c.fl->abort ? 0 : (spin_until(*c.p, ctr, target, c.fl, id) ? 1 : 0);
    csync();
    const bool ok = c.fl->ok != 0;
    csync();
    return ok;
}

__device__ __forceinline__ void signal(ConsumerCtx& c, unsigned* ctr) {
    csync();
    if (c.tid == 0) {
        __threadfence();
        red_release_gpu_add(ctr, 1u);
    }
}

// Consumes this CTA's tiles of weight operation `o`; applies the epilogue of `kind`.
// LM tracks the best (value, index) per lane in bv/bi. Returns false if the CTA aborted.
template <WeightType WT, int KIND>
__device__ bool run_tiles(ConsumerCtx& c, int o, float& bv, int& bi, int layer) {
    const StepParams& p = *c.p;
    const WOp op = weight_op(p, o);
    const TileGeom& g = op.g;
    constexpr int MAXN = (KIND == kGu ? 2 : 1) * kMaxTileRows;
    int lo, hi;
    split_rows(g.out_rows, lo, hi);
    const int R = g.rows_per_tile;
    const int ng = (hi - lo + R - 1) / R;
    const int nc = g.cols / Chunk<WT>::kCols;
    const int seg_chunks = g.seg_bytes / 16;
    float* my = c.scratch + c.cw * 32;
    bool ok = true;
    for (int grp = c.cw; grp < ng && ok; grp += kCw) {
        const int r0 = lo + grp * R;
        const int nr = min(R, hi - r0);
        const StageRows sr{r0, nr, nr * g.halves, g.out_rows};
        float acc[MAXN];
#pragma unroll
        for (int i = 0; i < MAXN; ++i) acc[i] = 0.f;
        for (int sg = 0; sg < g.n_seg; ++sg) {
            const int t = c.t_base + grp * g.n_seg + sg;
            const int s = t % kStages;
            if (!wait_bar(p, &c.full[s], (t / kStages) & 1, c.fl, true, 3000u + o)) {
                ok = false;
                break;
            }
            tile_accumulate<WT, MAXN>(c.ring + s * kStageBytes, sr, g.seg_bytes, sg * seg_chunks, c.xp, nc, c.xc, op.s, g.cols,
                                      acc, c.lane);
            __syncwarp();
            if (c.lane == 0) mbar_arrive(&c.empty[s]);
        }
        if (!ok) break;
#pragma unroll
        for (int i = 0; i < MAXN; ++i) {
            if (i < sr.n) {
                const float v = warp_sum(acc[i]);
                if (c.lane == 0) my[i] = finish_row<WT>(v, op.s, sr.global_row(i));
            }
        }
        __syncwarp();
        if (c.lane < nr) {
            const int r = r0 + c.lane;
            if constexpr (KIND == kQkv) {
                __stcg(p.qkv + r, my[c.lane]);
            } else if constexpr (KIND == kWo || KIND == kDown) {
                const float v = __ldcg(p.x + r) + my[c.lane];
                __stcg(p.x + r, v);
                if (KIND == kDown && p.debug_res) p.debug_res[static_cast<size_t>(layer + 1) * kH + r] = v;
            } else if constexpr (KIND == kGu) {
                __stcg(p.act + r, silu_f(my[c.lane]) * my[nr + c.lane]);
            } else {
                const float v = my[c.lane];
                __stcg(p.logits + r, v);
                if (better(v, r, bv, bi)) {
                    bv = v;
                    bi = r;
                }
            }
        }
        __syncwarp();
    }
    if (!ok) c.fl->abort = 1;
    c.t_base += op_tiles(g, lo, hi);
    csync();
    return c.fl->abort == 0;
}

template <WeightType WT, typename Src>
__device__ __forceinline__ void stage(ConsumerCtx& c, Src src, int K, const float* norm_w) {
    stage_vector<WT>(src, K, norm_w, c.p->eps, c.xp, c.xc, c.red, c.tid, kCt, [] { csync(); });
}

template <WeightType WT, typename KV>
__device__ void run_consumers(ConsumerCtx& c, float* cs) {
    const StepParams& p = *c.p;
    const int G = gridDim.x;
    const int pos = *p.d_pos;
    const int ctx = pos + 1;
    const int tok = p.token_override >= 0 ? p.token_override : *p.d_token;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    const int n_slots = p.max_seq / kAttnTile;
    rope_table(p.inv_freq, pos, cs, c.tid);
    {
        // Residual rows this CTA owns in the O/down projections start as the embedding.
        int lo, hi;
        split_rows(p.g_wo.out_rows, lo, hi);
        for (int r = lo + c.tid; r < hi; r += kCt) {
            const float v = emb_value<WT>(p, tok, r);
            __stcg(p.x + r, v);
            if (p.debug_res) p.debug_res[r] = v;
        }
    }
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int l = 0; l < kStepLayers; ++l) {
        const StepLayer& L = p.layers[l];
        const size_t layer_off = static_cast<size_t>(l) * kNkv * p.max_seq * kHd;
        KV* kc = static_cast<KV*>(p.k_cache) + layer_off;
        KV* vc = static_cast<KV*>(p.v_cache) + layer_off;
        // ---- QKV projection (fused RMSNorm) -------------------------------------------------
        if (l == 0) {
            stage<WT>(c, [&](int j) { return emb_value<WT>(p, tok, j); }, kH, L.attn_norm);
        } else {
            if (!dep_wait(c, p.sync + kSyncDown + l - 1, G, 10u + l)) return;
            stage<WT>(c, [&](int j) { return __ldcg(p.x + j); }, kH, L.attn_norm);
        }
        if (!run_tiles<WT, kQkv>(c, l * kOpsPerLayer + kQkv, bv, bi, l)) return;
        signal(c, p.sync + kSyncQkv + l);
        // ---- RoPE + KV write + split-K attention ---------------------------------------------
        if (!dep_wait(c, p.sync + kSyncQkv + l, G, 30u + l)) return;
        {
            AttSmem<KV>& sm = *reinterpret_cast<AttSmem<KV>*>(c.xp);
            for (int i = blockIdx.x; i < kNkv * n_tiles; i += G) {
                const int h = i / n_tiles, tile = i % n_tiles;
                attend_tile<KV, true>(p.qkv, kNh, kNkv, cs, kc, vc, p.max_seq, h, tile, ctx, n_slots, p.part_o, p.part_ml, sm,
                                      c.tid, [] { csync(); });
                if (c.tid == 0) {
                    __threadfence();
                    const unsigned old = atom_acq_rel_gpu_add(p.sync + kSyncTicket + l * kNkv + h, 1u);
                    c.fl->role = (old == static_cast<unsigned>(n_tiles - 1)) ? 1 : 0;
                }
                csync();
                const bool combiner = c.fl->role != 0;
                csync();
                if (combiner) {
                    combine_head(p.part_o, p.part_ml, h, n_tiles, n_slots, p.att, c.tid);
                    signal(c, p.sync + kSyncAtt + l);
                }
            }
        }
        // ---- O projection + residual ------------------------------------------------------
        if (!dep_wait(c, p.sync + kSyncAtt + l, kNkv, 50u + l)) return;
        stage<WT>(c, [&](int j) { return __ldcg(p.att + j); }, kH, nullptr);
        if (!run_tiles<WT, kWo>(c, l * kOpsPerLayer + kWo, bv, bi, l)) return;
        signal(c, p.sync + kSyncWo + l);
        // ---- RMSNorm + gate/up + SwiGLU ---------------------------------------------------
        if (!dep_wait(c, p.sync + kSyncWo + l, G, 70u + l)) return;
        stage<WT>(c, [&](int j) { return __ldcg(p.x + j); }, kH, L.ffn_norm);
        if (!run_tiles<WT, kGu>(c, l * kOpsPerLayer + kGu, bv, bi, l)) return;
        signal(c, p.sync + kSyncGu + l);
        // ---- down projection + residual ---------------------------------------------------
        if (!dep_wait(c, p.sync + kSyncGu + l, G, 90u + l)) return;
        stage<WT>(c, [&](int j) { return __ldcg(p.act + j); }, 4 * kH, nullptr);
        if (!run_tiles<WT, kDown>(c, l * kOpsPerLayer + kDown, bv, bi, l)) return;
        signal(c, p.sync + kSyncDown + l);
    }
    // ---- final RMSNorm + tied lm_head + argmax ---------------------------------------------
    if (!dep_wait(c, p.sync + kSyncDown + kStepLayers - 1, G, 110u)) return;
    stage<WT>(c, [&](int j) { return __ldcg(p.x + j); }, kH, p.final_norm);
    if (!run_tiles<WT, kLm>(c, kWeightOps - 1, bv, bi, kStepLayers)) return;
    float* am_v = reinterpret_cast<float*>(c.scratch);  // scratch is free again after run_tiles
    int* am_i = reinterpret_cast<int*>(c.scratch + kCw);
    warp_argmax(bv, bi);
    if (c.lane == 0) {
        am_v[c.cw] = bv;
        am_i[c.cw] = bi;
    }
    csync();
    if (c.tid == 0) {
        float v = am_v[0];
        int i = am_i[0];
        for (int w = 1; w < kCw; ++w) {
            if (better(am_v[w], am_i[w], v, i)) {
                v = am_v[w];
                i = am_i[w];
            }
        }
        __stcg(p.am_v + blockIdx.x, v);
        __stcg(p.am_i + blockIdx.x, i);
        __threadfence();
        const unsigned old = atom_acq_rel_gpu_add(p.sync + kSyncLm, 1u);
        c.fl->role = (old == static_cast<unsigned>(G - 1)) ? 1 : 0;
    }
    csync();
    if (c.fl->role == 0) return;
    // Last CTA: reduce the per-CTA winners, commit the token, advance the position, reset counters.
    float v = -INFINITY;
    int i = INT_MAX;
    for (int k = c.tid; k < G; k += kCt) {
        const float kv = __ldcg(p.am_v + k);
        const int ki = __ldcg(p.am_i + k);
        if (better(kv, ki, v, i)) {
            v = kv;
            i = ki;
        }
    }
    warp_argmax(v, i);
    if (c.lane == 0) {
        am_v[c.cw] = v;
        am_i[c.cw] = i;
    }
    csync();
    for (int k = c.tid; k < kSyncWords; k += kCt) p.sync[k] = 0u;
    if (c.tid == 0) {
        float bv2 = am_v[0];
        int bi2 = am_i[0];
        for (int w = 1; w < kCw; ++w) {
            if (better(am_v[w], am_i[w], bv2, bi2)) {
                bv2 = am_v[w];
                bi2 = am_i[w];
            }
        }
        *p.d_token = bi2 == INT_MAX ? 0 : bi2;
        *p.d_pos = pos + 1;
        __threadfence();
    }
}

template <WeightType WT, typename KV>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* empty = full + kStages;
    volatile Flags* fl = reinterpret_cast<volatile Flags*>(smem + kOffFlags);
    uint8_t* ring = smem + kOffRing;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fl->abort = 0;
        fl->ok = 0;
        fl->role = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) run_producer(p, ring, full, empty, fl);
        return;
    }
    ConsumerCtx c;
    c.p = &p;
    c.ring = ring;
    c.full = full;
    c.empty = empty;
    c.fl = fl;
    c.xp = reinterpret_cast<float*>(smem + kOffXp);
    c.xc = reinterpret_cast<float*>(smem + kOffXc);
    c.red = reinterpret_cast<float*>(smem + kOffRed);
    c.scratch = reinterpret_cast<float*>(smem + kOffScratch);
    c.tid = threadIdx.x - 32;
    c.cw = c.tid >> 5;
    c.lane = c.tid & 31;
    c.t_base = 0;
    run_consumers<WT, KV>(c, reinterpret_cast<float*>(smem + kOffCs));
    if (fl->abort) atomicOr(p.err, kErrAborted);
}

template <WeightType WT, typename KV>
void launch_typed(const StepParams& p, cudaStream_t stream) {
    auto kernel = decode_step_kernel<WT, KV>;
    static bool configured[64] = {};
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !configured[dev]) {
        CLLM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        int blocks = 0;
        CLLM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, kSmemBytes));
        CLLM_CHECK(blocks >= 1, "decode step: the persistent kernel does not fit on an SM");
        configured[dev] = true;
    }
    void* args[] = {const_cast<StepParams*>(&p)};
    CLLM_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(decode_step_grid()), dim3(kThreads), args,
                                          kSmemBytes, stream));
}

}  // namespace

int decode_step_smem_bytes() { return kSmemBytes; }

int decode_step_grid() { return num_sms(); }

void launch_decode_step(const StepParams& p, WeightType wt, KvType kv, cudaStream_t stream) {
    CLLM_CHECK(p.max_seq % kAttnTile == 0, "decode step: max_seq must be a multiple of 64");
    const bool f16 = kv == KvType::F16;
    switch (wt) {
        case WeightType::BF16:
            f16 ? launch_typed<WeightType::BF16, __half>(p, stream) : launch_typed<WeightType::BF16, __nv_bfloat16>(p, stream);
            return;
        case WeightType::INT8:
            f16 ? launch_typed<WeightType::INT8, __half>(p, stream) : launch_typed<WeightType::INT8, __nv_bfloat16>(p, stream);
            return;
        case WeightType::INT4:
            f16 ? launch_typed<WeightType::INT4, __half>(p, stream) : launch_typed<WeightType::INT4, __nv_bfloat16>(p, stream);
            return;
    }
    throw std::runtime_error("decode step: unknown weight type");
}

}  // namespace cudallm
