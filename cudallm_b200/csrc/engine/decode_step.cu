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
#include "kernels/sampling.cuh"

#ifndef CUDALLM_EARLY_RELEASE
#define CUDALLM_EARLY_RELEASE 1
#endif

namespace cudallm {

namespace {

constexpr int kCw = 8;             // consumer warps (warpgroups 1 and 2)
constexpr int kCt = 32 * kCw;      // consumer threads
// Warpgroup 0: the copy-producer warp, the L2-prefetch warp and two idle warps. Warpgroups exchange
// registers at start (setmaxnreg): the block is launched with kLaunchRegs per thread; warpgroup 0 drops
// to kProducerRegs and the consumers rise to kConsumerRegs. The two shares add up to exactly the launch
// allocation (the host checks the kernel's register count before the first launch), so the increase
// never waits for registers that are not there.
constexpr int kThreads = 128 + kCt;
constexpr int kLaunchRegs = 168;  // 65536 / 384 rounded down to a multiple of 8
constexpr int kProducerRegs = 88;
constexpr int kConsumerRegs = 208;
static_assert(kProducerRegs * 128 + kConsumerRegs * kCt == kLaunchRegs * kThreads, "register split must use the launch pool");
// Weight ring: kStages stages of 16 KiB in the short-context kernel; the split-attention kernel keeps
// kStages - kAttSlots of them and gives the rest to its K/V tile ring (one 64-token K tile + V tile,
// 16 KiB, per slot). Barrier and tile-word arrays are laid out for kStages.
constexpr int kStages = 12;
constexpr int kAttSlots = 4;
// The split attention's tiles are not prefetched into L2: at 16K-32K tokens every prefetch distance
// tried (the whole range at the layer's start, or 4-32 tiles ahead of the copies) measured slower.
static_assert(kStages <= 32, "one producer lane per stage");
template <bool SPLIT>
constexpr int ring_stages() {
    return SPLIT ? kStages - kAttSlots : kStages;
}
// bf16 tiles (one warp's work each): the warp copies its chunks of the stage into registers in two halves and
// releases the stage after loading the second, so the next copy into it is in flight during the second half's
// arithmetic (0: released after all of it). Measured at 256 steps: bf16 1618 -> 1640 tok/s; int8 tiles kept
// the late release (the same split took int8 from 1857 to 1743 tok/s).
constexpr bool kEarlyRelease = CUDALLM_EARLY_RELEASE;
constexpr int kMaxK = 8192;
constexpr int kOpsPerLayer = 4;
constexpr int kWeightOps = kStepLayers * kOpsPerLayer + 1;  // + tied lm_head
constexpr int kH = 2048, kNh = 32, kNkv = 8;

enum OpKind : int { kQkv = 0, kWo = 1, kGu = 2, kDown = 3, kLm = 4 };

struct Flags {
    int abort;
    int ok;
    int role;
    int issued;  // tiles the copy producer has issued (read by the prefetch warp)
};

// Shared-memory layout (byte offsets).
constexpr int kOffBars = 0;
constexpr int kOffTiles = 2 * kStages * 8;  // int per stage: tile the producer last issued into it
constexpr int kOffFlags = 256;
constexpr int kOffKinds = 288;  // KindRows[5]: this CTA's rows of each operation kind
constexpr int kOffAttFull = 352;  // split kernel: kAttSlots mbarriers of the K/V tile ring (room for 8)
constexpr int kOffRed = 416;      // kCw floats: one partial sum of squares per consumer warp
constexpr int kOffAttCnt = 448;   // split kernel: kAttSlots arrival counters, then kAttSlots pending words
constexpr int kOffCs = 512;
static_assert(kOffAttFull + kAttSlots * 8 <= kOffRed && kOffRed + 4 * kCw <= kOffAttCnt &&
                  kOffAttCnt + 2 * kAttSlots * 4 <= kOffCs,
              "attention ring words overflow");
constexpr int kOffScratch = 768;
constexpr int kOffAm = kOffScratch + kCw * 32 * 4;  // 1792
// The residual rows this CTA owns (the same row range in the O and down projections), kept on chip for
// the whole step so their epilogues add without reading x back.
constexpr int kOffRes = kOffAm + kCw * 8;  // 1856
constexpr int kMaxResRows = 48;
constexpr int kOffXc = 2048;
constexpr int kOffXp = 3072;
constexpr int kOffRing = kOffXp + kMaxK * 4;  // 35840
// Sampling scratch in the (idle) ring after the lm_head: the candidate keys of one CTA's rows, or of every
// CTA's top k in the last CTA, then the selection's scratch and result.
constexpr int kSampleKeyBytes = kSampleMaxGrid * kMaxTopK * 8;
static_assert(kSampleKeyBytes + static_cast<int>(sizeof(TopKScratch)) + kMaxTopK * 8 <= kStages * kStageBytes,
              "sampling scratch must fit in the ring");
constexpr int kSmemBytes = kOffRing + kStages * kStageBytes;
static_assert(kOffTiles + kStages * 4 <= kOffFlags, "barriers overflow");
static_assert(kOffAm + kCw * 8 <= kOffRes && kOffRes + kMaxResRows * 4 <= kOffXc, "argmax / residual scratch overflow");
static_assert(kOffXc + (kMaxK / 32) * 4 <= kOffXp, "chunk sums overflow");
static_assert(sizeof(AttSmem<__half>) <= kMaxK * 4, "attention scratch must fit in the vector area");
static_assert(sizeof(HeadPassSmem<__half>) <= kMaxK * 4, "attention scratch must fit in the vector area");
static_assert(kOffRing % 128 == 0, "ring alignment");

// Stage rows of each operation's tile (rows per tile x halves); the host builds the persistent path's
// geometry with the same rule (make_tile_geom with the default tile rows), checked at run time.
template <WeightType WT>
constexpr int weight_row_bytes(int k) {
    return WT == WeightType::BF16 ? 2 * k : (WT == WeightType::INT8 ? k : k / 2);
}
// Bytes of one tile's row segment: the whole row, except the down projection (K = 8192), whose rows are
// cut into kDownSegBytes segments (n_seg > 1 for bf16 and int8).
template <WeightType WT, int KIND>
constexpr int seg_bytes_of() {
    constexpr int rb = weight_row_bytes<WT>(KIND == 3 ? 4 * 2048 : 2048);
    return KIND == 3 && rb > kDownSegBytes ? kDownSegBytes : rb;
}
// Chunks per lane of one row segment.
template <WeightType WT, int KIND>
constexpr int seg_chunks_per_lane() {
    return seg_bytes_of<WT, KIND>() / 512;
}

template <WeightType WT, int KIND>
constexpr int stage_rows() {
    constexpr int halves = KIND == 2 ? 2 : 1;  // gate/up
    constexpr int rb = seg_bytes_of<WT, KIND>();
    constexpr int fit = kStageBytes / halves / rb;
    constexpr int cap = decode_step_tile_rows(WT);
    return (fit < cap ? fit : cap) * halves;
}

// How the consumer warps share the stages of one operation kind: kRows stage rows (both halves for the
// gate/up operation), kWps warps per stage (1: one warp consumes a whole stage; >1: the stage's rows are
// split over kWps warps and kCw / kWps warp groups take stages in turn), kNw rows per warp, kHalf of them
// per half, kCpl 16-byte chunks per lane of a row.
// Warps per stage by weight type and operation kind (qkv, o-proj, gate/up, down, lm_head).
constexpr int kBf16WarpsPerStage[5] = {1, 1, 1, 1, 1};
constexpr int kInt8WarpsPerStage[5] = {1, 1, 1, 1, 1};
constexpr int kInt4WarpsPerStage[5] = {4, 4, 4, 4, 4};
template <WeightType WT>
constexpr int warps_per_stage(int kind) {
    return WT == WeightType::INT4 ? kInt4WarpsPerStage[kind]
           : WT == WeightType::INT8 ? kInt8WarpsPerStage[kind] : kBf16WarpsPerStage[kind];
}
// Whether any operation of this weight type shares its stages (then every operation runs the shared loop).
template <WeightType WT>
constexpr bool shares_stages() {
    return warps_per_stage<WT>(0) > 1 || warps_per_stage<WT>(1) > 1 || warps_per_stage<WT>(2) > 1 ||
           warps_per_stage<WT>(3) > 1 || warps_per_stage<WT>(4) > 1;
}
template <WeightType WT, int KIND>
struct StageShape {
    static constexpr int kHalves = KIND == 2 ? 2 : 1;
    static constexpr int kRows = stage_rows<WT, KIND>();
    static constexpr int kWps = warps_per_stage<WT>(KIND);
    static constexpr int kNw = kRows / kWps;
    static constexpr int kHalf = kNw / kHalves;
    static constexpr int kCpl = seg_chunks_per_lane<WT, KIND>();
    static_assert(kRows % kWps == 0 && kNw % kHalves == 0 && kNw <= 32, "stage rows must split evenly over the warps");
};

struct WOp {
    const uint8_t* w;
    const void* s;
    TileGeom g;
};

// L1 prefetch of the scales of rows [r, r + n) of a quantised operation (int8: one fp32 per row; int4: one
// fp16 per 128 columns), lines i, i + step, ...: every line lies within the rows' bytes (the first one
// starts at or before them, inside the same weight arena). Nothing for bf16.
template <WeightType WT>
__device__ __forceinline__ void prefetch_scale_rows(const void* scales, int cols, int r, int n, int i, int step) {
    if constexpr (WT != WeightType::BF16) {
        const size_t row_bytes = WT == WeightType::INT8 ? 4 : static_cast<size_t>(cols / 128) * 2;
        const uintptr_t a = reinterpret_cast<uintptr_t>(scales) + static_cast<size_t>(r) * row_bytes;
        const uintptr_t b = a + static_cast<size_t>(n) * row_bytes;
        for (uintptr_t line = (a & ~static_cast<uintptr_t>(127)) + static_cast<uintptr_t>(i) * 128; line < b;
             line += static_cast<uintptr_t>(step) * 128) {
            prefetch_l1(reinterpret_cast<const void*>(line));
        }
    }
}
// Rows of scales an operation prefetches before its input wait; past them the tile loop prefetches the
// rows of the tile this many rows ahead (only the lm_head has more).
constexpr int kScaleAheadRows = 256;

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

// Rows [lo, hi) of an n-row operation owned by this CTA. 32-bit arithmetic: n * grid stays far below 2^32
// (vocab 128256 x 148 SMs).
__device__ __forceinline__ void split_rows(int n, int& lo, int& hi) {
    const unsigned un = static_cast<unsigned>(n), g = gridDim.x;
    lo = static_cast<int>(blockIdx.x * un / g);
    hi = static_cast<int>((blockIdx.x + 1) * un / g);
}

__device__ __forceinline__ int op_tiles(const TileGeom& g, int lo, int hi) {
    const int R = g.rows_per_tile;
    return ((hi - lo + R - 1) / R) * g.n_seg;
}

__device__ __forceinline__ void trace_mark(const StepParams& p, int op, int slot) {
    if (p.trace) p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + op * kTraceStamps + slot] = global_ns();
}

// Stamps slot `slot` of global tile t of CTA 0 when it lies in the traced window.
__device__ __forceinline__ void trace_tile(const StepParams& p, int t, int slot) {
    const int i = t - p.trace_t0;
    if (p.trace && blockIdx.x == 0 && i >= 0 && i < kTraceTiles) {
        p.trace[static_cast<size_t>(gridDim.x) * kTraceSlots + i * kTraceTileStamps + slot] = global_ns();
    }
}

__device__ __forceinline__ int trace_op_of_weight_op(int o) {
    if (o == kWeightOps - 1) return 80;
    const int l = o / kOpsPerLayer, k = o % kOpsPerLayer;
    return l * 5 + (k == kQkv ? 0 : k + 1);
}

__device__ __forceinline__ void fail(const StepParams& p, volatile Flags* fl, unsigned code, unsigned id) {
    fl->abort = 1;
    atomicOr(p.err, code);
    atomicCAS(p.err + 1, 0u, id);
}

// Bounded per-thread wait on an mbarrier phase (the producer lanes' drain of their last copies).
__device__ bool wait_bar(const StepParams& p, uint64_t* bar, uint32_t parity, volatile Flags* fl, uint64_t limit_ns,
                         unsigned id) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            const uint64_t t = global_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > limit_ns) {
                fail(p, fl, kErrWaitTimeout, id);
                return false;
            }
        }
    }
}

// Warp-collective bounded wait for tile `tile` in a ring stage (all 32 lanes of a consumer warp call it):
// first until the producer has published that tile into the stage (a parity wait alone only tells the
// barrier's current phase from the previous one, and a consumer warp can be further ahead), then for the
// stage's phase. Every decision is a warp vote, so the lanes leave together with the same answer; gives
// up when the CTA aborts or after the wait limit.
__device__ bool wait_tile(const StepParams& p, uint64_t* bar, uint32_t parity, volatile Flags* fl, unsigned id,
                          const volatile int* tile_word, int tile) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        const bool ready = *tile_word == tile && mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ready)) return true;
        if ((it & 63) == 0) {
            if (__any_sync(0xffffffffu, fl->abort != 0)) return false;
            const uint64_t t = __shfl_sync(0xffffffffu, global_ns(), 0);
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > p.wait_limit_ns) {
                if ((threadIdx.x & 31) == 0) fail(p, fl, kErrWaitTimeout, id);
                return false;
            }
        }
    }
}

// Cursor over this CTA's tiles of the whole step (operation by operation).
__device__ __forceinline__ uint8_t* smem_base() {
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    return smem_dyn;
}

// This CTA's rows and tile count of one operation kind (the same in every layer).
struct KindRows {
    int lo, hi, nt;
};
static_assert(kOffKinds + 5 * sizeof(KindRows) <= kOffAttFull, "kind table overflow");
__device__ __forceinline__ KindRows kind_rows(const TileGeom& g) {
    KindRows r;
    split_rows(g.out_rows, r.lo, r.hi);
    r.nt = op_tiles(g, r.lo, r.hi);
    return r;
}

// Fills the shared table of this CTA's rows per operation kind (qkv, o-proj, gate/up, down, lm_head);
// one thread, before the block's first barrier.
__device__ __forceinline__ void init_kind_rows(const StepParams& p, KindRows* kinds) {
    kinds[kQkv] = kind_rows(p.g_qkv);
    kinds[kWo] = kind_rows(p.g_wo);
    kinds[kGu] = kind_rows(p.g_gu);
    kinds[kDown] = kind_rows(p.g_down);
    kinds[kLm] = kind_rows(p.g_lm);
}

// Cursor over this CTA's tiles of the whole step (operation by operation). Row ranges come from the
// shared per-kind table, so crossing an operation costs no division.
__device__ __forceinline__ const KindRows* kind_table() { return reinterpret_cast<const KindRows*>(smem_base() + kOffKinds); }

struct TileCursor {
    int o = 0, i = 0, nt = 0, lo = 0, hi = 0;
    __device__ void init() {
        o = 0;
        i = 0;
        load();
    }
    __device__ void load() {
        const KindRows r = kind_table()[o == kWeightOps - 1 ? kLm : o % kOpsPerLayer];
        lo = r.lo;
        hi = r.hi;
        nt = r.nt;
    }
    __device__ bool valid() const { return o < kWeightOps; }
    // Moves n tiles forward.
    __device__ void advance(int n) {
        i += n;
        while (o < kWeightOps && i >= nt) {
            i -= nt;
            if (++o < kWeightOps) load();
        }
    }
};

__device__ __forceinline__ void issue_tile(const WOp& op, int lo, int hi, int i, uint8_t* dst, uint64_t* bar, uint64_t pol) {
    const TileGeom& g = op.g;
    const int grp = g.n_seg == 1 ? i : i / g.n_seg, sg = g.n_seg == 1 ? 0 : i % g.n_seg;
    const int r0 = lo + grp * g.rows_per_tile;
    const int nr = min(g.rows_per_tile, hi - r0);
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nr * g.seg_bytes * g.halves));
    for (int h = 0; h < g.halves; ++h) {
        const size_t row = static_cast<size_t>(r0) + static_cast<size_t>(h) * g.out_rows;
        if (g.n_seg == 1) {
            bulk_load(dst + h * g.rows_per_tile * g.seg_bytes, op.w + row * g.row_bytes, static_cast<uint32_t>(nr * g.row_bytes),
                      bar, pol);
        } else {
            for (int r = 0; r < nr; ++r) {
                bulk_load(dst + (h * g.rows_per_tile + r) * g.seg_bytes,
                          op.w + (row + r) * g.row_bytes + static_cast<size_t>(sg) * g.seg_bytes,
                          static_cast<uint32_t>(g.seg_bytes), bar, pol);
            }
        }
    }
}

// Warp 0: lane s < kStages owns stage s and streams the tiles t = s, s + kStages, ... of the step (in use
// order) into it, issuing each copy as soon as the stage is released. The lanes poll their stages with
// non-blocking tests in one converged loop, so a stage that is still in use never holds back another
// lane's copy. Lane 0 publishes the lowest tile index not yet issued for the prefetch warp.
template <int ST>
__device__ void run_producer(const StepParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty, volatile int* stage_tile,
                             volatile Flags* fl) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = l2_policy_evict_first();
    TileCursor cur;
    cur.init();
    cur.advance(lane);
    int t = lane, k = 0;  // next tile of this lane; copies issued into its stage so far
    bool more = lane < ST && cur.valid();
    uint64_t t_idle = 0;
    for (uint32_t it = 1;; ++it) {
        bool progressed = false;
        if (more && (k == 0 || mbar_test_wait(&empty[lane], (k - 1) & 1))) {
            if (cur.i == 0) trace_mark(p, trace_op_of_weight_op(cur.o), 3);
            stage_tile[lane] = t;
            trace_tile(p, t, 0);
            issue_tile(weight_op(p, cur.o), cur.lo, cur.hi, cur.i, ring + lane * kStageBytes, &full[lane], pol);
            ++k;
            t += ST;
            cur.advance(ST);
            more = cur.valid();
            progressed = true;
        }
        const int front = __reduce_min_sync(0xffffffffu, more ? t : (1 << 30));
        if (lane == 0) fl->issued = front;  // 1 << 30 once every tile is issued: releases the prefetch warp
        if (!__any_sync(0xffffffffu, more)) break;
        if (__any_sync(0xffffffffu, progressed)) {
            t_idle = 0;
        } else if ((it & 63) == 0) {
            // Warp-uniform decisions: every lane leaves the loop at the same iteration.
            if (__any_sync(0xffffffffu, fl->abort != 0)) break;
            const uint64_t now = __shfl_sync(0xffffffffu, global_ns(), 0);
            if (t_idle == 0) {
                t_idle = now;
            } else if (now - t_idle > p.wait_limit_ns) {
                if (lane == 0) fail(p, fl, kErrWaitTimeout, 1000u);
                break;
            }
        }
    }
    // Every copy issued lands before the CTA may exit. The drain has its own limit, independent of the
    // (possibly short) dependency-wait limit: the copies are plain reads and always finish.
    if (lane < ST && k > 0) wait_bar(p, &full[lane], (k - 1) & 1, fl, p.drain_limit_ns, 2000u);
}

// Warp 1: L2 prefetch of the weight stream with ordinary prefetch instructions (load/store units,
// not the TMA engine the copies use), p.prefetch_tiles tiles ahead of the copy producer.
__device__ void run_prefetcher(const StepParams& p, volatile Flags* fl) {
    const int lane = threadIdx.x & 31;
    TileCursor pf;
    pf.init();
    int pt = 0;
    uint64_t t0 = 0;
    while (pf.valid()) {
        for (uint32_t it = 1; pt >= fl->issued + p.prefetch_tiles; ++it) {
            if (fl->abort) return;
            if ((it & 63) == 0) {
                const uint64_t t = global_ns();
                if (t0 == 0) t0 = t;
                if (t - t0 > p.wait_limit_ns) return;  // the copy producer stopped; nothing to wait for
            }
            __nanosleep(128);
        }
        t0 = 0;
        // Tile i of the operation: row group i / n_seg, segment i % n_seg. Whole-row tiles (n_seg == 1) are
        // one contiguous range per half; segmented tiles one range per row.
        const WOp op = weight_op(p, pf.o);
        const TileGeom& g = op.g;
        const int grp = pf.i / g.n_seg, sg = pf.i % g.n_seg;
        const int r0 = pf.lo + grp * g.rows_per_tile;
        const int nr = min(g.rows_per_tile, pf.hi - r0);
        for (int h = 0; h < g.halves; ++h) {
            const size_t row = static_cast<size_t>(r0) + static_cast<size_t>(h) * g.out_rows;
            const uint8_t* a = op.w + row * g.row_bytes + static_cast<size_t>(sg) * g.seg_bytes;
            const int pieces = g.n_seg == 1 ? 1 : nr;
            const int bytes = g.n_seg == 1 ? nr * g.row_bytes : g.seg_bytes;
            if (p.prefetch_mode == 3) {
                // one bulk request per contiguous range (bulk engine)
                if (lane < pieces) bulk_prefetch_l2(a + static_cast<size_t>(lane) * g.row_bytes, static_cast<uint32_t>(bytes));
            } else {
                for (int q = 0; q < pieces; ++q) {
                    for (int off = lane * 128; off < bytes; off += 32 * 128) {
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(a + static_cast<size_t>(q) * g.row_bytes + off) : "memory");
                    }
                }
            }
        }
        if (lane == 0) trace_tile(p, pt, 4);
        pf.advance(1);
        ++pt;
    }
}

// Columns 4q..4q+3 of embedding row `tok`, dequantised (one 8/4/2-byte load).
template <WeightType WT>
struct EmbVec4 {
    const StepParams* p;
    int tok;
    __device__ __forceinline__ float4 operator()(int q) const {
        if constexpr (WT == WeightType::BF16) {
            const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p->emb_w) +
                                                                 static_cast<size_t>(tok) * kH) + q);
            return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                               __uint_as_float(w.y & 0xffff0000u));
        } else if constexpr (WT == WeightType::INT8) {
            const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(static_cast<const int8_t*>(p->emb_w) +
                                                                      static_cast<size_t>(tok) * kH) + q);
            const float s = __ldg(static_cast<const float*>(p->emb_s) + tok);
            return make_float4(static_cast<float>(static_cast<int8_t>(w & 0xff)) * s,
                               static_cast<float>(static_cast<int8_t>((w >> 8) & 0xff)) * s,
                               static_cast<float>(static_cast<int8_t>((w >> 16) & 0xff)) * s,
                               static_cast<float>(static_cast<int8_t>(w >> 24)) * s);
        } else {
            const uint16_t w = __ldg(reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(p->emb_w) +
                                                                      static_cast<size_t>(tok) * (kH / 2)) + q);
            const float s = __half2float(__ldg(static_cast<const __half*>(p->emb_s) +
                                               static_cast<size_t>(tok) * (kH / p->group_size) + (4 * q) / p->group_size));
            return make_float4(static_cast<float>(static_cast<int>(w & 0xF) - 8) * s,
                               static_cast<float>(static_cast<int>((w >> 4) & 0xF) - 8) * s,
                               static_cast<float>(static_cast<int>((w >> 8) & 0xF) - 8) * s,
                               static_cast<float>(static_cast<int>((w >> 12) & 0xF) - 8) * s);
        }
    }
};

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
    volatile int* stage_tile;
    volatile Flags* fl;
    float* xp;
    float* xc;
    float* red;
    float* scratch;
    float* res;  // [kMaxResRows] this CTA's residual rows
    int tid, cw, lane;
    int t_base;      // global tile index of the current operation's first tile
    float in_scale;  // factor of the current operation's outputs: 1/rms of its input when RMS-normalised, else 1
};

__device__ __forceinline__ void csync() { named_barrier(1, kCt); }

// ---- Tagged activations ----------------------------------------------------------------------------
// Every activation that crosses CTAs is written as one 64-bit word (tag << 32 | fp32 bits) by a single
// 8-byte store, which is single-copy atomic: a reader that sees the current tag sees the value written
// with it. The tag names the launch (step_tag), the layer and the vector, so a reader needs no counter,
// no release and no second round trip: it polls the data until the tags are current. A slot is
// rewritten only after every CTA has passed a later all-to-all dependency, hence after all its readers.
enum TagKind : uint32_t { kTagQkv = 1, kTagAtt = 2, kTagXmid = 3, kTagXout = 4, kTagAct = 5, kTagPart = 6 };
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t act_tag(const StepParams& p, int layer, uint32_t kind) {
    return (p.step_tag << 8) | (static_cast<uint32_t>(layer) << 3) | kind;
}
__device__ __forceinline__ void st_tagged(unsigned long long* dst, float v, uint32_t tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* src) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
    return w;
}
__device__ __forceinline__ void ld_tagged2(const unsigned long long* src, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
}
__device__ __forceinline__ bool tag_is(unsigned long long w, uint32_t tag) { return static_cast<uint32_t>(w >> 32) == tag; }
__device__ __forceinline__ float tag_value(unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); }

// Bounded poll bookkeeping: false once the wait limit passed (recorded as a timeout) or another CTA
// reported an error.
struct PollClock {
    uint64_t t0 = 0;
    uint32_t n = 0;
    __device__ __forceinline__ bool keep_going(const StepParams& p, volatile Flags* fl, unsigned id) {
        if (fl->abort) return false;
        // Another CTA's failure (the global error word, one memory round trip during which the poll does not
        // advance) is looked at on every 8th call only; the wall-clock limit on every call.
        if ((++n & 7) == 0 && *reinterpret_cast<volatile unsigned*>(p.err) != 0) {
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
        return true;
    }
};

// One element of a tagged vector, polled until it carries `tag` (or the wait gives up).
__device__ __forceinline__ float get_tagged(const StepParams& p, volatile Flags* fl, const unsigned long long* src, uint32_t tag,
                                            unsigned id) {
    unsigned long long w = ld_tagged(src);
    PollClock clk;
    // No back-off between polls: each poll already waits one L2 round trip, and a sleep only delays seeing
    // the value (measured: 32-64 ns sleeps here and in load_input cost bf16 2.3 % of its tok/s).
    for (uint32_t it = 1; !tag_is(w, tag); ++it) {
        w = ld_tagged(src);
        if ((it & 15) == 0 && !clk.keep_going(p, fl, id)) break;
    }
    return tag_value(w);
}

// Two elements of a tagged vector: both loads are in flight together and each is re-polled until current,
// so the pair costs one memory round trip, not two.
__device__ __forceinline__ float2 get_tagged_pair(const StepParams& p, volatile Flags* fl, const unsigned long long* a,
                                                  const unsigned long long* b, uint32_t tag, unsigned id) {
    unsigned long long wa = ld_tagged(a), wb = ld_tagged(b);
    PollClock clk;
    for (uint32_t it = 1; !(tag_is(wa, tag) && tag_is(wb, tag)); ++it) {
        if (!tag_is(wa, tag)) wa = ld_tagged(a);
        if (!tag_is(wb, tag)) wb = ld_tagged(b);
        if ((it & 15) == 0 && !clk.keep_going(p, fl, id)) break;
    }
    return make_float2(tag_value(wa), tag_value(wb));
}

struct TaggedSrc {
    const StepParams* p;
    volatile Flags* fl;
    const unsigned long long* v;
    uint32_t tag;
    unsigned id;
    __device__ __forceinline__ float operator()(int i) const { return get_tagged(*p, fl, v + i, tag, id); }
    __device__ __forceinline__ float2 pair(int i, int j) const { return get_tagged_pair(*p, fl, v + i, v + j, tag, id); }
};
struct TaggedDst {
    unsigned long long* v;
    uint32_t tag;
    __device__ __forceinline__ void operator()(int i, float x) const { st_tagged(v + i, x, tag); }
};

// Ranges per KV head for the attention of a context of n_tiles 64-token tiles (n_pass 128-token passes):
// 1 = one CTA per head over the whole context; else S ranges plus one merging CTA per head.
__device__ __forceinline__ int attn_splits(const StepParams& p, int n_tiles, int n_pass) {
    if (n_tiles <= p.whole_head_max_tiles) return 1;
    const int s = min(min(kAttnMaxSplits, (static_cast<int>(gridDim.x) - kNkv) / kNkv), n_pass);
    return s > 1 ? s : 1;
}

// This CTA's attention work for a context of ctx tokens (the same in every layer; recomputed where it is
// used so that none of it stays live across the weight operations): KV head `head` (-1: none) over the
// 128-token passes [p0, p1), or, when the context is split (S > 1), merging head `merge`'s S ranges.
struct AttnRole {
    int S, n_pass, head, split, p0, p1, merge;
};
__device__ __forceinline__ AttnRole attn_role(const StepParams& p, int ctx) {
    AttnRole r;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    r.n_pass = (ctx + kHeadPassTokens - 1) / kHeadPassTokens;
    r.S = attn_splits(p, n_tiles, r.n_pass);
    r.head = -1;
    r.split = 0;
    r.p0 = 0;
    r.p1 = 0;
    r.merge = -1;
    const int b = blockIdx.x;
    if (r.S == 1) {
        const int stride = gridDim.x / kNkv;
        if (b % stride == 0 && b / stride < kNkv) {
            r.head = b / stride;
            r.p1 = r.n_pass;
        }
    } else if (b < kNkv * r.S) {
        r.head = b / r.S;
        r.split = b % r.S;
        r.p0 = r.split * r.n_pass / r.S;
        r.p1 = (r.split + 1) * r.n_pass / r.S;
    } else if (b < kNkv * r.S + kNkv) {
        r.merge = b - kNkv * r.S;
    }
    return r;
}

// ---- Range attention of the split kernel --------------------------------------------------------------
// One CTA computes the 4 query heads of KV head h over the 64-token tiles [T0, T1) of the context. Each
// tile's K and V rows (8 KiB each, contiguous in the cache) arrive by bulk copies in one of kAttSlots
// shared-memory slots, completing on the slot's mbarrier; the copies of the first tiles are issued before
// the step's q is waited for. Warp w takes tokens 8w .. 8w + 7 of every tile: it copies its rows into
// registers, releases the slot (the last of the 8 warps to do so issues the copy of the tile kAttSlots
// ahead into it) and then computes, so no block barrier separates the tiles. Lane l works on token l / 4
// of the group: its 16-dimension quarter (l % 4) of the key for the 4 heads' scores, completed over the
// token's 4 lanes by two exchange steps that leave lane l with head hl = 2 (l & 1) + ((l >> 1) & 1); and
// output dimensions 2l, 2l + 1 of the 4 heads for p.V, the group's probabilities passing through a
// per-warp shared-memory slot. Each warp keeps its own running softmax; the warps' states are merged in
// warp order at the end and handed to emit(hq, d, O, M, L). The range that holds pos rotates the new key,
// rounds k and v to the cache type, writes them to the cache and uses the rounded values for token pos.
// Every wait is bounded; after a wait gives up, every issued copy lands before the CTA goes on.
template <typename KV>
struct RangeAttnSmem {
    float qs[kGqa][kHd];
    alignas(16) KV kn[kHd];
    alignas(16) KV vn[kHd];
    alignas(16) float pw[kCw][8][kGqa];  // per warp: the current group's probabilities [token][head]
    alignas(16) float aw[kCw][kGqa];     // per warp: the group's rescale factors per head
    float wo[kCw][kGqa][kHd];
    float wm[kCw][kGqa], wl[kCw][kGqa];
};
static_assert(sizeof(RangeAttnSmem<__half>) <= kMaxK * 4, "range attention scratch must fit in the vector area");

// One 8-token group's cached rows as this lane holds them: its key quarter, and dims 2l, 2l + 1 of the 8
// values.
struct GroupRows {
    uint4 k0, k1;
    uint32_t v[8];
};

// This lane's part of the group of 8 tokens starting at row jt of a staged 64-token tile: its key quarter of
// token jt + lane / 4, and dims 2l, 2l + 1 of the 8 values (zero for tokens at or past `nt`, the tile's
// valid rows, whose staged bytes are stale).
template <typename KV>
__device__ __forceinline__ void stage_group(const KV* kt, const KV* vt, int jt, int nt, int lane, GroupRows& r) {
    const int j = jt + (lane >> 2);
    if (j < nt) {
        const uint4* kp = reinterpret_cast<const uint4*>(kt + j * kHd + 16 * (lane & 3));
        r.k0 = kp[0];
        r.k1 = kp[1];
    } else {
        r.k0 = r.k1 = make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) r.v[t] = jt + t < nt ? reinterpret_cast<const uint32_t*>(vt + (jt + t) * kHd)[lane] : 0u;
}

// Scores, online softmax and p.V of one group (tokens j0 .. j0 + 7, valid below `end`) for this warp.
template <typename KV>
__device__ __forceinline__ void attend_group(const GroupRows& r, int j0, int end, int lane, int warp, const float2 (&q)[kGqa][8],
                                             float& m_run, float& l_run, float2 (&acc)[kGqa], RangeAttnSmem<KV>& sm) {
    using KV2 = typename Kv2<KV>::T;
    const KV2* k2a = reinterpret_cast<const KV2*>(&r.k0);
    const KV2* k2b = reinterpret_cast<const KV2*>(&r.k1);
    float sc[kGqa];
#pragma unroll
    for (int g = 0; g < kGqa; ++g) {
        float2 a = make_float2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 4; ++e) a = fma2(kv2_to_float2(k2a[e]), q[g][e], a);
#pragma unroll
        for (int e = 0; e < 4; ++e) a = fma2(kv2_to_float2(k2b[e]), q[g][4 + e], a);
        sc[g] = a.x + a.y;
    }
    // Two exchanges over the token's 4 lanes: lane bit 0 picks heads {0,1} or {2,3}, bit 1 one of the pair.
    const bool b0 = (lane & 1) != 0, b1 = (lane & 2) != 0;
    const float x0 = __shfl_xor_sync(0xffffffffu, b0 ? sc[0] : sc[2], 1);
    const float x1 = __shfl_xor_sync(0xffffffffu, b0 ? sc[1] : sc[3], 1);
    const float t0 = (b0 ? sc[2] : sc[0]) + x0, t1 = (b0 ? sc[3] : sc[1]) + x1;
    const float y = __shfl_xor_sync(0xffffffffu, b1 ? t0 : t1, 2);
    const int hl = 2 * (lane & 1) + ((lane >> 1) & 1);
    const int j = j0 + (lane >> 2);
    const float s = j < end ? 0.125f * ((b1 ? t1 : t0) + y) : -INFINITY;
    // Online softmax of head hl over the group's 8 tokens (the lanes with this lane's bits 0-1).
    float mg = s;
    mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, 4));
    mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, 8));
    mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, 16));
    const float m_new = fmaxf(m_run, mg);  // finite: token j0 is valid
    const float p = expf(s - m_new);
    float ps = p;
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    const float alpha = expf(m_run - m_new);
    l_run = l_run * alpha + ps;
    m_run = m_new;
    sm.pw[warp][lane >> 2][hl] = p;
    if (lane < 4) sm.aw[warp][hl] = alpha;
    __syncwarp();
    const float4 al = *reinterpret_cast<const float4*>(sm.aw[warp]);
    acc[0] = make_float2(acc[0].x * al.x, acc[0].y * al.x);
    acc[1] = make_float2(acc[1].x * al.y, acc[1].y * al.y);
    acc[2] = make_float2(acc[2].x * al.z, acc[2].y * al.z);
    acc[3] = make_float2(acc[3].x * al.w, acc[3].y * al.w);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const float4 p4 = *reinterpret_cast<const float4*>(sm.pw[warp][t]);
        const float2 vf = kv2_to_float2(*reinterpret_cast<const KV2*>(&r.v[t]));
        acc[0] = fma2(make_float2(p4.x, p4.x), vf, acc[0]);
        acc[1] = fma2(make_float2(p4.y, p4.y), vf, acc[1]);
        acc[2] = fma2(make_float2(p4.z, p4.z), vf, acc[2]);
        acc[3] = fma2(make_float2(p4.w, p4.w), vf, acc[3]);
    }
    __syncwarp();  // pw / aw are rewritten by the next group
}

// Rotates the 4 query heads of KV head h into sm.qs and, for the range that holds pos, rotates the new
// key, rounds k and v to the cache type, writes them to the cache and keeps the rounded values in sm.kn /
// sm.vn. Threads 0..127 the queries, 128..159 the key, 160..223 the value; the caller's barrier follows.
template <typename KV, typename Src>
__device__ __forceinline__ void load_query_insert_kv(const ConsumerCtx& c, int h, int pos, bool insert_new, const float* cs,
                                                     KV* k_cache, KV* v_cache, Src qkv, RangeAttnSmem<KV>& sm) {
    const StepParams& p = *c.p;
    const int tid = c.tid;
    if (tid < kGqa * kHd / 2) {
        const int g = tid >> 5, i = tid & 31;
        const int q = (h * kGqa + g) * kHd;
        const float2 x = qkv.pair(q + i, q + i + kHd / 2);
        const float x0 = x.x, x1 = x.y;
        const float cz = cs[i], sz = cs[kHd / 2 + i];
        sm.qs[g][i] = x0 * cz - x1 * sz;
        sm.qs[g][i + kHd / 2] = x1 * cz + x0 * sz;
    } else if (insert_new && tid < kGqa * kHd / 2 + kHd / 2) {
        const int i = tid - kGqa * kHd / 2;
        const int kp = (kNh + h) * kHd;
        const float2 x = qkv.pair(kp + i, kp + i + kHd / 2);
        const float x0 = x.x, x1 = x.y;
        const float cz = cs[i], sz = cs[kHd / 2 + i];
        const KV k0 = to_kv<KV>(x0 * cz - x1 * sz), k1 = to_kv<KV>(x1 * cz + x0 * sz);
        sm.kn[i] = k0;
        sm.kn[i + kHd / 2] = k1;
        KV* kdst = k_cache + (static_cast<size_t>(h) * p.max_seq + pos) * kHd;
        kdst[i] = k0;
        kdst[i + kHd / 2] = k1;
    } else if (insert_new && tid < kGqa * kHd / 2 + kHd / 2 + kHd) {
        const int d = tid - kGqa * kHd / 2 - kHd / 2;
        const KV vv = to_kv<KV>(qkv((kNh + kNkv + h) * kHd + d));
        sm.vn[d] = vv;
        v_cache[(static_cast<size_t>(h) * p.max_seq + pos) * kHd + d] = vv;
    }
}

// Token `row` of a group is the new token: its key quarter and value pair come from the rounded values in
// shared memory (the staged copy of its cache row may predate this step's store).
template <typename KV>
__device__ __forceinline__ void patch_new_token(GroupRows& r, int row, int lane, const RangeAttnSmem<KV>& sm) {
    if ((lane >> 2) == row) {
        const uint4* ks = reinterpret_cast<const uint4*>(sm.kn + 16 * (lane & 3));
        r.k0 = ks[0];
        r.k1 = ks[1];
    }
    r.v[row] = reinterpret_cast<const uint32_t*>(sm.vn)[lane];
}

// Merges the 8 warps' softmax states in warp order (a warp that saw no token has M = -inf, L = 0, O = 0)
// and hands emit(hq, d, O, M, L) to thread 64 (hq - 4h) + d. Ends with a barrier.
template <typename KV, typename Emit>
__device__ __forceinline__ void merge_warp_states(const ConsumerCtx& c, int h, float m_run, float l_run,
                                                  const float2 (&acc)[kGqa], RangeAttnSmem<KV>& sm, Emit emit) {
    const int warp = c.cw, lane = c.lane, tid = c.tid;
    const int hl = 2 * (lane & 1) + ((lane >> 1) & 1);
#pragma unroll
    for (int g = 0; g < kGqa; ++g) *reinterpret_cast<float2*>(&sm.wo[warp][g][2 * lane]) = acc[g];
    if (lane < 4) {
        sm.wm[warp][hl] = m_run;
        sm.wl[warp][hl] = l_run;
    }
    csync();
    {
        const int g = tid >> 6, d = tid & 63;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kCw; ++w) M = fmaxf(M, sm.wm[w][g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kCw; ++w) {
            const float e = expf(sm.wm[w][g] - M);
            L = fmaf(sm.wl[w][g], e, L);
            O = fmaf(sm.wo[w][g][d], e, O);
        }
        emit(h * kGqa + g, d, O, M, L);
    }
    fence_proxy_async_shared();  // this layer's reads of the K/V slots precede the next layer's copies
    csync();
}

template <typename KV, typename Src, typename Emit>
__device__ void attend_range_tiles(const ConsumerCtx& c, int layer, int h, int T0, int T1, int ctx, bool insert_new,
                                   const float* cs, KV* k_cache, KV* v_cache, Src qkv, Emit emit) {
    constexpr int kTileBytes = kAttnTile * kHd * static_cast<int>(sizeof(KV));
    const StepParams& p = *c.p;
    const int pos = ctx - 1;
    const int tid = c.tid, warp = c.cw, lane = c.lane;
    RangeAttnSmem<KV>& sm = *reinterpret_cast<RangeAttnSmem<KV>*>(c.xp);
    uint8_t* ring = smem_base() + kOffRing + ring_stages<true>() * kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_base() + kOffAttFull);
    int* cnt = reinterpret_cast<int*>(smem_base() + kOffAttCnt);  // arrivals per slot, then pending parity + 1
    int* pend = cnt + kAttSlots;
    const int n = T1 - T0;
    auto slot_k = [&](int sl) { return reinterpret_cast<KV*>(ring + sl * 2 * kTileBytes); };
    auto slot_v = [&](int sl) { return reinterpret_cast<KV*>(ring + sl * 2 * kTileBytes + kTileBytes); };
    // Every layer of a step uses each slot the same number of times, so tile i's phase parity follows.
    auto parity = [&](int i) {
        const int sl = i % kAttSlots;
        const int per_layer = sl < n ? (n - sl + kAttSlots - 1) / kAttSlots : 0;
        return static_cast<uint32_t>((layer * per_layer + i / kAttSlots) & 1);
    };
    const KV* kg = k_cache + static_cast<size_t>(h) * p.max_seq * kHd;
    const KV* vg = v_cache + static_cast<size_t>(h) * p.max_seq * kHd;
    auto issue = [&](int i) {
        const int t = T0 + i, sl = i % kAttSlots;
        const uint32_t bytes = static_cast<uint32_t>(min(kAttnTile, ctx - t * kAttnTile) * kHd * sizeof(KV));
        const uint64_t pol = l2_policy_evict_first();
        pend[sl] = static_cast<int>(parity(i)) + 1;
        mbar_arrive_expect_tx(&full[sl], 2 * bytes);
        bulk_load(slot_k(sl), kg + static_cast<size_t>(t) * kAttnTile * kHd, bytes, &full[sl], pol);
        bulk_load(slot_v(sl), vg + static_cast<size_t>(t) * kAttnTile * kHd, bytes, &full[sl], pol);
    };
    // Cached tiles do not depend on this step: their copies start before q is waited for.
    if (tid == 0) {
        for (int i = 0; i < min(kAttSlots, n); ++i) issue(i);
    }
    load_query_insert_kv<KV>(c, h, pos, insert_new, cs, k_cache, v_cache, qkv, sm);
    csync();
    float2 q[kGqa][8];
#pragma unroll
    for (int g = 0; g < kGqa; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[g][e] = *reinterpret_cast<const float2*>(&sm.qs[g][16 * (lane & 3) + 2 * e]);
    }
    float m_run = -INFINITY, l_run = 0.f;
    float2 acc[kGqa];
#pragma unroll
    for (int g = 0; g < kGqa; ++g) acc[g] = make_float2(0.f, 0.f);
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
        const int sl = i % kAttSlots, t = T0 + i;
        uint64_t t0 = 0;
        for (uint32_t it = 1; !__all_sync(0xffffffffu, mbar_try_wait(&full[sl], parity(i))); ++it) {
            if ((it & 63) == 0) {
                if (__any_sync(0xffffffffu, c.fl->abort != 0)) {
                    ok = false;
                    break;
                }
                const uint64_t now = __shfl_sync(0xffffffffu, global_ns(), 0);
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > p.wait_limit_ns) {
                    if (lane == 0) fail(p, c.fl, kErrWaitTimeout, 60u + layer);
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) break;
        const int nt = min(kAttnTile, ctx - t * kAttnTile);
        const int jt = 8 * warp;
        GroupRows r;
        if (jt < nt) stage_group<KV>(slot_k(sl), slot_v(sl), jt, nt, lane, r);
        // The warp's rows are in registers: it releases the slot; the last of the 8 warps refills it.
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&cnt[sl], 1) == kCw - 1) {
                cnt[sl] = 0;
                if (i + kAttSlots < n) {
                    fence_proxy_async_shared();
                    issue(i + kAttSlots);
                }
            }
        }
        if (jt < nt) {
            const int j0 = t * kAttnTile + jt;
            if (insert_new && pos >= j0 && pos < j0 + 8) patch_new_token<KV>(r, pos - j0, lane, sm);
            attend_group<KV>(r, j0, t * kAttnTile + nt, lane, warp, q, m_run, l_run, acc, sm);
        }
    }
    if (named_barrier_or(1, kCt, !ok) && tid == 0) {
        // A wait gave up: every copy issued lands before the CTA goes on (bounded).
        for (int sl = 0; sl < kAttSlots; ++sl) {
            const uint64_t t0 = global_ns();
            while (pend[sl] != 0 && !mbar_try_wait(&full[sl], static_cast<uint32_t>(pend[sl] - 1)) &&
                   global_ns() - t0 < p.drain_limit_ns) {
            }
        }
    }
    merge_warp_states<KV>(c, h, m_run, l_run, acc, sm, emit);
}

// Merges the S partials of KV head h in range order and writes the 4 query heads' outputs. Threads 0..S-1
// each acquire one range's flag (bounded polls); one barrier, which also agrees on an abort, then makes the
// partials visible to every thread. The (M, L) pairs are staged in shared memory by one load per thread;
// thread (g, d) issues the loads of all S partial outputs of query head 4h + g, dim d at once and merges them
// in range order. Returns false (all threads) if the CTA gave up.
template <typename Dst>
__device__ bool combine_splits(const ConsumerCtx& c, int h, int S, int n_slots, uint32_t tag, Dst out, unsigned id) {
    const StepParams& p = *c.p;
    if (c.tid < S) {
        const unsigned* flag = p.sync + kSyncFlags + 32 * h + c.tid;
        PollClock clk;
        for (uint32_t it = 1; ld_acquire_gpu(flag) != tag; ++it) {
            __nanosleep(64);
            if ((it & 7) == 0 && !clk.keep_going(p, c.fl, id)) break;
        }
    }
    if (named_barrier_or(1, kCt, c.fl->abort != 0)) return false;
    float2* ml = reinterpret_cast<float2*>(c.xp);  // [4][S]
    if (c.tid < kGqa * S) {
        const int g = c.tid / S, sp = c.tid % S;
        ml[c.tid] = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + static_cast<size_t>(h * kGqa + g) * n_slots + sp);
    }
    csync();
    const int g = c.tid >> 6, d = c.tid & 63;
    const float* po = p.part_o + static_cast<size_t>(h * kGqa + g) * n_slots * kHd + d;
    float ov[kAttnMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kAttnMaxSplits; ++sp) ov[sp] = sp < S ? __ldcg(po + static_cast<size_t>(sp) * kHd) : 0.f;
    float M = -INFINITY, L = 0.f, acc = 0.f;
#pragma unroll
    for (int sp = 0; sp < kAttnMaxSplits; ++sp) {
        if (sp < S) {
            const float2 m_l = ml[g * S + sp];
            const float o = ov[sp];
            const float mn = fmaxf(M, m_l.x);
            const float a = expf(M - mn), b = expf(m_l.x - mn);
            L = L * a + m_l.y * b;
            acc = acc * a + o * b;
            M = mn;
        }
    }
    out((h * kGqa + g) * kHd + d, acc / L);
    csync();
    return true;
}

// Loads the input vector of an operation into v[i] (columns 4q..4q+3, q = tid + i * kCt): the
// embedding row for the first QKV projection (src == null), else a tagged vector, where every thread
// issues all of its loads and then re-reads only the elements whose tag is not yet current (their CTAs
// are still computing) until all are. Returns false (all threads) if the CTA gave up.
template <WeightType WT>
__device__ bool load_input(ConsumerCtx& c, const unsigned long long* src, uint32_t tag, int K, int tok, unsigned id,
                           int top, float4 (&v)[kStagePer]) {
    const StepParams& p = *c.p;
    const int n4 = K / 4;
    if (src == nullptr) {
#pragma unroll
        for (int i = 0; i < kStagePer; ++i) {
            const int q = c.tid + i * kCt;
            if (q < n4) v[i] = EmbVec4<WT>{&p, tok}(q);
        }
        if (c.tid == 0) trace_mark(p, top, 1);
        return true;
    }
    uint32_t pending = 0;
#pragma unroll
    for (int i = 0; i < kStagePer; ++i) {
        const int q = c.tid + i * kCt;
        if (q < n4) {
            unsigned long long a, b, d, e;
            ld_tagged2(src + 4 * q, a, b);
            ld_tagged2(src + 4 * q + 2, d, e);
            v[i] = make_float4(tag_value(a), tag_value(b), tag_value(d), tag_value(e));
            if (!(tag_is(a, tag) && tag_is(b, tag) && tag_is(d, tag) && tag_is(e, tag))) pending |= 1u << i;
        }
    }
    PollClock clk;
    for (uint32_t it = 1; pending != 0; ++it) {  // no back-off: see get_tagged
#pragma unroll
        for (int i = 0; i < kStagePer; ++i) {
            if (pending & (1u << i)) {
                const int q = c.tid + i * kCt;
                unsigned long long a, b, d, e;
                ld_tagged2(src + 4 * q, a, b);
                ld_tagged2(src + 4 * q + 2, d, e);
                v[i] = make_float4(tag_value(a), tag_value(b), tag_value(d), tag_value(e));
                if (tag_is(a, tag) && tag_is(b, tag) && tag_is(d, tag) && tag_is(e, tag)) pending &= ~(1u << i);
            }
        }
        if ((it & 7) == 0 && !clk.keep_going(p, c.fl, id)) break;
    }
    // One barrier that also agrees on the abort flag: every consumer thread takes the same branch.
    const bool ok = !named_barrier_or(1, kCt, c.fl->abort != 0);
    if (c.tid == 0) trace_mark(p, top, 1);
    return ok;
}


// Waits for, accumulates and releases the n_seg tiles of one row group (first global tile `t0`),
// reduces the N stage rows across the warp and leaves row i's value in my[i]. Not inlined: one copy
// per (type, N) serves every operation with that tile shape.
template <WeightType WT, int N, int CPL, int ST>
__device__ __forceinline__ bool group_dot(const ConsumerCtx& c, int t0, int r0, const WOp& op, float* my) {
    const StepParams& p = *c.p;
    const TileGeom& g = op.g;
    const TileRows tr{r0, g.rows_per_tile, g.halves == 2 ? g.out_rows : 0, g.out_rows * g.halves - 1};
    const int nc = g.cols / Chunk<WT>::kCols;
    float acc[N];
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = 0.f;
    for (int sg = 0; sg < g.n_seg; ++sg) {
        const int t = t0 + sg;
        const int s = t % ST;
        if (!wait_tile(p, &c.full[s], (t / ST) & 1, c.fl, 3000u, &c.stage_tile[s], t)) return false;
        if (c.lane == 0 && sg == 0) trace_tile(p, t0, 2);
        if constexpr (kEarlyRelease && WT == WeightType::BF16) {
            // A stage a warp computes on is not refilling: with 8 warps computing, only 4 of the 12 stages carry
            // copies, which bounds the ring's refill from L2 after a hand-off near the HBM rate. Loading the
            // tile into registers in two halves (64 registers each) frees the stage half-way through its
            // arithmetic.
            constexpr int H = CPL / 2;
            static_assert(CPL % 2 == 0, "chunks per lane split in halves");
            const uint8_t* st = c.ring + s * kStageBytes;
            const int chunk0 = sg * (g.seg_bytes / 16);
            uint4 w[N][H];
            float2 a[N];
#pragma unroll
            for (int i = 0; i < N; ++i) a[i] = make_float2(0.f, 0.f);
            load_tile_regs<WT, N, H, CPL>(st, w, c.lane, 0);
            tile_dot_regs<WT, N, H>(w, chunk0, c.xp, nc, a, c.lane);
            load_tile_regs<WT, N, H, CPL>(st, w, c.lane, H);
            __syncwarp();
            if (c.lane == 0) mbar_arrive(&c.empty[s]);
            tile_dot_regs<WT, N, H>(w, chunk0 + 32 * H, c.xp, nc, a, c.lane);
#pragma unroll
            for (int i = 0; i < N; ++i) acc[i] += a[i].x + a[i].y;
        } else {
            tile_dot<WT, N, CPL>(c.ring + s * kStageBytes, tr, g.seg_bytes, sg * (g.seg_bytes / 16), c.xp, nc, c.xc, op.s,
                                 g.cols, acc, c.lane);
            __syncwarp();
            if (c.lane == 0) mbar_arrive(&c.empty[s]);
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float v = warp_sum(acc[i]);
        if (c.lane == 0) my[i] = finish_row<WT>(v, op.s, tr.global_row(i)) * c.in_scale;
    }
    __syncwarp();
    return true;
}

// Consumes this CTA's tiles of weight operation `o`; applies the epilogue of KIND.
// LM tracks the best (value, index) per lane in bv/bi. Returns false if the CTA aborted.
// Consumes this CTA's tiles of weight operation `o` (tile shape N x CPL) and applies the epilogue of
// `kind` (runtime: one copy of the tile loop serves every operation with this shape). LM tracks the
// best (value, index) per lane in bv/bi. Returns false if the CTA aborted.
template <WeightType WT, int N, int CPL, int ST>
__device__ bool run_tiles(ConsumerCtx& c, int o, int kind, float& bv, int& bi, int layer) {
    const StepParams& p = *c.p;
    const WOp op = weight_op(p, o);
    const TileGeom& g = op.g;
    const KindRows kr = reinterpret_cast<const KindRows*>(smem_base() + kOffKinds)[kind];
    const int lo = kr.lo, hi = kr.hi;
    const int R = g.rows_per_tile;
    const int ng = (hi - lo + R - 1) / R;
    float* my = c.scratch + c.cw * 32;
    if (R * g.halves != N || g.n_seg * g.seg_bytes != g.row_bytes || g.seg_bytes != CPL * 512) {
        if (c.tid == 0) fail(p, c.fl, kErrWaitTimeout, 4000u + o);  // geometry mismatch: never expected
        csync();
        return false;
    }
    bool ok = true;
    for (int grp = c.cw; grp < ng && ok; grp += kCw) {
        const int r0 = lo + grp * R;
        const int nr = min(R, hi - r0);
        if (c.lane == 0) trace_tile(p, c.t_base + grp * g.n_seg, 1);
        if (r0 + kScaleAheadRows < hi) {
            prefetch_scale_rows<WT>(op.s, g.cols, r0 + kScaleAheadRows, min(R, hi - r0 - kScaleAheadRows), c.lane, 32);
        }
        ok = group_dot<WT, N, CPL, ST>(c, c.t_base + grp * g.n_seg, r0, op, my);
        if (!ok) break;
        if (grp == 0 && c.lane == 0) trace_mark(p, trace_op_of_weight_op(o), 5);
        if (c.lane == 0) trace_tile(p, c.t_base + grp * g.n_seg, 3);
        if (c.lane < nr) {
            const int r = r0 + c.lane;
            const float d = my[c.lane];
            if (kind == kQkv) {
                st_tagged(p.t_qkv + r, d, act_tag(p, layer, kTagQkv));
            } else if (kind == kWo || kind == kDown) {
                const float v = c.res[r - lo] + d;
                c.res[r - lo] = v;
                if (kind == kWo) {
                    st_tagged(p.t_xmid + r, v, act_tag(p, layer, kTagXmid));
                } else {
                    st_tagged(p.t_xout + r, v, act_tag(p, layer, kTagXout));
                    if (p.debug_res) p.debug_res[static_cast<size_t>(layer + 1) * kH + r] = v;
                }
            } else if (kind == kGu) {
                st_tagged(p.t_act + r, silu_f(d) * my[R + c.lane], act_tag(p, layer, kTagAct));
            } else {
                __stcg(p.logits + r, d);
                if (better(d, r, bv, bi)) {
                    bv = d;
                    bi = r;
                }
            }
        }
        __syncwarp();
    }
    if (!ok) c.fl->abort = 1;
    c.t_base += kr.nt;
    return !named_barrier_or(1, kCt, !ok || c.fl->abort != 0);
}

// The epilogue of one output row (value d; SwiGLU: gate d, up u) of operation kind `kind`, row r of an
// operation whose CTA rows start at lo.
__device__ __forceinline__ void row_epilogue(const ConsumerCtx& c, int kind, int layer, int r, int lo, float d, float u,
                                             float& bv, int& bi) {
    const StepParams& p = *c.p;
    if (kind == kQkv) {
        st_tagged(p.t_qkv + r, d, act_tag(p, layer, kTagQkv));
    } else if (kind == kWo || kind == kDown) {
        const float v = c.res[r - lo] + d;
        c.res[r - lo] = v;
        if (kind == kWo) {
            st_tagged(p.t_xmid + r, v, act_tag(p, layer, kTagXmid));
        } else {
            st_tagged(p.t_xout + r, v, act_tag(p, layer, kTagXout));
            if (p.debug_res) p.debug_res[static_cast<size_t>(layer + 1) * kH + r] = v;
        }
    } else if (kind == kGu) {
        st_tagged(p.t_act + r, silu_f(d) * u, act_tag(p, layer, kTagAct));
    } else {
        __stcg(p.logits + r, d);
        if (better(d, r, bv, bi)) {
            bv = d;
            bi = r;
        }
    }
}

// Consumes this CTA's stages of weight operation `o` when several warps share each stage
// (StageShape<WT, SHAPE>::kWps > 1): warp group G = warp / kWps takes stages G, G + groups, ...; warp i of the
// group computes rows i*kHalf .. of each half of the stage, the group agrees (one named barrier, which also
// ORs a failed wait) and one thread releases the stage; then each warp applies the epilogue to its rows.
template <WeightType WT, int SHAPE, int ST>
__device__ bool run_tiles_shared(ConsumerCtx& c, int o, int kind, float& bv, int& bi, int layer) {
    using SS = StageShape<WT, SHAPE>;
    constexpr int kGroups = kCw / SS::kWps;
    constexpr int kRw = SS::kHalf;
    const StepParams& p = *c.p;
    const WOp op = weight_op(p, o);
    const TileGeom& g = op.g;
    const KindRows kr = kind_table()[kind];
    const int lo = kr.lo, hi = kr.hi;
    const int R = g.rows_per_tile;  // rows per half of a stage
    const int ng = (hi - lo + R - 1) / R;
    float* my = c.scratch + c.cw * 32;
    if (R * g.halves != SS::kRows || g.n_seg != 1 || g.seg_bytes != SS::kCpl * 512) {
        if (c.tid == 0) fail(p, c.fl, kErrWaitTimeout, 4000u + o);  // geometry mismatch: never expected
        csync();
        return false;
    }
    const int grp0 = c.cw / SS::kWps, wi = c.cw % SS::kWps;
    const int my0 = wi * kRw;  // this warp's first row (per half) within a stage
    const int nc = g.cols / Chunk<WT>::kCols;
    const int up_off = g.halves == 2 ? g.out_rows : 0, last = g.out_rows * g.halves - 1;
    bool ok = true;
    for (int grp = grp0; grp < ng; grp += kGroups) {
        const int r0 = lo + grp * R;
        const int nr = min(R, hi - r0);
        const int t = c.t_base + grp;
        const int s = t % ST;
        if (c.lane == 0 && wi == 0) trace_tile(p, t, 1);
        const TileRows tr{r0 + my0, kRw, up_off, last};
        if (wi == 0 && r0 + kScaleAheadRows < hi) {
            prefetch_scale_rows<WT>(op.s, g.cols, r0 + kScaleAheadRows, min(R, hi - r0 - kScaleAheadRows), c.lane, 32);
        }
        const bool got = wait_tile(p, &c.full[s], (t / ST) & 1, c.fl, 3000u, &c.stage_tile[s], t);
        if (c.lane == 0 && wi == 0 && got) trace_tile(p, t, 2);
        float acc[SS::kNw];
#pragma unroll
        for (int i = 0; i < SS::kNw; ++i) acc[i] = 0.f;
        if (got) {
            const uint8_t* st = c.ring + s * kStageBytes;
            tile_dot<WT, SS::kNw, SS::kCpl, kRw>(st + my0 * g.seg_bytes, tr, g.seg_bytes, 0, c.xp, nc, c.xc, op.s, g.cols, acc,
                                                  c.lane, st + (R + my0) * g.seg_bytes);
        }
        const bool failed = SS::kWps == kCw ? named_barrier_or(1, kCt, !got)
                                            : named_barrier_or(2 + grp0, SS::kWps * 32, !got);
        if (failed) {
            ok = false;
            break;
        }
        if (wi == 0 && c.lane == 0) mbar_arrive(&c.empty[s]);
#pragma unroll
        for (int i = 0; i < SS::kNw; ++i) {
            const float v = warp_sum(acc[i]);
            if (c.lane == 0) my[i] = finish_row<WT>(v, op.s, tr.global_row(i)) * c.in_scale;
        }
        __syncwarp();
        if (grp == 0 && c.lane == 0 && wi == 0) trace_mark(p, trace_op_of_weight_op(o), 5);
        if (c.lane == 0 && wi == 0) trace_tile(p, t, 3);
        if (c.lane < kRw && my0 + c.lane < nr) {
            row_epilogue(c, kind, layer, r0 + my0 + c.lane, lo, my[c.lane], g.halves == 2 ? my[kRw + c.lane] : 0.f, bv, bi);
        }
        __syncwarp();
    }
    if (!ok) c.fl->abort = 1;
    c.t_base += kr.nt;
    return !named_barrier_or(1, kCt, !ok || c.fl->abort != 0);
}

// Stages an operation's input vector into the planes of c.xp (int4: and the chunk sums into c.xc) with the
// RMSNorm's 1/rms deferred: the planes hold x * gain, and the returned factor (1/rms, or 1 without a norm)
// scales each output row after its dot product (the projection is linear). So the sum of squares needs no
// barrier of its own: each warp leaves its partial in c.red before the barrier that publishes the planes,
// and every thread then adds the kCw partials in warp order. A norm is over K == kH columns, whose gain
// (kGainPre float4s per thread) the caller loaded before it waited for v.
static_assert(kGainPre * 4 * kCt == kH, "the gain of a norm is kGainPre float4s per consumer thread");
template <WeightType WT>
__device__ __forceinline__ float stage_input(ConsumerCtx& c, float4 (&v)[kStagePer], int K, const float* norm_w,
                                             const float4 (&gain)[kGainPre], float eps) {
    constexpr int C = Chunk<WT>::kCols;
    const int nc = K / C, n4 = K / 4;
    if (norm_w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kGainPre; ++i) {
            ss = fmaf(v[i].x, v[i].x, ss);
            ss = fmaf(v[i].y, v[i].y, ss);
            ss = fmaf(v[i].z, v[i].z, ss);
            ss = fmaf(v[i].w, v[i].w, ss);
            v[i] = make_float4(v[i].x * gain[i].x, v[i].y * gain[i].y, v[i].z * gain[i].z, v[i].w * gain[i].w);
        }
        ss = warp_sum(ss);
        if (c.lane == 0) c.red[c.cw] = ss;
    }
    float4* p4 = reinterpret_cast<float4*>(c.xp);
#pragma unroll
    for (int i = 0; i < kStagePer; ++i) {
        const int q = c.tid + i * kCt;
        if (q >= n4) continue;
        const int ch = (4 * q) / C, i0 = (4 * q) % C;
        p4[(i0 >> 2) * nc + ch] = v[i];
    }
    csync();
    if constexpr (WT == WeightType::INT4) {
        for (int ch = c.tid; ch < nc; ch += kCt) {
            // Per word k: the even columns 8k, 8k+2, 8k+4, 8k+6, then the odd ones.
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 a = p4[(2 * k) * nc + ch], b = p4[(2 * k + 1) * nc + ch];
                s += a.x + a.z + b.x + b.z;
                s += a.y + a.w + b.y + b.w;
            }
            c.xc[ch] = s;
        }
        csync();
    }
    if (norm_w == nullptr) return 1.f;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kCw; ++w) t += c.red[w];
    return rsqrtf(t / static_cast<float>(K) + eps);
}

template <WeightType WT, typename KV, bool SPLIT>
__device__ void run_consumers(ConsumerCtx& c, float* cs) {
    const StepParams& p = *c.p;
    const int G = gridDim.x;
    const int pos = *p.d_pos;
    const int ctx = pos + 1;
    const int tok = p.token_override >= 0 ? p.token_override : *p.d_token;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    // SPLIT: the instantiation launched for contexts past whole_head_max_tiles (ranges of the context over
    // many CTAs, merged per head); the other runs every head on one CTA. Each is correct at any length.
    const bool whole_head = SPLIT ? attn_splits(p, n_tiles, (ctx + kHeadPassTokens - 1) / kHeadPassTokens) == 1 : true;
    const int head_stride = G / kNkv;
    rope_table(p.inv_freq, pos, cs, c.tid);
    if (c.tid == 0) {
        trace_mark(p, 0, 0);
        trace_mark(p, 0, 1);
        if (p.trace) {  // the SM this CTA runs on (slot 3 of the step-end entry is otherwise unused)
            unsigned smid;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
            p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + 81 * kTraceStamps + 3] = smid;
        }
    }
    {
        // Residual rows this CTA owns in the O/down projections start as the embedding.
        int lo, hi;
        split_rows(p.g_wo.out_rows, lo, hi);
        for (int r = lo + c.tid; r < hi; r += kCt) {
            const float v = emb_value<WT>(p, tok, r);
            c.res[r - lo] = v;
            if (p.debug_res) p.debug_res[r] = v;
        }
        csync();
    }
    constexpr int kN = stage_rows<WT, kQkv>(), kCpl = seg_chunks_per_lane<WT, kQkv>();
    constexpr int kNd = stage_rows<WT, kDown>(), kCpld = seg_chunks_per_lane<WT, kDown>();
    constexpr int kNg = stage_rows<WT, kGu>();  // gate + up rows of one tile
    static_assert(stage_rows<WT, kWo>() == kN && seg_chunks_per_lane<WT, kGu>() == kCpl, "shared tile shape");
    static_assert(seg_chunks_per_lane<WT, kWo>() == kCpl && seg_chunks_per_lane<WT, kGu>() == kCpl, "shared tile shape");
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int o = 0; o < kWeightOps; ++o) {
        const bool lm = o == kWeightOps - 1;
        const int l = lm ? kStepLayers : o / kOpsPerLayer;
        const int kind = lm ? kLm : o % kOpsPerLayer;
        const int top = lm ? 80 : l * 5 + (kind == kQkv ? 0 : kind + 1);  // trace entry of this operation
        // Input: the tagged vector the previous operation of every CTA wrote (the embedding row for the
        // first QKV projection), RMS-normalised before the QKV, gate/up and lm_head projections.
        const unsigned long long* tsrc = nullptr;
        uint32_t tag = 0;
        const float* snorm = nullptr;
        int sK = kH;
        if (kind == kQkv) {
            const size_t layer_bytes = static_cast<size_t>(l) * kNkv * p.max_seq * kHd * sizeof(KV);
            // The cached K/V rows this CTA's attention will read do not depend on this step: pull them
            // into L2 now (the same assignment as the attention below).
            if (whole_head) {
                if (blockIdx.x % head_stride == 0 && blockIdx.x / head_stride < kNkv) {
                    const int h = blockIdx.x / head_stride;
                    for (int q = c.tid; q < 2 * n_tiles; q += kCt) {
                        const int tile = q >> 1;
                        const int n = min(kAttnTile, ctx - tile * kAttnTile);
                        const size_t off = (static_cast<size_t>(h) * p.max_seq + tile * kAttnTile) * kHd * sizeof(KV);
                        const uint8_t* base = static_cast<const uint8_t*>((q & 1) ? p.v_cache : p.k_cache);
                        bulk_prefetch_l2(base + layer_bytes + off, static_cast<uint32_t>(n * kHd * sizeof(KV)));
                    }
                }
            }
            if (l > 0) {
                tsrc = p.t_xout;
                tag = act_tag(p, l - 1, kTagXout);
            }
            snorm = p.layers[l].attn_norm;
        } else if (kind == kWo) {
            // RoPE + KV write + attention (reading this layer's tagged q/k/v), then the O projection's input.
            if (c.tid == 0) {  // no separate wait: the attention polls its tagged inputs
                trace_mark(p, l * 5 + 1, 0);
                trace_mark(p, l * 5 + 1, 1);
            }
            if (whole_head) {
                if (blockIdx.x % head_stride == 0 && blockIdx.x / head_stride < kNkv) {
                    const size_t layer_off = static_cast<size_t>(l) * kNkv * p.max_seq * kHd;
                    KV* kc = static_cast<KV*>(p.k_cache) + layer_off;
                    KV* vc = static_cast<KV*>(p.v_cache) + layer_off;
                    const TaggedSrc qkv_src{&p, c.fl, p.t_qkv, act_tag(p, l, kTagQkv), 30u + l};
                    const TaggedDst att_dst{p.t_att, act_tag(p, l, kTagAtt)};
                    const int h = blockIdx.x / head_stride;
                    uint4 hk[4];  // cached keys of the first pass: independent of this step's projections
                    if (kHeadWarpTokens * c.cw < ctx) head_load_keys<KV>(kc, p.max_seq, h, pos, 0, c.cw, c.lane, hk);
                    HeadPassSmem<KV>& sm = *reinterpret_cast<HeadPassSmem<KV>*>(c.xp);
                    attend_head_pass<KV>(qkv_src, kNh, kNkv, cs, kc, vc, p.max_seq, h, ctx, att_dst, sm, c.tid, hk,
                                         [] { csync(); });
                    csync();
                }
            } else if constexpr (SPLIT) {
                const size_t layer_off = static_cast<size_t>(l) * kNkv * p.max_seq * kHd;
                KV* kc = static_cast<KV*>(p.k_cache) + layer_off;
                KV* vc = static_cast<KV*>(p.v_cache) + layer_off;
                const TaggedSrc qkv_src{&p, c.fl, p.t_qkv, act_tag(p, l, kTagQkv), 30u + l};
                const TaggedDst att_dst{p.t_att, act_tag(p, l, kTagAtt)};
                const AttnRole ar = attn_role(p, ctx);
                const int n_slots = p.max_seq / kAttnTile;  // partial slots per query head (>= any S)
                if (ar.head >= 0) {
                    const int h = ar.head, sp = ar.split;
                    // The range that holds pos inserts the new token. Partials go to slot = range; after a
                    // barrier (all of the CTA's stores done) one release store of the step's tag publishes them.
                    attend_range_tiles<KV>(
                        c, l, h, 2 * ar.p0, min(n_tiles, 2 * ar.p1), ctx, ar.p1 == ar.n_pass, cs, kc, vc, qkv_src,
                        [&](int hq, int d, float O, float M, float L) {
                            const size_t slot = static_cast<size_t>(hq) * n_slots + sp;
                            __stcg(p.part_o + slot * kHd + d, O);
                            if (d == 0) __stcg(reinterpret_cast<float2*>(p.part_ml) + slot, make_float2(M, L));
                        });
                    if (c.tid == 0) st_release_gpu(p.sync + kSyncFlags + 32 * h + sp, act_tag(p, l, kTagPart));
                } else if (ar.merge >= 0) {
                    combine_splits(c, ar.merge, ar.S, n_slots, act_tag(p, l, kTagPart), att_dst, 50u + l);
                }
            }
            if (c.tid == 0) trace_mark(p, l * 5 + 1, 2);
            if (named_barrier_or(1, kCt, c.fl->abort != 0)) return;
            tsrc = p.t_att;
            tag = act_tag(p, l, kTagAtt);
        } else if (kind == kGu) {
            tsrc = p.t_xmid;
            tag = act_tag(p, l, kTagXmid);
            snorm = p.layers[l].ffn_norm;
        } else if (kind == kDown) {
            tsrc = p.t_act;
            tag = act_tag(p, l, kTagAct);
            sK = 4 * kH;
        } else {
            tsrc = p.t_xout;
            tag = act_tag(p, kStepLayers - 1, kTagXout);
            snorm = p.final_norm;
        }
        // Neither depends on the input, so they are issued before its wait: the RMSNorm gain (into
        // registers) and the first scale rows of this CTA's tiles (into L1).
        float4 gain[kGainPre];
        if (snorm != nullptr) {
#pragma unroll
            for (int i = 0; i < kGainPre; ++i) {
                const int q = c.tid + i * kCt;
                if (q < sK / 4) gain[i] = __ldg(reinterpret_cast<const float4*>(snorm) + q);
            }
        }
        if constexpr (WT != WeightType::BF16) {
            const WOp op = weight_op(p, o);
            const KindRows kr = kind_table()[kind];
            const int n = min(kr.hi - kr.lo, kScaleAheadRows);
            prefetch_scale_rows<WT>(op.s, op.g.cols, kr.lo, n, c.tid, kCt);
            if (op.g.halves == 2) prefetch_scale_rows<WT>(op.s, op.g.cols, kr.lo + op.g.out_rows, n, c.tid, kCt);
        }
        if (c.tid == 0) trace_mark(p, top, 0);
        if (o == p.stall_op && tsrc != nullptr) tag ^= 1u << 7;  // bit 7 is in no tag a writer produces
        {
            float4 v[kStagePer];
            if (!load_input<WT>(c, tsrc, tag, sK, tok, 10u + o, top, v)) return;
            c.in_scale = stage_input<WT>(c, v, sK, snorm, gain, p.eps);
        }
        if (c.tid == 0) trace_mark(p, top, 4);
        bool ok;
        constexpr int ST = ring_stages<SPLIT>();
        if constexpr (shares_stages<WT>()) {
            ok = kind == kDown ? run_tiles_shared<WT, kDown, ST>(c, o, kind, bv, bi, l)
                 : kind == kGu ? run_tiles_shared<WT, kGu, ST>(c, o, kind, bv, bi, l)
                 : kind == kLm ? run_tiles_shared<WT, kLm, ST>(c, o, kind, bv, bi, l)
                               : run_tiles_shared<WT, kQkv, ST>(c, o, kind, bv, bi, l);
        } else {
            ok = kind == kDown ? run_tiles<WT, kNd, kCpld, ST>(c, o, kind, bv, bi, l)
                 : (kNg != kN && kind == kGu) ? run_tiles<WT, kNg, kCpl, ST>(c, o, kind, bv, bi, l)
                                              : run_tiles<WT, kN, kCpl, ST>(c, o, kind, bv, bi, l);
        }
        if (!ok) return;
        if (kind != kLm && c.tid == 0) trace_mark(p, top, 2);  // run_tiles ended with a block barrier
    }
    // ---- lm_head done: CTA argmax, then the last CTA commits the token ----------------------
    float* am_v = reinterpret_cast<float*>(c.scratch);  // scratch is free again after run_tiles
    int* am_i = reinterpret_cast<int*>(c.scratch + kCw);
    // Sampling: this CTA's top k lm_head rows become candidate keys (its logits, stored above, are read back
    // through L2; the weight ring is idle now and holds the selection's keys).
    const bool sampling = p.sample_temperature > 0.f;
    const int kk = p.sample_top_k;
    uint64_t* keys = reinterpret_cast<uint64_t*>(smem_base() + kOffRing);
    TopKScratch& tks = *reinterpret_cast<TopKScratch*>(smem_base() + kOffRing + kSampleKeyBytes);
    uint64_t* top = reinterpret_cast<uint64_t*>(smem_base() + kOffRing + kSampleKeyBytes + sizeof(TopKScratch));
    if (sampling) {
        const KindRows kr = kind_table()[kLm];
        const int n = kr.hi - kr.lo;
        csync();  // every row of this CTA stored
        for (int i = c.tid; i < n; i += kCt) keys[i] = candidate_key(__ldcg(p.logits + kr.lo + i), kr.lo + i);
        csync();
        select_top_k(keys, n, kk, top, tks, c.tid, kCt, [] { csync(); });
        for (int j = c.tid; j < kk; j += kCt) __stcg(p.cand + static_cast<size_t>(blockIdx.x) * kMaxTopK + j, top[j]);
    }
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
        const unsigned old = atom_acq_rel_gpu_add(p.sync + kSyncLm, 1u);
        c.fl->role = (old == static_cast<unsigned>(G - 1)) ? 1 : 0;
    }
    csync();
    if (c.tid == 0) {
        trace_mark(p, 80, 2);
        trace_mark(p, 81, 2);
    }
    if (c.fl->role == 0) return;
    // Last CTA: reduce the per-CTA winners (sampling: select among the CTAs' candidates and draw), commit the
    // token, advance the position, reset counters.
    int drawn = -1;
    if (sampling) {
        const int n = G * kk;
        for (int i = c.tid; i < n; i += kCt) keys[i] = __ldcg(p.cand + static_cast<size_t>(i / kk) * kMaxTopK + i % kk);
        csync();
        select_top_k(keys, n, kk, top, tks, c.tid, kCt, [] { csync(); });
        if (c.tid == 0) drawn = draw_from_top_k(top, kk, p.sample_temperature, p.sample_top_p, sample_uniform(p.sample_seed, pos));
    }
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
        *p.d_token = drawn >= 0 ? drawn : (bi2 == INT_MAX ? 0 : bi2);
        *p.d_pos = pos + 1;
        __threadfence();
    }
}

template <WeightType WT, typename KV, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* empty = full + kStages;
    volatile Flags* fl = reinterpret_cast<volatile Flags*>(smem + kOffFlags);
    volatile int* stage_tile = reinterpret_cast<volatile int*>(smem + kOffTiles);
    uint8_t* ring = smem + kOffRing;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            stage_tile[s] = -1;
        }
        if constexpr (SPLIT) {
            int* att_words = reinterpret_cast<int*>(smem + kOffAttCnt);
            for (int s = 0; s < kAttSlots; ++s) {
                mbar_init(reinterpret_cast<uint64_t*>(smem + kOffAttFull) + s, 1);
                att_words[s] = 0;              // arrivals
                att_words[kAttSlots + s] = 0;  // pending copy: none
            }
        }
        fl->abort = 0;
        fl->ok = 0;
        fl->role = 0;
        fl->issued = 0;
        init_kind_rows(p, reinterpret_cast<KindRows*>(smem + kOffKinds));
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        if (threadIdx.x < 32) {
            run_producer<ring_stages<SPLIT>()>(p, ring, full, empty, stage_tile, fl);
        } else if (threadIdx.x >= 32 && threadIdx.x < 64 && p.prefetch_mode >= 2) {
            run_prefetcher(p, fl);
        }
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
    ConsumerCtx c;
    c.p = &p;
    c.ring = ring;
    c.full = full;
    c.empty = empty;
    c.stage_tile = stage_tile;
    c.fl = fl;
    c.xp = reinterpret_cast<float*>(smem + kOffXp);
    c.xc = reinterpret_cast<float*>(smem + kOffXc);
    c.red = reinterpret_cast<float*>(smem + kOffRed);
    c.scratch = reinterpret_cast<float*>(smem + kOffScratch);
    c.res = reinterpret_cast<float*>(smem + kOffRes);
    c.tid = threadIdx.x - 128;
    c.cw = c.tid >> 5;
    c.lane = c.tid & 31;
    c.t_base = 0;
    run_consumers<WT, KV, SPLIT>(c, reinterpret_cast<float*>(smem + kOffCs));
    if (fl->abort) atomicOr(p.err, kErrAborted);
}

template <WeightType WT, typename KV, bool SPLIT>
void launch_typed(const StepParams& p, cudaStream_t stream) {
    auto kernel = decode_step_kernel<WT, KV, SPLIT>;
    static bool configured[64] = {};
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !configured[dev]) {
        CLLM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        int blocks = 0;
        CLLM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, kSmemBytes));
        CLLM_CHECK(blocks >= 1, "decode step: the persistent kernel does not fit on an SM");
        cudaFuncAttributes fa{};
        CLLM_CUDA(cudaFuncGetAttributes(&fa, kernel));
        CLLM_CHECK(fa.numRegs == kLaunchRegs, "decode step: unexpected register count; the warpgroup register split assumes 168");
        configured[dev] = true;
    }
    void* args[] = {const_cast<StepParams*>(&p)};
    CLLM_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(decode_step_grid()), dim3(kThreads), args,
                                          kSmemBytes, stream));
}

template <WeightType WT, typename KV>
void launch_kv(const StepParams& p, bool split, cudaStream_t stream) {
    if (split) {
        launch_typed<WT, KV, true>(p, stream);
    } else {
        launch_typed<WT, KV, false>(p, stream);
    }
}

}  // namespace

int decode_step_smem_bytes() { return kSmemBytes; }

int decode_step_grid() { return num_sms(); }

void launch_decode_step(const StepParams& p, WeightType wt, KvType kv, bool split, cudaStream_t stream) {
    CLLM_CHECK(p.max_seq % kAttnTile == 0, "decode step: max_seq must be a multiple of 64");
    CLLM_CHECK((kH + decode_step_grid() - 1) / decode_step_grid() <= kMaxResRows,
               "decode step: too few SMs for the on-chip residual rows");
    const bool f16 = kv == KvType::F16;
    switch (wt) {
        case WeightType::BF16:
            f16 ? launch_kv<WeightType::BF16, __half>(p, split, stream) : launch_kv<WeightType::BF16, __nv_bfloat16>(p, split, stream);
            return;
        case WeightType::INT8:
            f16 ? launch_kv<WeightType::INT8, __half>(p, split, stream) : launch_kv<WeightType::INT8, __nv_bfloat16>(p, split, stream);
            return;
        case WeightType::INT4:
            f16 ? launch_kv<WeightType::INT4, __half>(p, split, stream) : launch_kv<WeightType::INT4, __nv_bfloat16>(p, split, stream);
            return;
    }
    throw InternalError("decode step: unknown weight type");
}

}  // namespace cudallm
