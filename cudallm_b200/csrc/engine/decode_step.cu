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
constexpr int kStages = 12;
static_assert(kStages <= 32, "one producer lane per stage");
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
constexpr int kOffRed = 384;
constexpr int kOffCs = 512;
constexpr int kOffScratch = 768;
constexpr int kOffAm = kOffScratch + kCw * 32 * 4;  // 1792
// The residual rows this CTA owns (the same row range in the O and down projections), kept on chip for
// the whole step so their epilogues add without reading x back.
constexpr int kOffRes = kOffAm + kCw * 8;  // 1856
constexpr int kMaxResRows = 48;
constexpr int kOffXc = 2048;
constexpr int kOffXp = 3072;
constexpr int kOffRing = kOffXp + kMaxK * 4;  // 35840
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
// Chunks per lane of one row segment (the whole row: every Llama operation has n_seg == 1).
template <WeightType WT, int KIND>
constexpr int seg_chunks_per_lane() {
    return weight_row_bytes<WT>(KIND == 3 ? 4 * 2048 : 2048) / 512;
}

template <WeightType WT, int KIND>
constexpr int stage_rows() {
    constexpr int halves = KIND == 2 ? 2 : 1;  // gate/up
    constexpr int rb = weight_row_bytes<WT>(KIND == 3 ? 4 * 2048 : 2048);  // down has K = 8192
    constexpr int fit = kStageBytes / halves / rb;
    constexpr int cap = decode_step_tile_rows(WT);
    return (fit < cap ? fit : cap) * halves;
}

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
static_assert(kOffKinds + 5 * sizeof(KindRows) <= kOffRed, "kind table overflow");
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
__device__ void run_producer(const StepParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty, volatile int* stage_tile,
                             volatile Flags* fl) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = l2_policy_evict_first();
    TileCursor cur;
    cur.init();
    cur.advance(lane);
    int t = lane, k = 0;  // next tile of this lane; copies issued into its stage so far
    bool more = lane < kStages && cur.valid();
    uint64_t t_idle = 0;
    for (uint32_t it = 1;; ++it) {
        bool progressed = false;
        if (more && (k == 0 || mbar_test_wait(&empty[lane], (k - 1) & 1))) {
            if (cur.i == 0) trace_mark(p, trace_op_of_weight_op(cur.o), 3);
            stage_tile[lane] = t;
            trace_tile(p, t, 0);
            issue_tile(weight_op(p, cur.o), cur.lo, cur.hi, cur.i, ring + lane * kStageBytes, &full[lane], pol);
            ++k;
            t += kStages;
            cur.advance(kStages);
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
    if (lane < kStages && k > 0) wait_bar(p, &full[lane], (k - 1) & 1, fl, p.drain_limit_ns, 2000u);
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
        // Whole-row tiles (every operation of the step): rows r0 .. r0+nr-1 of each half are contiguous.
        const WOp op = weight_op(p, pf.o);
        const int r0 = pf.lo + pf.i * op.g.rows_per_tile;
        const int bytes = min(op.g.rows_per_tile, pf.hi - r0) * op.g.row_bytes;
        for (int h = 0; h < op.g.halves; ++h) {
            const uint8_t* a = op.w + (static_cast<size_t>(r0) + static_cast<size_t>(h) * op.g.out_rows) * op.g.row_bytes;
            if (p.prefetch_mode == 3) {
                if (lane == 0) bulk_prefetch_l2(a, static_cast<uint32_t>(bytes));  // one request per half (bulk engine)
            } else {
                for (int off = lane * 128; off < bytes; off += 32 * 128) {
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(a + off) : "memory");
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
    int t_base;  // global tile index of the current operation's first tile
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
    __device__ __forceinline__ bool keep_going(const StepParams& p, volatile Flags* fl, unsigned id) {
        if (fl->abort) return false;
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
        return true;
    }
};

// One element of a tagged vector, polled until it carries `tag` (or the wait gives up).
__device__ __forceinline__ float get_tagged(const StepParams& p, volatile Flags* fl, const unsigned long long* src, uint32_t tag,
                                            unsigned id) {
    unsigned long long w = ld_tagged(src);
    PollClock clk;
    for (uint32_t it = 1; !tag_is(w, tag); ++it) {
        __nanosleep(32);
        w = ld_tagged(src);
        if ((it & 15) == 0 && !clk.keep_going(p, fl, id)) break;
    }
    return tag_value(w);
}

struct TaggedSrc {
    const StepParams* p;
    volatile Flags* fl;
    const unsigned long long* v;
    uint32_t tag;
    unsigned id;
    __device__ __forceinline__ float operator()(int i) const { return get_tagged(*p, fl, v + i, tag, id); }
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
    for (uint32_t it = 1; pending != 0; ++it) {
        __nanosleep(64);
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
template <WeightType WT, int N, int CPL>
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
        const int s = t % kStages;
        if (!wait_tile(p, &c.full[s], (t / kStages) & 1, c.fl, 3000u, &c.stage_tile[s], t)) return false;
        if (c.lane == 0 && sg == 0) trace_tile(p, t0, 2);
        tile_dot<WT, N, CPL>(c.ring + s * kStageBytes, tr, g.seg_bytes, sg * (g.seg_bytes / 16), c.xp, nc, c.xc, op.s, g.cols,
                             acc, c.lane);
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&c.empty[s]);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float v = warp_sum(acc[i]);
        if (c.lane == 0) my[i] = finish_row<WT>(v, op.s, tr.global_row(i));
    }
    __syncwarp();
    return true;
}

// Consumes this CTA's tiles of weight operation `o`; applies the epilogue of KIND.
// LM tracks the best (value, index) per lane in bv/bi. Returns false if the CTA aborted.
// Consumes this CTA's tiles of weight operation `o` (tile shape N x CPL) and applies the epilogue of
// `kind` (runtime: one copy of the tile loop serves every operation with this shape). LM tracks the
// best (value, index) per lane in bv/bi. Returns false if the CTA aborted.
template <WeightType WT, int N, int CPL>
__device__ bool run_tiles(ConsumerCtx& c, int o, int kind, float& bv, int& bi, int layer) {
    const StepParams& p = *c.p;
    const WOp op = weight_op(p, o);
    const TileGeom& g = op.g;
    const KindRows kr = reinterpret_cast<const KindRows*>(smem_base() + kOffKinds)[kind];
    const int lo = kr.lo, hi = kr.hi;
    const int R = g.rows_per_tile;
    const int ng = (hi - lo + R - 1) / R;
    float* my = c.scratch + c.cw * 32;
    if (R * g.halves != N || g.n_seg != 1 || g.seg_bytes != CPL * 512) {
        if (c.tid == 0) fail(p, c.fl, kErrWaitTimeout, 4000u + o);  // geometry mismatch: never expected
        csync();
        return false;
    }
    bool ok = true;
    for (int grp = c.cw; grp < ng && ok; grp += kCw) {
        const int r0 = lo + grp * R;
        const int nr = min(R, hi - r0);
        if (c.lane == 0) trace_tile(p, c.t_base + grp * g.n_seg, 1);
        ok = group_dot<WT, N, CPL>(c, c.t_base + grp * g.n_seg, r0, op, my);
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

// The cached K/V rows of this CTA's range (split contexts) into L2, before the layer's attention needs them.
template <typename KV>
__device__ __forceinline__ void prefetch_split_kv(const ConsumerCtx& c, size_t layer_bytes, int ctx) {
    const StepParams& p = *c.p;
    const AttnRole ar = attn_role(p, ctx);
    if (ar.head < 0) return;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    const int t0 = 2 * ar.p0, t1 = min(n_tiles, 2 * ar.p1);
    for (int q = c.tid; q < 2 * (t1 - t0); q += kCt) {
        const int tile = t0 + (q >> 1);
        const int n = min(kAttnTile, ctx - tile * kAttnTile);
        const size_t off = (static_cast<size_t>(ar.head) * p.max_seq + tile * kAttnTile) * kHd * sizeof(KV);
        const uint8_t* base = static_cast<const uint8_t*>((q & 1) ? p.v_cache : p.k_cache);
        bulk_prefetch_l2(base + layer_bytes + off, static_cast<uint32_t>(n * kHd * sizeof(KV)));
    }
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
            } else if constexpr (SPLIT) {
                prefetch_split_kv<KV>(c, layer_bytes, ctx);
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
                    uint4 hk[4];  // cached keys of the range's first pass: independent of this step's projections
                    if (ar.p0 * kHeadPassTokens + kHeadWarpTokens * c.cw < ctx) {
                        head_load_keys<KV>(kc, p.max_seq, h, pos, ar.p0, c.cw, c.lane, hk);
                    }
                    HeadPassSmem<KV>& sm = *reinterpret_cast<HeadPassSmem<KV>*>(c.xp);
                    // The range that holds pos inserts the new token. Partials go to slot = range; after a
                    // barrier (all of the CTA's stores done) one release store of the step's tag publishes them.
                    attend_head_span<KV>(
                        qkv_src, kNh, kNkv, cs, kc, vc, p.max_seq, h, ctx, ar.p0, ar.p1, ar.p1 == ar.n_pass,
                        [&](int hq, int d, float O, float M, float L) {
                            const size_t slot = static_cast<size_t>(hq) * n_slots + sp;
                            __stcg(p.part_o + slot * kHd + d, O);
                            if (d == 0) __stcg(reinterpret_cast<float2*>(p.part_ml) + slot, make_float2(M, L));
                        },
                        sm, c.tid, hk, [] { csync(); });
                    csync();
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
        if (c.tid == 0) trace_mark(p, top, 0);
        if (o == p.stall_op && tsrc != nullptr) tag ^= 1u << 7;  // bit 7 is in no tag a writer produces
        {
            float4 v[kStagePer];
            if (!load_input<WT>(c, tsrc, tag, sK, tok, 10u + o, top, v)) return;
            stage_commit<WT>(v, sK, snorm, p.eps, c.xp, c.xc, c.red, c.tid, kCt, [] { csync(); });
        }
        if (c.tid == 0) trace_mark(p, top, 4);
        const bool ok = kind == kDown ? run_tiles<WT, kNd, kCpld>(c, o, kind, bv, bi, l)
                        : (kNg != kN && kind == kGu) ? run_tiles<WT, kNg, kCpl>(c, o, kind, bv, bi, l)
                                                     : run_tiles<WT, kN, kCpl>(c, o, kind, bv, bi, l);
        if (!ok) return;
        if (kind != kLm && c.tid == 0) trace_mark(p, top, 2);  // run_tiles ended with a block barrier
    }
    // ---- lm_head done: CTA argmax, then the last CTA commits the token ----------------------
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
        const unsigned old = atom_acq_rel_gpu_add(p.sync + kSyncLm, 1u);
        c.fl->role = (old == static_cast<unsigned>(G - 1)) ? 1 : 0;
    }
    csync();
    if (c.tid == 0) {
        trace_mark(p, 80, 2);
        trace_mark(p, 81, 2);
    }
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
            run_producer(p, ring, full, empty, stage_tile, fl);
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
