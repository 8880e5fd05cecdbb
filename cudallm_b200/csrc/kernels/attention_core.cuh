// Decode attention building blocks, shared by the per-op split-K kernels and the persistent decode
// step. Semantics follow wasiqnauman/cudallm src/kernels/attention_opt.cu:24-134 and
// python/cudallm/reference.py:141-149: GQA with 4 query heads per KV head, head_dim 64, score
// scale 0.125, per-split (m, l, unnormalised o) partials merged in fixed split order (no atomics in
// the arithmetic, so results are bit-reproducible).
//
// One *attention tile* = (KV head h, 64 consecutive context tokens). A 256-thread group loads the
// tile's K and V once into shared memory and serves all 4 query heads of the group: warp w scores
// query head w/2 against tokens 32*(w%2)+lane (K rows padded to 66 halves so the lane-per-token reads
// are conflict-free), then thread (g, d) = (tid/64, tid%64) accumulates p.V for its output dim.
// RoPE (HF rotate_half pairs (i, i+32), angle = float(pos) * inv_freq[i] in fp32,
// reference src/kernels/rope_kv.cu:48-79) is applied to the query heads here, and the tile holding
// the current position also rotates the new key, rounds k and v to the cache type, writes them to the
// cache and uses the rounded values, exactly as a cache round trip would.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "kernels/matvec_core.cuh"

namespace cudallm {

constexpr int kHd = 64;           // head_dim
constexpr int kGqa = 4;           // query heads per KV head
constexpr int kAttThreads = 256;  // threads serving one tile
constexpr int kKsStride = kHd + 2;

template <typename KV>
__device__ __forceinline__ KV to_kv(float v);
template <>
__device__ __forceinline__ __half to_kv<__half>(float v) {
    return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 to_kv<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
__device__ __forceinline__ float kv_to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float kv_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float2 kv2_to_float2(__half2 v) { return __half22float2(v); }
__device__ __forceinline__ float2 kv2_to_float2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
template <typename KV>
struct Kv2;
template <>
struct Kv2<__half> {
    using T = __half2;
};
template <>
struct Kv2<__nv_bfloat16> {
    using T = __nv_bfloat162;
};

template <typename KV>
struct AttSmem {
    KV ks[kAttnTile][kKsStride];
    alignas(16) KV vs[kAttnTile][kHd];
    float qs[kGqa][kHd];
    float ps[kGqa][kAttnTile];
    float red[2][kGqa][2];
};

// Element access of the q/k/v input and of the attention output: plain fp32 vectors read and written
// through L2 (the per-op kernels); the persistent step supplies tagged-word accessors instead.
struct PlainSrc {
    const float* p;
    __device__ __forceinline__ float operator()(int i) const { return __ldcg(p + i); }
    __device__ __forceinline__ float2 pair(int i, int j) const { return make_float2(__ldcg(p + i), __ldcg(p + j)); }
};
struct PlainDst {
    float* p;
    __device__ __forceinline__ void operator()(int i, float v) const { __stcg(p + i, v); }
};

// cos/sin of angle float(pos) * inv_freq[i] for i < 32, into cs[0..31] (cos) and cs[32..63] (sin).
__device__ __forceinline__ void rope_table(const float* __restrict__ inv_freq, int pos, float* cs, int tid) {
    if (tid < kHd / 2) {
        const float ang = static_cast<float>(pos) * inv_freq[tid];
        float s, c;
        sincosf(ang, &s, &c);
        cs[tid] = c;
        cs[kHd / 2 + tid] = s;
    }
}

// Processes tile `tile` of KV head `h` for context length ctx (= pos + 1). qkv holds the raw
// (un-rotated) projections [q 32x64 | k 8x64 | v 8x64]; cs is the rope table of pos. Writes the
// partial (o[4][64], m[4], l[4]) at slot `tile` of part_o [32][n_slots][64] / part_ml [32][n_slots][2].
// `sync()` is a barrier over the 256 participating threads (tid 0..255). Loads of data produced by
// other CTAs of the same kernel go through L2 (ld.cg).
// FUSED = true (persistent decode step): q/k/v are the raw projections in qkv ([q nh | k nkv | v nkv]
// heads of 64), q is rotated here and the new token is inserted. FUSED = false: qkv points at the final
// (already rotated) q [nh][64] and the cache already holds every context token.
template <typename KV, bool FUSED, typename Sync, typename Src = PlainSrc>
__device__ __forceinline__ void attend_tile(Src qkv, int nh, int nkv, const float* cs, KV* k_cache, KV* v_cache,
                                            int max_seq, int h, int tile, int ctx, int n_slots, float* part_o,
                                            float* part_ml, AttSmem<KV>& sm, int tid, Sync sync) {
    using KV2 = typename Kv2<KV>::T;
    const int pos = ctx - 1;
    const int t0 = tile * kAttnTile;
    const int n = min(kAttnTile, ctx - t0);
    const KV* Kg = k_cache + (static_cast<size_t>(h) * max_seq + t0) * kHd;
    const KV* Vg = v_cache + (static_cast<size_t>(h) * max_seq + t0) * kHd;
    for (int idx = tid; idx < n * 8; idx += kAttThreads) {
        const int t = idx >> 3, c = idx & 7;
        const uint4 kv = __ldcg(reinterpret_cast<const uint4*>(Kg + t * kHd) + c);
        const uint4 vv = __ldcg(reinterpret_cast<const uint4*>(Vg + t * kHd) + c);
        uint32_t* kd = reinterpret_cast<uint32_t*>(&sm.ks[t][c * 8]);
        kd[0] = kv.x;
        kd[1] = kv.y;
        kd[2] = kv.z;
        kd[3] = kv.w;
        *reinterpret_cast<uint4*>(&sm.vs[t][c * 8]) = vv;
    }
    // Query heads h*4 .. h*4+3 (rotated here when FUSED).
    if (tid < kGqa * kHd / 2) {
        const int g = tid >> 5, i = tid & 31;
        const int q = (h * kGqa + g) * kHd;
        const float x0 = qkv(q + i), x1 = qkv(q + i + kHd / 2);
        if constexpr (FUSED) {
            const float c = cs[i], s = cs[kHd / 2 + i];
            sm.qs[g][i] = x0 * c - x1 * s;
            sm.qs[g][i + kHd / 2] = x1 * c + x0 * s;
        } else {
            sm.qs[g][i] = x0;
            sm.qs[g][i + kHd / 2] = x1;
        }
    }
    sync();
    if (FUSED && pos >= t0 && pos < t0 + n) {
        // This tile holds the new token: rotate k, round k/v to the cache type, publish, use.
        const int r = pos - t0;
        if (tid < kHd / 2) {
            const int k = (nh + h) * kHd;
            const float x0 = qkv(k + tid), x1 = qkv(k + tid + kHd / 2);
            const float c = cs[tid], s = cs[kHd / 2 + tid];
            const KV k0 = to_kv<KV>(x0 * c - x1 * s);
            const KV k1 = to_kv<KV>(x1 * c + x0 * s);
            sm.ks[r][tid] = k0;
            sm.ks[r][tid + kHd / 2] = k1;
            KV* kdst = k_cache + (static_cast<size_t>(h) * max_seq + pos) * kHd;
            kdst[tid] = k0;
            kdst[tid + kHd / 2] = k1;
        } else if (tid < kHd / 2 + kHd) {
            const int d = tid - kHd / 2;
            const KV v = to_kv<KV>(qkv((nh + nkv + h) * kHd + d));
            sm.vs[r][d] = v;
            v_cache[(static_cast<size_t>(h) * max_seq + pos) * kHd + d] = v;
        }
        sync();
    }
    const int w = tid >> 5, lane = tid & 31;
    const int g = w >> 1, half = w & 1;
    const int j = half * 32 + lane;
    float s = -INFINITY;
    if (j < n) {
        const KV2* krow = reinterpret_cast<const KV2*>(&sm.ks[j][0]);
        float dot = 0.f;
#pragma unroll 8
        for (int d2 = 0; d2 < kHd / 2; ++d2) {
            const float2 kf = kv2_to_float2(krow[d2]);
            dot = fmaf(kf.x, sm.qs[g][2 * d2], dot);
            dot = fmaf(kf.y, sm.qs[g][2 * d2 + 1], dot);
        }
        s = 0.125f * dot;
    }
    const float wm = warp_max(s);
    if (lane == 0) sm.red[0][g][half] = wm;
    sync();
    const float m = fmaxf(sm.red[0][g][0], sm.red[0][g][1]);
    const float p = (j < n) ? expf(s - m) : 0.f;
    sm.ps[g][j] = p;
    const float wl = warp_sum(p);
    if (lane == 0) sm.red[1][g][half] = wl;
    sync();
    {
        const int gg = tid >> 6, d = tid & 63;
        float o = 0.f;
        for (int t = 0; t < n; ++t) o = fmaf(sm.ps[gg][t], kv_to_float(sm.vs[t][d]), o);
        const int hq = h * kGqa + gg;
        const size_t slot = static_cast<size_t>(hq) * n_slots + tile;
        __stcg(part_o + slot * kHd + d, o);
        if (d == 0) {
            __stcg(part_ml + slot * 2, fmaxf(sm.red[0][gg][0], sm.red[0][gg][1]));
            __stcg(part_ml + slot * 2 + 1, sm.red[1][gg][0] + sm.red[1][gg][1]);
        }
    }
    sync();
}

// Merges the n_tiles partials of the 4 query heads of KV head h in tile order (one pass with a
// running maximum) and writes out[hq*64 + d]. Thread (g, d) = (tid/64, tid%64) of a 256-thread group.
template <typename Dst = PlainDst>
__device__ __forceinline__ void combine_head(const float* part_o, const float* part_ml, int h, int n_tiles, int n_slots,
                                             Dst out, int tid) {
    const int g = tid >> 6, d = tid & 63;
    const int hq = h * kGqa + g;
    const float2* ml = reinterpret_cast<const float2*>(part_ml + static_cast<size_t>(hq) * n_slots * 2);
    const float* po = part_o + static_cast<size_t>(hq) * n_slots * kHd;
    float M = -INFINITY, L = 0.f, acc = 0.f;
#pragma unroll 4
    for (int c = 0; c < n_tiles; ++c) {
        const float2 mlc = __ldcg(ml + c);
        const float o = __ldcg(po + static_cast<size_t>(c) * kHd + d);
        const float mn = fmaxf(M, mlc.x);
        const float a = expf(M - mn), b = expf(mlc.x - mn);
        L = L * a + mlc.y * b;
        acc = acc * a + o * b;
        M = mn;
    }
    out(hq * kHd + d, acc / L);
}

// ---- whole-head attention (short contexts) -------------------------------------------------------
// One 256-thread group computes all 4 query heads of KV head h over the whole context: warp w takes
// tiles w, w+8, ... (64 tokens each) straight from the cache (through L2), keeps a running softmax
// (max, sum, p.V) per head, and the 8 warp states are merged in warp order. No partials leave the
// CTA, so there is no second pass. Lane j scores tokens t0+j and t0+j+32; for p.V, lane group
// g = lane/8 takes tokens t0 + 4i + g and lane sub = lane%8 owns dims 8*sub .. 8*sub+7.
template <typename KV>
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
    using KV2 = typename Kv2<KV>::T;
    const KV2* h2 = reinterpret_cast<const KV2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 f = kv2_to_float2(h2[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
    }
}

// ---- Whole-head attention (short contexts) -------------------------------------------------------
// One 256-thread group computes all 4 query heads of KV head h over the whole context, in passes of
// 128 tokens: warp w owns tokens p0 + 16w + i. For the scores, lane pair (2i, 2i+1) holds the key row of
// token i (dims 0-31 and 32-63); for p.V, lane l holds V[token][2l .. 2l+1] of each of the 16 tokens.
// The keys of pass 0 are loaded before the step's QKV dependency (they are cached rows); later passes
// load their keys at the pass start. Values are loaded right after the scores (their latency overlaps
// the softmax). Each warp keeps a running softmax (max, sum, p.V) per query head; the 8 warp states are
// merged in warp order.
constexpr int kHeadWarpTokens = 16;
constexpr int kHeadPassTokens = 8 * kHeadWarpTokens;

template <typename KV>
struct HeadPassSmem {
    float qs[kGqa][kHd];
    alignas(16) KV kn[kHd];
    alignas(16) KV vn[kHd];
    float4 ps[8][kHeadWarpTokens];  // p of the 4 query heads for each token of the warp
    float wm[8][kGqa];
    float wl[8][kGqa];
    float wo[8][kGqa][kHd];
};

// Key loads (lane pair per token) and value loads (row by row) of pass `pass` for warp w: cached
// tokens below pos only (the current token is inserted from shared memory); everything else is zero.
template <typename KV>
__device__ __forceinline__ void head_load_keys(const KV* k_cache, int max_seq, int h, int pos, int pass, int w, int lane,
                                               uint4 (&k)[4]) {
    const KV* Kh = k_cache + static_cast<size_t>(h) * max_seq * kHd;
    const int j = pass * kHeadPassTokens + kHeadWarpTokens * w + (lane >> 1);
    const uint4* krow = reinterpret_cast<const uint4*>(Kh + static_cast<size_t>(j) * kHd) + 4 * (lane & 1);
#pragma unroll
    for (int c = 0; c < 4; ++c) k[c] = j < pos ? __ldcg(krow + c) : make_uint4(0, 0, 0, 0);
}
template <typename KV>
__device__ __forceinline__ void head_load_values(const KV* v_cache, int max_seq, int h, int pos, int pass, int w, int lane,
                                                 uint32_t (&v)[kHeadWarpTokens]) {
    const KV* Vh = v_cache + static_cast<size_t>(h) * max_seq * kHd;
    const int base = pass * kHeadPassTokens + kHeadWarpTokens * w;
#pragma unroll
    for (int i = 0; i < kHeadWarpTokens; ++i) {
        v[i] = base + i < pos ? __ldcg(reinterpret_cast<const uint32_t*>(Vh + static_cast<size_t>(base + i) * kHd) + lane) : 0u;
    }
}

// Attention of KV head h for context ctx (= pos + 1) over the 128-token passes [pass_lo, pass_hi): rotates
// the 4 query heads (cs = rope table of pos). The range that holds pos (insert_new) also rotates the new key,
// rounds k and v to the cache type, writes them to the cache and uses the rounded values; every other range
// only reads cached tokens below pos. k holds the keys of pass pass_lo (head_load_keys, issued by the caller
// before it waited for the QKV projection: they do not depend on this step); later passes load their keys
// at the pass start, and every pass loads its values after the scores (their latency overlaps the softmax).
// The caller prefetches the range's cached rows into L2 when the layer starts. The 8 warps' running softmax states are merged in warp order and handed to
// emit(hq, d, O, M, L) for query head hq = 4h + 0..3 and dim d (thread tid = 64 (hq - 4h) + d): O = sum of
// exp(s - M) v over the range, L = sum of exp(s - M). `sync()` is a barrier over the 256 participating threads.
template <typename KV, typename Sync, typename Src, typename Emit>
__device__ __forceinline__ void attend_head_span(Src qkv, int nh, int nkv, const float* cs, KV* k_cache, KV* v_cache,
                                                 int max_seq, int h, int ctx, int pass_lo, int pass_hi, bool insert_new,
                                                 Emit emit, HeadPassSmem<KV>& sm, int tid, uint4 (&k)[4], Sync sync) {
    using KV2 = typename Kv2<KV>::T;
    const int pos = ctx - 1;
    const int w = tid >> 5, lane = tid & 31;
    if (tid < kGqa * kHd / 2) {
        const int g = tid >> 5, i = tid & 31;
        const int q = (h * kGqa + g) * kHd;
        const float2 x = qkv.pair(q + i, q + i + kHd / 2);  // both loads in flight at once
        const float x0 = x.x, x1 = x.y;
        const float c = cs[i], s = cs[kHd / 2 + i];
        sm.qs[g][i] = x0 * c - x1 * s;
        sm.qs[g][i + kHd / 2] = x1 * c + x0 * s;
    } else if (insert_new && tid < kGqa * kHd / 2 + kHd / 2) {
        const int i = tid - kGqa * kHd / 2;
        const int kp = (nh + h) * kHd;
        const float2 x = qkv.pair(kp + i, kp + i + kHd / 2);
        const float x0 = x.x, x1 = x.y;
        const float c = cs[i], s = cs[kHd / 2 + i];
        const KV k0 = to_kv<KV>(x0 * c - x1 * s), k1 = to_kv<KV>(x1 * c + x0 * s);
        sm.kn[i] = k0;
        sm.kn[i + kHd / 2] = k1;
        KV* kdst = k_cache + (static_cast<size_t>(h) * max_seq + pos) * kHd;
        kdst[i] = k0;
        kdst[i + kHd / 2] = k1;
    } else if (insert_new && tid < kGqa * kHd / 2 + kHd / 2 + kHd) {
        const int d = tid - kGqa * kHd / 2 - kHd / 2;
        const KV vv = to_kv<KV>(qkv((nh + nkv + h) * kHd + d));
        sm.vn[d] = vv;
        v_cache[(static_cast<size_t>(h) * max_seq + pos) * kHd + d] = vv;
    }
    sync();
    float m_run[kGqa], l_run[kGqa], o[kGqa][2];
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
        m_run[hq] = -INFINITY;
        l_run[hq] = 0.f;
        o[hq][0] = o[hq][1] = 0.f;
    }
    for (int pass = pass_lo; pass < pass_hi; ++pass) {
        const int base = pass * kHeadPassTokens + kHeadWarpTokens * w;
        if (base >= ctx) break;  // warp-uniform: no token of this warp is in the context
        if (pass > pass_lo) head_load_keys<KV>(k_cache, max_seq, h, pos, pass, w, lane, k);
        const int j = base + (lane >> 1), half = lane & 1;
        if (j == pos) {
#pragma unroll
            for (int c = 0; c < 4; ++c) k[c] = reinterpret_cast<const uint4*>(sm.kn)[4 * half + c];
        }
        float dot[kGqa] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float kf[8];
            unpack8<KV>(k[c], kf);
#pragma unroll
            for (int hq = 0; hq < kGqa; ++hq) {
#pragma unroll
                for (int e = 0; e < 8; ++e) dot[hq] = fmaf(kf[e], sm.qs[hq][32 * half + 8 * c + e], dot[hq]);
            }
        }
        // Values: loaded once the key registers are free; their latency overlaps the softmax.
        uint32_t v[kHeadWarpTokens];
        head_load_values<KV>(v_cache, max_seq, h, pos, pass, w, lane, v);
        if (pos >= base && pos < base + kHeadWarpTokens) {
#pragma unroll
            for (int i = 0; i < kHeadWarpTokens; ++i) {
                if (base + i == pos) v[i] = reinterpret_cast<const uint32_t*>(sm.vn)[lane];
            }
        }
        float pj[kGqa];
#pragma unroll
        for (int hq = 0; hq < kGqa; ++hq) {
            const float d = dot[hq] + __shfl_xor_sync(0xffffffffu, dot[hq], 1);  // both halves of the row
            const float sc = j < ctx ? 0.125f * d : -INFINITY;
            const float mn = fmaxf(m_run[hq], warp_max(sc));  // finite: the warp's first token is in the context
            const float a = expf(m_run[hq] - mn);
            pj[hq] = expf(sc - mn);
            l_run[hq] = l_run[hq] * a + 0.5f * warp_sum(pj[hq]);  // every token is counted by its two lanes
            o[hq][0] *= a;
            o[hq][1] *= a;
            m_run[hq] = mn;
        }
        if (half == 0) sm.ps[w][lane >> 1] = make_float4(pj[0], pj[1], pj[2], pj[3]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < kHeadWarpTokens; ++i) {
            const float4 p4 = sm.ps[w][i];
            const float2 vf = kv2_to_float2(*reinterpret_cast<const KV2*>(&v[i]));
            o[0][0] = fmaf(p4.x, vf.x, o[0][0]);
            o[0][1] = fmaf(p4.x, vf.y, o[0][1]);
            o[1][0] = fmaf(p4.y, vf.x, o[1][0]);
            o[1][1] = fmaf(p4.y, vf.y, o[1][1]);
            o[2][0] = fmaf(p4.z, vf.x, o[2][0]);
            o[2][1] = fmaf(p4.z, vf.y, o[2][1]);
            o[3][0] = fmaf(p4.w, vf.x, o[3][0]);
            o[3][1] = fmaf(p4.w, vf.y, o[3][1]);
        }
        __syncwarp();
    }
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
        *reinterpret_cast<float2*>(&sm.wo[w][hq][2 * lane]) = make_float2(o[hq][0], o[hq][1]);
        if (lane == 0) {
            sm.wm[w][hq] = m_run[hq];
            sm.wl[w][hq] = l_run[hq];
        }
    }
    sync();
    {
        const int g = tid >> 6, d = tid & 63;
        float M = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) M = fmaxf(M, sm.wm[ww][g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) {
            const float e = expf(sm.wm[ww][g] - M);  // 0 for a warp that had no token
            L = fmaf(sm.wl[ww][g], e, L);
            O = fmaf(sm.wo[ww][g][d], e, O);
        }
        emit(h * kGqa + g, d, O, M, L);
    }
}

// Attention of KV head h for context ctx (= pos + 1): rotates the 4 query heads and the new key
// (cs = rope table of pos), rounds k and v to the cache type, writes them to the cache and uses the
// rounded values. out receives [4][64] at query head 4h. k holds the keys of pass 0 (head_load_keys,
// issued by the caller before it waited for the QKV projection: they do not depend on this step).
// `sync()` is a barrier over the 256 participating threads.
template <typename KV, typename Sync, typename Src, typename Dst>
__device__ __forceinline__ void attend_head_pass(Src qkv, int nh, int nkv, const float* cs, KV* k_cache, KV* v_cache,
                                                 int max_seq, int h, int ctx, Dst out, HeadPassSmem<KV>& sm, int tid,
                                                 uint4 (&k)[4], Sync sync) {
    using KV2 = typename Kv2<KV>::T;
    const int pos = ctx - 1;
    const int w = tid >> 5, lane = tid & 31;
    if (tid < kGqa * kHd / 2) {
        const int g = tid >> 5, i = tid & 31;
        const int q = (h * kGqa + g) * kHd;
        const float2 x = qkv.pair(q + i, q + i + kHd / 2);  // both loads in flight at once
        const float x0 = x.x, x1 = x.y;
        const float c = cs[i], s = cs[kHd / 2 + i];
        sm.qs[g][i] = x0 * c - x1 * s;
        sm.qs[g][i + kHd / 2] = x1 * c + x0 * s;
    } else if (tid < kGqa * kHd / 2 + kHd / 2) {
        const int i = tid - kGqa * kHd / 2;
        const int kp = (nh + h) * kHd;
        const float2 x = qkv.pair(kp + i, kp + i + kHd / 2);
        const float x0 = x.x, x1 = x.y;
        const float c = cs[i], s = cs[kHd / 2 + i];
        const KV k0 = to_kv<KV>(x0 * c - x1 * s), k1 = to_kv<KV>(x1 * c + x0 * s);
        sm.kn[i] = k0;
        sm.kn[i + kHd / 2] = k1;
        KV* kdst = k_cache + (static_cast<size_t>(h) * max_seq + pos) * kHd;
        kdst[i] = k0;
        kdst[i + kHd / 2] = k1;
    } else if (tid < kGqa * kHd / 2 + kHd / 2 + kHd) {
        const int d = tid - kGqa * kHd / 2 - kHd / 2;
        const KV vv = to_kv<KV>(qkv((nh + nkv + h) * kHd + d));
        sm.vn[d] = vv;
        v_cache[(static_cast<size_t>(h) * max_seq + pos) * kHd + d] = vv;
    }
    sync();
    float m_run[kGqa], l_run[kGqa], o[kGqa][2];
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
        m_run[hq] = -INFINITY;
        l_run[hq] = 0.f;
        o[hq][0] = o[hq][1] = 0.f;
    }
    const int n_pass = (ctx + kHeadPassTokens - 1) / kHeadPassTokens;
    for (int pass = 0; pass < n_pass; ++pass) {
        const int base = pass * kHeadPassTokens + kHeadWarpTokens * w;
        if (base >= ctx) break;  // warp-uniform: no token of this warp is in the context
        if (pass > 0) head_load_keys<KV>(k_cache, max_seq, h, pos, pass, w, lane, k);
        const int j = base + (lane >> 1), half = lane & 1;
        if (j == pos) {
#pragma unroll
            for (int c = 0; c < 4; ++c) k[c] = reinterpret_cast<const uint4*>(sm.kn)[4 * half + c];
        }
        float dot[kGqa] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float kf[8];
            unpack8<KV>(k[c], kf);
#pragma unroll
            for (int hq = 0; hq < kGqa; ++hq) {
#pragma unroll
                for (int e = 0; e < 8; ++e) dot[hq] = fmaf(kf[e], sm.qs[hq][32 * half + 8 * c + e], dot[hq]);
            }
        }
        // Values: loaded once the key registers are free; their latency overlaps the softmax.
        uint32_t v[kHeadWarpTokens];
        head_load_values<KV>(v_cache, max_seq, h, pos, pass, w, lane, v);
        if (pos >= base && pos < base + kHeadWarpTokens) {
#pragma unroll
            for (int i = 0; i < kHeadWarpTokens; ++i) {
                if (base + i == pos) v[i] = reinterpret_cast<const uint32_t*>(sm.vn)[lane];
            }
        }
        float pj[kGqa];
#pragma unroll
        for (int hq = 0; hq < kGqa; ++hq) {
            const float d = dot[hq] + __shfl_xor_sync(0xffffffffu, dot[hq], 1);  // both halves of the row
            const float sc = j < ctx ? 0.125f * d : -INFINITY;
            const float mn = fmaxf(m_run[hq], warp_max(sc));  // finite: the warp's first token is in the context
            const float a = expf(m_run[hq] - mn);
            pj[hq] = expf(sc - mn);
            l_run[hq] = l_run[hq] * a + 0.5f * warp_sum(pj[hq]);  // every token is counted by its two lanes
            o[hq][0] *= a;
            o[hq][1] *= a;
            m_run[hq] = mn;
        }
        if (half == 0) sm.ps[w][lane >> 1] = make_float4(pj[0], pj[1], pj[2], pj[3]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < kHeadWarpTokens; ++i) {
            const float4 p4 = sm.ps[w][i];
            const float2 vf = kv2_to_float2(*reinterpret_cast<const KV2*>(&v[i]));
            o[0][0] = fmaf(p4.x, vf.x, o[0][0]);
            o[0][1] = fmaf(p4.x, vf.y, o[0][1]);
            o[1][0] = fmaf(p4.y, vf.x, o[1][0]);
            o[1][1] = fmaf(p4.y, vf.y, o[1][1]);
            o[2][0] = fmaf(p4.z, vf.x, o[2][0]);
            o[2][1] = fmaf(p4.z, vf.y, o[2][1]);
            o[3][0] = fmaf(p4.w, vf.x, o[3][0]);
            o[3][1] = fmaf(p4.w, vf.y, o[3][1]);
        }
        __syncwarp();
    }
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
        *reinterpret_cast<float2*>(&sm.wo[w][hq][2 * lane]) = make_float2(o[hq][0], o[hq][1]);
        if (lane == 0) {
            sm.wm[w][hq] = m_run[hq];
            sm.wl[w][hq] = l_run[hq];
        }
    }
    sync();
    {
        const int hq = tid >> 6, d = tid & 63;
        float M = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) M = fmaxf(M, sm.wm[ww][hq]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) {
            const float e = expf(sm.wm[ww][hq] - M);  // 0 for a warp that had no token
            L = fmaf(sm.wl[ww][hq], e, L);
            O = fmaf(sm.wo[ww][hq][d], e, O);
        }
        out((h * kGqa + hq) * kHd + d, O / L);
    }
}

}  // namespace cudallm
