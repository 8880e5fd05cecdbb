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
template <typename KV, bool FUSED, typename Sync>
__device__ __forceinline__ void attend_tile(const float* qkv, int nh, int nkv, const float* cs, KV* k_cache, KV* v_cache,
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
        const float* q = qkv + (h * kGqa + g) * kHd;
        const float x0 = __ldcg(q + i), x1 = __ldcg(q + i + kHd / 2);
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
            const float* k = qkv + (nh + h) * kHd;
            const float x0 = __ldcg(k + tid), x1 = __ldcg(k + tid + kHd / 2);
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
            const KV v = to_kv<KV>(__ldcg(qkv + (nh + nkv + h) * kHd + d));
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
__device__ __forceinline__ void combine_head(const float* part_o, const float* part_ml, int h, int n_tiles, int n_slots,
                                             float* out, int tid) {
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
    __stcg(out + hq * kHd + d, acc / L);
}

// ---- whole-head attention (short contexts) -------------------------------------------------------
// One 256-thread group computes all 4 query heads of KV head h over the whole context: warp w takes
// tiles w, w+8, ... (64 tokens each) straight from the cache (through L2), keeps a running softmax
// (max, sum, p.V) per head, and the 8 warp states are merged in warp order. No partials leave the
// CTA, so there is no second pass. Lane j scores tokens t0+j and t0+j+32; for p.V, lane group
// g = lane/8 takes tokens t0 + 4i + g and lane sub = lane%8 owns dims 8*sub .. 8*sub+7.
template <typename KV>
struct HeadSmem {
    float qs[kGqa][kHd];
    alignas(16) KV kn[kHd];
    alignas(16) KV vn[kHd];
    float ps[8][kGqa][kAttnTile];
    float wm[8][kGqa];
    float wl[8][kGqa];
    float wo[8][kGqa][kHd];
};

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

template <typename KV, typename Sync>
__device__ __forceinline__ void attend_head(const float* qkv, int nh, int nkv, const float* cs, KV* k_cache, KV* v_cache,
                                            int max_seq, int h, int ctx, float* out, HeadSmem<KV>& sm, int tid, Sync sync) {
    const int pos = ctx - 1;
    const int w = tid >> 5, lane = tid & 31;
    // Rotated query heads, and the new token's k (rotated) and v, rounded to the cache type.
    if (tid < kGqa * kHd / 2) {
        const int g = tid >> 5, i = tid & 31;
        const float* q = qkv + (h * kGqa + g) * kHd;
        const float x0 = __ldcg(q + i), x1 = __ldcg(q + i + kHd / 2);
        const float c = cs[i], s = cs[kHd / 2 + i];
        sm.qs[g][i] = x0 * c - x1 * s;
        sm.qs[g][i + kHd / 2] = x1 * c + x0 * s;
    } else if (tid < kGqa * kHd / 2 + kHd / 2) {
        const int i = tid - kGqa * kHd / 2;
        const float* k = qkv + (nh + h) * kHd;
        const float x0 = __ldcg(k + i), x1 = __ldcg(k + i + kHd / 2);
        const float c = cs[i], s = cs[kHd / 2 + i];
        const KV k0 = to_kv<KV>(x0 * c - x1 * s), k1 = to_kv<KV>(x1 * c + x0 * s);
        sm.kn[i] = k0;
        sm.kn[i + kHd / 2] = k1;
        KV* kdst = k_cache + (static_cast<size_t>(h) * max_seq + pos) * kHd;
        kdst[i] = k0;
        kdst[i + kHd / 2] = k1;
    } else if (tid < kGqa * kHd / 2 + kHd / 2 + kHd) {
        const int d = tid - kGqa * kHd / 2 - kHd / 2;
        const KV v = to_kv<KV>(__ldcg(qkv + (nh + nkv + h) * kHd + d));
        sm.vn[d] = v;
        v_cache[(static_cast<size_t>(h) * max_seq + pos) * kHd + d] = v;
    }
    sync();
    const KV* Kh = k_cache + static_cast<size_t>(h) * max_seq * kHd;
    const KV* Vh = v_cache + static_cast<size_t>(h) * max_seq * kHd;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    const int g = lane >> 3, sub = lane & 7;
    float m_run[kGqa], l_run[kGqa], o_run[kGqa][8];
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
        m_run[hq] = -INFINITY;
        l_run[hq] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o_run[hq][e] = 0.f;
    }
    for (int tl = w; tl < n_tiles; tl += 8) {
        const int t0 = tl * kAttnTile;
        // Scores for tokens t0 + lane (half 0) and t0 + lane + 32 (half 1), one key row at a time.
        float sc[2][kGqa];
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            const int j = t0 + lane + 32 * half;
            const uint4* src = (j < ctx && j != pos) ? reinterpret_cast<const uint4*>(Kh + static_cast<size_t>(j) * kHd)
                                                     : reinterpret_cast<const uint4*>(sm.kn);
            uint4 kr[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) kr[c] = (j < ctx && j != pos) ? __ldcg(src + c) : src[c];
            float dot[kGqa] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float kf[8];
                unpack8<KV>(kr[c], kf);
#pragma unroll
                for (int hq = 0; hq < kGqa; ++hq) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) dot[hq] = fmaf(kf[e], sm.qs[hq][8 * c + e], dot[hq]);
                }
            }
#pragma unroll
            for (int hq = 0; hq < kGqa; ++hq) sc[half][hq] = j < ctx ? 0.125f * dot[hq] : -INFINITY;
        }
        // Running softmax: rescale the state to the new maximum, weight this tile's p by it directly.
#pragma unroll
        for (int hq = 0; hq < kGqa; ++hq) {
            const float mn = fmaxf(m_run[hq], warp_max(fmaxf(sc[0][hq], sc[1][hq])));
            const float a = expf(m_run[hq] - mn);
            const float pa = expf(sc[0][hq] - mn), pb = expf(sc[1][hq] - mn);
            sm.ps[w][hq][lane] = pa;
            sm.ps[w][hq][lane + 32] = pb;
            l_run[hq] = l_run[hq] * a + warp_sum(pa + pb);
#pragma unroll
            for (int e = 0; e < 8; ++e) o_run[hq][e] *= a;
            m_run[hq] = mn;
        }
        __syncwarp();
#pragma unroll 1
        for (int batch = 0; batch < 2; ++batch) {
            uint4 vr[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int j = t0 + 4 * (8 * batch + i) + g;
                vr[i] = (j < ctx && j != pos) ? __ldcg(reinterpret_cast<const uint4*>(Vh + static_cast<size_t>(j) * kHd) + sub)
                                              : reinterpret_cast<const uint4*>(sm.vn)[sub];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int jt = 4 * (8 * batch + i) + g;  // token within the tile; p is 0 past the context
                float vf[8];
                unpack8<KV>(vr[i], vf);
#pragma unroll
                for (int hq = 0; hq < kGqa; ++hq) {
                    const float pv = sm.ps[w][hq][jt];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o_run[hq][e] = fmaf(pv, vf[e], o_run[hq][e]);
                }
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int hq = 0; hq < kGqa; ++hq) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float v = o_run[hq][e];
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (g == 0) sm.wo[w][hq][8 * sub + e] = v;
        }
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
            const float e = expf(sm.wm[ww][hq] - M);
            L = fmaf(sm.wl[ww][hq], e, L);
            O = fmaf(sm.wo[ww][hq][d], e, O);
        }
        __stcg(out + (h * kGqa + hq) * kHd + d, O / L);
    }
    sync();
}

}  // namespace cudallm
