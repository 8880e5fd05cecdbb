// Per-row kernels of the batched decode step (batch of independent sequences, one row per sequence):
// embedding gather, RMSNorm into the bf16 GEMM operand, RoPE + KV-cache write, split-K GQA attention
// and argmax. The arithmetic of each row is the single-sequence path's (same RoPE angle, rounding of
// k/v to the cache type, tile partials merged in tile order, lowest index on ties); rows only differ in
// their token, position and KV-cache region.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <climits>

#include "common/check.h"
#include "kernels/attention_core.cuh"
#include "kernels/batch.h"
#include "kernels/batch_ops.h"
#include "kernels/launch.cuh"
#include "kernels/ptx.cuh"

namespace cudallm {
namespace {

// v as the hi / lo bf16 pair of the GEMM activation planes (plane = elements between the two planes).
__device__ __forceinline__ void store_planes(__nv_bfloat16* p, size_t plane, size_t i, float v) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    p[i] = hi;
    p[plane + i] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

struct PlaneDst {
    __nv_bfloat16* p;
    size_t plane;
    __device__ __forceinline__ void operator()(int i, float v) const { store_planes(p, plane, i, v); }
};

// Token of row b: tok_in[b] when >= 0 (fed by the caller), else the previous step's argmax tok[b].
// x[b][j] = embedding row of the token: bf16 weights, or int4 codes re-packed by interleave_int4_codes
// ((u - 8) * fp16 scale of the 128-column group, in fp32); planes of x[b][j] * gain[j] (the first RMSNorm's
// input) and ssq[b] = sum_j x[b][j]^2 (reduced in a fixed order), one 256-thread block per row.
template <bool INT4>
__global__ void __launch_bounds__(256) embed_rows_kernel(const void* __restrict__ emb, const __half* __restrict__ emb_s,
                                                         const int* __restrict__ tok_in, const int* tok,
                                                         const float* __restrict__ gain, float* __restrict__ x,
                                                         __nv_bfloat16* __restrict__ planes, float* __restrict__ ssq,
                                                         int hidden) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ float red[8];
    const int b = blockIdx.x;
    const int t = tok_in[b] >= 0 ? tok_in[b] : tok[b];
    float ss = 0.f;
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) {
        float v;
        if constexpr (INT4) {
            const uint32_t* row = static_cast<const uint32_t*>(emb) + static_cast<size_t>(t) * (hidden / 8);
            const int c = j & 7;
            const uint32_t code = (row[j >> 3] >> (8 * (c & 3) + 4 * (c >> 2))) & 0xFu;
            v = static_cast<float>(static_cast<int>(code) - 8) * __half2float(emb_s[static_cast<size_t>(t) * (hidden / 128) + j / 128]);
        } else {
            const uint16_t* row = static_cast<const uint16_t*>(emb) + static_cast<size_t>(t) * hidden;
            v = __uint_as_float(static_cast<uint32_t>(row[j]) << 16);
        }
        x[static_cast<size_t>(b) * hidden + j] = v;
        ss = fmaf(v, v, ss);
        store_planes(planes, static_cast<size_t>(kBatchMax) * hidden, static_cast<size_t>(b) * hidden + j, v * gain[j]);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s2 = 0.f;
        for (int i = 0; i < 8; ++i) s2 += red[i];
        ssq[b] = s2;
    }
}

// out planes [2][kBatchMax][n] of x[b][j] * rsqrt(mean(x[b]^2) + eps) * w[j], one 256-thread block per
// row; the sum of squares is reduced in a fixed order.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                                           __nv_bfloat16* __restrict__ out, int n) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ float red[8];
    const int b = blockIdx.x;
    const float* xr = x + static_cast<size_t>(b) * n;
    float ss = 0.f;
    for (int j = threadIdx.x; j < n; j += 256) ss = fmaf(xr[j], xr[j], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float inv = rsqrtf(t / static_cast<float>(n) + eps);
    for (int j = threadIdx.x; j < n; j += 256) {
        store_planes(out, static_cast<size_t>(kBatchMax) * n, static_cast<size_t>(b) * n + j, xr[j] * inv * w[j]);
    }
}

// grid (nh + 2 nkv, batch), block hd/2: rotates q head h of row b in place, writes the rotated k head or
// the v head of row b into that sequence's cache at its position.
template <typename KV>
__global__ void rope_kv_rows_kernel(float* __restrict__ qkv, const float* __restrict__ inv_freq, KV* __restrict__ k_cache,
                                    KV* __restrict__ v_cache, size_t seq_stride, const int* __restrict__ pos_v, int nh,
                                    int nkv, int hd, int max_seq) {
    grid_dep_launch();
    grid_dep_wait();
    const int head = blockIdx.x, b = blockIdx.y, i = threadIdx.x, half = hd / 2;
    const int pos = pos_v[b];
    float* q = qkv + static_cast<size_t>(b) * (nh + 2 * nkv) * hd;
    KV* kc = k_cache + seq_stride * b;
    KV* vc = v_cache + seq_stride * b;
    if (head < nh + nkv) {
        float* v = q + static_cast<size_t>(head) * hd;
        const float ang = static_cast<float>(pos) * inv_freq[i];
        float s, c;
        sincosf(ang, &s, &c);
        const float r0 = v[i] * c - v[i + half] * s, r1 = v[i + half] * c + v[i] * s;
        if (head < nh) {
            v[i] = r0;
            v[i + half] = r1;
        } else {
            KV* dst = kc + (static_cast<size_t>(head - nh) * max_seq + pos) * hd;
            dst[i] = to_kv<KV>(r0);
            dst[i + half] = to_kv<KV>(r1);
        }
    } else {
        const int h = head - nh - nkv;
        const float* src = q + static_cast<size_t>(nh + nkv + h) * hd;
        KV* dst = vc + (static_cast<size_t>(h) * max_seq + pos) * hd;
        dst[2 * i] = to_kv<KV>(src[2 * i]);
        dst[2 * i + 1] = to_kv<KV>(src[2 * i + 1]);
    }
}

// grid (nkv, max tiles, batch): partial of 64-token tile t of KV head h for row b.
template <typename KV>
__global__ void __launch_bounds__(kAttThreads) attention_rows_partial_kernel(const float* __restrict__ qkv, const KV* k_cache,
                                                                             const KV* v_cache, size_t seq_stride,
                                                                             const int* __restrict__ pos_v, float* part_o,
                                                                             float* part_ml, int nh, int nkv, int max_seq) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ AttSmem<KV> sm;
    const int b = blockIdx.z, tile = blockIdx.y, ctx = pos_v[b] + 1;
    if (tile * kAttnTile >= ctx) return;
    const int n_slots = max_seq / kAttnTile;
    const float* q = qkv + static_cast<size_t>(b) * (nh + 2 * nkv) * kHd;
    float* po = part_o + static_cast<size_t>(b) * nh * n_slots * kHd;
    float* pml = part_ml + static_cast<size_t>(b) * nh * n_slots * 2;
    attend_tile<KV, false>(PlainSrc{q}, nh, 0, nullptr, const_cast<KV*>(k_cache + seq_stride * b),
                           const_cast<KV*>(v_cache + seq_stride * b), max_seq, blockIdx.x, tile, ctx, n_slots, po, pml, sm,
                           threadIdx.x, [] { __syncthreads(); });
}

// ---- streaming attention: one CTA per (KV head, row) -------------------------------------------------
// The CTA walks row b's whole context in 64-token tiles. Thread 0 brings each tile's K and V rows (8 KiB
// each, contiguous in the cache) into a kRowAttStages-deep shared-memory ring with bulk async copies that
// complete on an mbarrier, so later tiles stream in while the current one is used. The 4 query heads of
// the KV head share every K and V element a thread loads:
//   scores: in 4 passes of 16 tokens, thread (token j, dims 8c..8c+7) forms partial dots for all 4 heads
//           with q held in registers; a 3-step butterfly over the 8 lanes of the token (4 shuffles)
//           leaves each head's full dot in one lane pair;
//   softmax: warp h advances head h's running (max, sum) over the tile;
//   p.V:     thread (token group jg, dims 8c..8c+7) accumulates, for all 4 heads, tokens jg + 16i, after
//            rescaling its accumulators by the heads' correction factors;
// and the 16 token groups are summed once at the end. The result leaves as activation planes; there are
// no partials and no second kernel.
constexpr int kRowAttStages = 3;
constexpr int kRowAttThreads = 128;

template <typename KV>
struct alignas(16) RowAttSmem {
    KV k[kRowAttStages][kAttnTile][kHd];
    KV v[kRowAttStages][kAttnTile][kHd];
    float s[kAttnTile][kGqa];  // scores, then probabilities, of token j for the 4 heads
    float alpha[kGqa];         // per head: exp(previous max - new max)
    float l[kGqa];             // per head: final softmax sum
    uint64_t full[kRowAttStages];
    int ok;
};
static_assert(sizeof(float) * 16 * kGqa * kHd <= sizeof(__half) * kRowAttStages * kAttnTile * kHd,
              "the end-of-kernel reduction reuses the K ring");

template <typename KV>
__global__ void __launch_bounds__(kRowAttThreads) attention_rows_stream_kernel(const float* __restrict__ qkv, const KV* k_cache,
                                                                               const KV* v_cache, size_t seq_stride,
                                                                               const int* __restrict__ pos_v,
                                                                               __nv_bfloat16* out, int nh, int nkv,
                                                                               int max_seq, unsigned* err, int one_seq) {
    using KV2 = typename Kv2<KV>::T;
    grid_dep_launch();
    // A direct cast keeps the shared address space visible to the compiler (shared loads, not generic);
    // dynamic shared memory is 16-byte aligned, which is all the bulk copies need.
    extern __shared__ __align__(16) uint8_t att_raw[];
    RowAttSmem<KV>& sm = *reinterpret_cast<RowAttSmem<KV>*>(att_raw);
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c8 = tid & 7;  // dims 8*c8 .. 8*c8+7
    if (tid == 0) {
        for (int st = 0; st < kRowAttStages; ++st) mbar_init(&sm.full[st], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // pos and the cached tokens before pos were written by earlier steps, so tiles that end before pos
    // are fetched before waiting for the kernel that produces q and the new token's k / v. When every row
    // is one position of a single sequence (one_seq: a prefill chunk, row 0 at its first position), this
    // step writes all positions from row 0's on, so only tiles ending before that one are fetched early.
    const int ctx = pos_v[b] + 1;
    const int fresh = one_seq ? pos_v[0] : ctx - 1;
    const int n_tiles = (ctx + kAttnTile - 1) / kAttnTile;
    const KV* kg = k_cache + seq_stride * b + static_cast<size_t>(h) * max_seq * kHd;
    const KV* vg = v_cache + seq_stride * b + static_cast<size_t>(h) * max_seq * kHd;
    const uint64_t pol = l2_policy_evict_first();
    auto issue = [&](int t) {
        const int st = t % kRowAttStages;
        const uint32_t bytes = static_cast<uint32_t>(min(kAttnTile, ctx - t * kAttnTile) * kHd * sizeof(KV));
        mbar_arrive_expect_tx(&sm.full[st], 2 * bytes);
        bulk_load(&sm.k[st][0][0], kg + static_cast<size_t>(t) * kAttnTile * kHd, bytes, &sm.full[st], pol);
        bulk_load(&sm.v[st][0][0], vg + static_cast<size_t>(t) * kAttnTile * kHd, bytes, &sm.full[st], pol);
    };
    const int first = min(kRowAttStages, n_tiles);
    const int early = min(first, fresh / kAttnTile);  // tiles wholly before the first position written now
    if (tid == 0) {
        for (int t = 0; t < early; ++t) issue(t);
    }
    grid_dep_wait();  // q, the new k / v come from the kernel before
    if (tid == 0) {
        for (int t = early; t < first; ++t) issue(t);
    }
    // q of the 4 heads, dims 8*c8 .. 8*c8+7, pre-scaled pairs.
    float2 q[kGqa][4];
    {
        const float* qb = qkv + static_cast<size_t>(b) * (nh + 2 * nkv) * kHd + static_cast<size_t>(h) * kGqa * kHd + 8 * c8;
#pragma unroll
        for (int g = 0; g < kGqa; ++g) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(qb + g * kHd));
            const float4 c = __ldcg(reinterpret_cast<const float4*>(qb + g * kHd + 4));
            q[g][0] = make_float2(a.x, a.y);
            q[g][1] = make_float2(a.z, a.w);
            q[g][2] = make_float2(c.x, c.y);
            q[g][3] = make_float2(c.z, c.w);
        }
    }
    float2 acc[kGqa][4];
#pragma unroll
    for (int g = 0; g < kGqa; ++g) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = make_float2(0.f, 0.f);
    }
    float m_run = -INFINITY, l_run = 0.f;  // head `warp`'s running softmax (warps 0..3)
    const bool hi4 = (lane & 4) != 0, hi2 = (lane & 2) != 0;
    const int my_head = (hi4 ? 2 : 0) + (hi2 ? 1 : 0);
    int t = 0;
    for (; t < n_tiles; ++t) {
        const int st = t % kRowAttStages;
        if (tid == 0) {
            // Bounded wait for the tile (1 s); on a time-out every thread leaves the loop together.
            uint64_t t0 = 0;
            int ok = 1;
            for (uint32_t it = 1; !mbar_try_wait(&sm.full[st], (t / kRowAttStages) & 1); ++it) {
                if ((it & 63) == 0) {
                    const uint64_t now = global_ns();
                    if (t0 == 0) {
                        t0 = now;
                    } else if (now - t0 > 1000000000ull) {
                        atomicOr(err, 2u);
                        ok = 0;
                        break;
                    }
                }
            }
            sm.ok = ok;
        }
        __syncthreads();
        if (!sm.ok) break;
        const int n = min(kAttnTile, ctx - t * kAttnTile);
        // Scores.
#pragma unroll
        for (int ps = 0; ps < 4; ++ps) {
            const int j = ps * 16 + (tid >> 3);
            float sc[kGqa] = {0.f, 0.f, 0.f, 0.f};
            if (j < n) {
                const uint4 u = *reinterpret_cast<const uint4*>(&sm.k[st][j][8 * c8]);
                const KV2* k2 = reinterpret_cast<const KV2*>(&u);
#pragma unroll
                for (int g = 0; g < kGqa; ++g) {
                    float2 a = make_float2(0.f, 0.f);
#pragma unroll
                    for (int e = 0; e < 4; ++e) a = fma2(kv2_to_float2(k2[e]), q[g][e], a);
                    sc[g] = a.x + a.y;
                }
            }
            // Butterfly over the token's 8 lanes: heads {0,1} / {2,3} by lane bit 2, then one head by bit
            // 1, then the full sum by bit 0.
            const float r0 = __shfl_xor_sync(0xffffffffu, hi4 ? sc[0] : sc[2], 4);
            const float r1 = __shfl_xor_sync(0xffffffffu, hi4 ? sc[1] : sc[3], 4);
            const float a0 = (hi4 ? sc[2] : sc[0]) + r0;
            const float a1 = (hi4 ? sc[3] : sc[1]) + r1;
            const float r2 = __shfl_xor_sync(0xffffffffu, hi2 ? a0 : a1, 2);
            float c = (hi2 ? a1 : a0) + r2;
            c += __shfl_xor_sync(0xffffffffu, c, 1);
            if ((lane & 1) == 0) sm.s[j][my_head] = j < n ? 0.125f * c : -INFINITY;
        }
        __syncthreads();
        // Softmax: warp g = head g, tokens lane and lane + 32.
        if (warp < kGqa) {
            const float s0 = sm.s[lane][warp], s1 = sm.s[lane + 32][warp];
            const float m_new = fmaxf(m_run, warp_max(fmaxf(s0, s1)));
            const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
            sm.s[lane][warp] = p0;
            sm.s[lane + 32][warp] = p1;
            const float alpha = expf(m_run - m_new);
            l_run = l_run * alpha + warp_sum(p0 + p1);
            m_run = m_new;
            if (lane == 0) sm.alpha[warp] = alpha;
        }
        __syncthreads();
        // p.V for tokens jg + 16 i.
        {
            const float4 al = *reinterpret_cast<const float4*>(sm.alpha);
            const float alv[kGqa] = {al.x, al.y, al.z, al.w};
#pragma unroll
            for (int g = 0; g < kGqa; ++g) {
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[g][e] = make_float2(acc[g][e].x * alv[g], acc[g][e].y * alv[g]);
            }
            const int jg = tid >> 3;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = jg + 16 * i;
                if (j < n) {
                    const uint4 u = *reinterpret_cast<const uint4*>(&sm.v[st][j][8 * c8]);
                    const KV2* v2 = reinterpret_cast<const KV2*>(&u);
                    const float4 p4 = *reinterpret_cast<const float4*>(&sm.s[j][0]);
                    const float pv[kGqa] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 vf = kv2_to_float2(v2[e]);
#pragma unroll
                        for (int g = 0; g < kGqa; ++g) acc[g][e] = fma2(make_float2(pv[g], pv[g]), vf, acc[g][e]);
                    }
                }
            }
        }
        __syncthreads();  // stage st and the score buffer are free again
        if (tid == 0 && t + kRowAttStages < n_tiles) issue(t + kRowAttStages);
    }
    if (t < n_tiles) {
        // Gave up on a tile: wait (bounded) for the copies still in flight before the CTA exits.
        if (tid == 0) {
            for (int u = t; u < min(n_tiles, t + kRowAttStages); ++u) {
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait(&sm.full[u % kRowAttStages], (u / kRowAttStages) & 1) &&
                       global_ns() - t0 < 1000000000ull) {
                }
            }
        }
        return;
    }
    // Sum the 16 token groups: red[jg][g][d] in the (now idle) K ring.
    float* red = reinterpret_cast<float*>(&sm.k[0][0][0]);
    {
        const int jg = tid >> 3;
#pragma unroll
        for (int g = 0; g < kGqa; ++g) {
            float4* dst = reinterpret_cast<float4*>(red + (jg * kGqa + g) * kHd + 8 * c8);
            dst[0] = make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
            dst[1] = make_float4(acc[g][2].x, acc[g][2].y, acc[g][3].x, acc[g][3].y);
        }
    }
    if (warp < kGqa && lane == 0) sm.l[warp] = l_run;
    __syncthreads();
    {
        const int g = tid >> 5, d = 2 * lane;
        float2 o = make_float2(0.f, 0.f);
#pragma unroll
        for (int jg = 0; jg < 16; ++jg) {
            const float2 r = *reinterpret_cast<const float2*>(red + (jg * kGqa + g) * kHd + d);
            o = add2(o, r);
        }
        const float inv_l = 1.f / sm.l[g];
        const size_t plane = static_cast<size_t>(kBatchMax) * nh * kHd;
        const size_t base = static_cast<size_t>(b) * nh * kHd + static_cast<size_t>(h * kGqa + g) * kHd + d;
        store_planes(out, plane, base, o.x * inv_l);
        store_planes(out, plane, base + 1, o.y * inv_l);
    }
}

// grid (nkv, batch): merges row b's tile partials of KV head h into the attention output planes
// [2][kBatchMax][nh * 64].
__global__ void __launch_bounds__(kAttThreads) attention_rows_combine_kernel(const float* part_o, const float* part_ml,
                                                                             const int* __restrict__ pos_v,
                                                                             __nv_bfloat16* out, int nh, int max_seq) {
    grid_dep_launch();
    grid_dep_wait();
    const int b = blockIdx.y, ctx = pos_v[b] + 1, n_slots = max_seq / kAttnTile;
    combine_head(part_o + static_cast<size_t>(b) * nh * n_slots * kHd, part_ml + static_cast<size_t>(b) * nh * n_slots * 2,
                 blockIdx.x, (ctx + kAttnTile - 1) / kAttnTile, n_slots, PlaneDst{out + static_cast<size_t>(b) * nh * kHd, static_cast<size_t>(kBatchMax) * nh * kHd},
                 threadIdx.x);
}

// grid (kArgmaxSplit, batch), block 1024: block p of row b finds the largest logit of slice p of the row
// (lowest index on ties; all-NaN slice -> index INT_MAX) into pv/pi[b][p]; the last block of the row to
// finish (a ticket per row) merges the slices in slice order, writes tok[b] (0 for an all-NaN row),
// advances pos[b] and re-arms the ticket.
__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, int n, float* pv, int* pi,
                                                           unsigned* ticket, int* tok, int* pos_v) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ bool last;
    const int b = blockIdx.y, p = blockIdx.x;
    const int per = (n + kArgmaxSplit - 1) / kArgmaxSplit;
    const int j0 = p * per, j1 = min(n, j0 + per);
    const float* row = logits + static_cast<size_t>(b) * n;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int j = j0 + threadIdx.x; j < j1; j += 1024) better(bv, bi, row[j], j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = sv[0];
        int i = si[0];
        for (int w = 1; w < 32; ++w) better(v, i, sv[w], si[w]);
        pv[b * kArgmaxSplit + p] = v;
        pi[b * kArgmaxSplit + p] = i;
        __threadfence();
        last = atomicAdd(&ticket[b], 1u) == kArgmaxSplit - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float v = __ldcg(pv + b * kArgmaxSplit);
        int i = __ldcg(pi + b * kArgmaxSplit);
        for (int q = 1; q < kArgmaxSplit; ++q) better(v, i, __ldcg(pv + b * kArgmaxSplit + q), __ldcg(pi + b * kArgmaxSplit + q));
        tok[b] = i == INT_MAX ? 0 : i;
        pos_v[b] += 1;
        ticket[b] = 0;
    }
}

// grid batch, block 256: tok[b] = the best of row b's per-tile (value, index) partials (lowest index on
// ties; all-NaN row -> 0), pos[b] += 1.
__global__ void __launch_bounds__(256) argmax_tiles_kernel(const float* __restrict__ am_v, const int* __restrict__ am_i,
                                                           int n_tiles, int* tok, int* pos_v) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ float sv[8];
    __shared__ int si[8];
    const int b = blockIdx.x;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int t = threadIdx.x; t < n_tiles; t += 256) {
        better(bv, bi, am_v[static_cast<size_t>(b) * n_tiles + t], am_i[static_cast<size_t>(b) * n_tiles + t]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = sv[0];
        int i = si[0];
        for (int w = 1; w < 8; ++w) better(v, i, sv[w], si[w]);
        tok[b] = i == INT_MAX ? 0 : i;
        pos_v[b] += 1;
    }
}

}  // namespace

void launch_argmax_tiles(const float* am_v, const int* am_i, int n_tiles, int* tok, int* pos, int batch, cudaStream_t stream,
                         bool pdl) {
    CLLM_CHECK(am_v && am_i && tok && pos && batch >= 1 && n_tiles >= 1, "launch_argmax_tiles: bad arguments");
    launch_kernel(argmax_tiles_kernel, dim3(batch), dim3(256), 0, stream, pdl, am_v, am_i, n_tiles, tok, pos);
}

void launch_embed_rows(const void* emb, const __half* emb_scales, const int* tok_in, const int* tok, const float* gain,
                       float* x, __nv_bfloat16* planes, float* ssq, int batch, int hidden, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(emb && tok_in && tok && gain && x && planes && ssq && batch >= 1 && batch <= kBatchMax && hidden % 128 == 0,
               "launch_embed_rows: bad arguments");
    if (emb_scales) {
        launch_kernel(embed_rows_kernel<true>, dim3(batch), dim3(256), 0, stream, pdl, emb, emb_scales, tok_in, tok, gain, x,
                      planes, ssq, hidden);
    } else {
        launch_kernel(embed_rows_kernel<false>, dim3(batch), dim3(256), 0, stream, pdl, emb, emb_scales, tok_in, tok, gain, x,
                      planes, ssq, hidden);
    }
}

void launch_rmsnorm_rows(const float* x, const float* w, float eps, __nv_bfloat16* out, int batch, int n, cudaStream_t stream,
                         bool pdl) {
    CLLM_CHECK(x && w && out && batch >= 1 && batch <= kBatchMax && n >= 1, "launch_rmsnorm_rows: bad arguments");
    launch_kernel(rmsnorm_rows_kernel, dim3(batch), dim3(256), 0, stream, pdl, x, w, eps, out, n);
}

template <typename KV>
void launch_rope_kv_rows(float* qkv, const float* inv_freq, KV* k_cache, KV* v_cache, size_t seq_stride, const int* pos,
                         int batch, int nh, int nkv, int hd, int max_seq, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(qkv && inv_freq && k_cache && v_cache && pos && batch >= 1, "launch_rope_kv_rows: bad arguments");
    launch_kernel(rope_kv_rows_kernel<KV>, dim3(nh + 2 * nkv, batch), dim3(hd / 2), 0, stream, pdl, qkv, inv_freq, k_cache,
                  v_cache, seq_stride, pos, nh, nkv, hd, max_seq);
}

template <typename KV>
void launch_attention_rows(const float* qkv, const KV* k_cache, const KV* v_cache, size_t seq_stride, const int* pos,
                           int max_ctx, float* part_o, float* part_ml, __nv_bfloat16* out, int batch, int nh, int nkv,
                           int max_seq, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(qkv && k_cache && v_cache && pos && part_o && part_ml && out && batch >= 1 && batch <= kBatchMax,
               "launch_attention_rows: bad arguments");
    CLLM_CHECK(nh == nkv * kGqa && max_seq % kAttnTile == 0 && max_ctx >= 1 && max_ctx <= max_seq,
               "launch_attention_rows: unsupported shape");
    const int tiles = (max_ctx + kAttnTile - 1) / kAttnTile;
    launch_kernel(attention_rows_partial_kernel<KV>, dim3(nkv, tiles, batch), dim3(kAttThreads), 0, stream, pdl, qkv, k_cache,
                  v_cache, seq_stride, pos, part_o, part_ml, nh, nkv, max_seq);
    launch_kernel(attention_rows_combine_kernel, dim3(nkv, batch), dim3(kAttThreads), 0, stream, pdl,
                  static_cast<const float*>(part_o), static_cast<const float*>(part_ml), pos, out, nh, max_seq);
}

template <typename KV>
void launch_attention_rows_stream(const float* qkv, const KV* k_cache, const KV* v_cache, size_t seq_stride, const int* pos,
                                  __nv_bfloat16* out, int batch, int nh, int nkv, int max_seq, unsigned* err,
                                  cudaStream_t stream, bool pdl, bool one_seq) {
    CLLM_CHECK(qkv && k_cache && v_cache && pos && out && err && batch >= 1 && batch <= kBatchMax,
               "launch_attention_rows_stream: bad arguments");
    CLLM_CHECK(nh == nkv * kGqa && max_seq % kAttnTile == 0, "launch_attention_rows_stream: unsupported shape");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(k_cache) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_cache) & 15) == 0 &&
                   (seq_stride * sizeof(KV)) % 16 == 0,
               "launch_attention_rows_stream: caches must be 16-byte aligned");
    constexpr int smem = static_cast<int>(sizeof(RowAttSmem<KV>));
    static bool configured[64] = {};
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || !configured[dev]) {
        CLLM_CUDA(cudaFuncSetAttribute(attention_rows_stream_kernel<KV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        if (dev < 64) configured[dev] = true;
    }
    launch_kernel(attention_rows_stream_kernel<KV>, dim3(nkv, batch), dim3(kRowAttThreads), smem, stream, pdl, qkv, k_cache,
                  v_cache, seq_stride, pos, out, nh, nkv, max_seq, err, one_seq ? 1 : 0);
}

void launch_argmax_rows(const float* logits, int n, float* scratch_v, int* scratch_i, unsigned* ticket, int* tok, int* pos,
                        int batch, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(logits && scratch_v && scratch_i && ticket && tok && pos && batch >= 1 && n >= kArgmaxSplit,
               "launch_argmax_rows: bad arguments");
    launch_kernel(argmax_rows_kernel, dim3(kArgmaxSplit, batch), dim3(1024), 0, stream, pdl, logits, n, scratch_v, scratch_i,
                  ticket, tok, pos);
}

template void launch_rope_kv_rows<__nv_bfloat16>(float*, const float*, __nv_bfloat16*, __nv_bfloat16*, size_t, const int*, int,
                                                 int, int, int, int, cudaStream_t, bool);
template void launch_rope_kv_rows<__half>(float*, const float*, __half*, __half*, size_t, const int*, int, int, int, int, int,
                                          cudaStream_t, bool);
template void launch_attention_rows_stream<__nv_bfloat16>(const float*, const __nv_bfloat16*, const __nv_bfloat16*, size_t,
                                                          const int*, __nv_bfloat16*, int, int, int, int, unsigned*,
                                                          cudaStream_t, bool, bool);
template void launch_attention_rows_stream<__half>(const float*, const __half*, const __half*, size_t, const int*,
                                                   __nv_bfloat16*, int, int, int, int, unsigned*, cudaStream_t, bool, bool);
template void launch_attention_rows<__nv_bfloat16>(const float*, const __nv_bfloat16*, const __nv_bfloat16*, size_t, const int*,
                                                   int, float*, float*, __nv_bfloat16*, int, int, int, int, cudaStream_t, bool);
template void launch_attention_rows<__half>(const float*, const __half*, const __half*, size_t, const int*, int, float*, float*,
                                            __nv_bfloat16*, int, int, int, int, cudaStream_t, bool);

}  // namespace cudallm
