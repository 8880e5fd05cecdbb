// Batched decode GEMM on the sm_100a tensor cores with fused epilogues. s[b][j] = sum_k X[b][k] * W[j][k]:
// W the [N][K] bf16 weight matrix (row-major, as stored in the .cudallm file), X the fp32 activations of
// up to 64 sequences carried as two bf16 planes, X = hi + lo (hi = bf16(X), lo = bf16(X - hi)), so the
// product keeps ~16 mantissa bits of the fp32 activation, like the batch-1 path's fp32 vectors.
//
// Mainloop: weight rows are the MMA's M side; a CTA computes 128 weight rows x 64 batch columns
// (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 64, K = 16 per instruction; one MMA per plane into
// the same accumulator) in a 64-column fp32 TMEM accumulator, so every weight element is read from HBM
// once per step and used for the whole batch. Operands arrive by 2D TMA tensor loads (128-byte swizzle,
// no multicast) through a 7-stage ring of (W 128 x 64, X 2 x 64 x 64) tiles; one thread issues the loads,
// one thread the MMAs. The CTAs of one 128-row tile split K (grid rows = cluster ranks) and start at
// different chunks of their range, so they do not all read the same activation tile at once.
//
// Epilogue: the accumulator goes from TMEM to shared memory; the tile's cluster adds the K-split partial
// sums through distributed shared memory (rank r reduces slice r of the tile, peers added in rank order,
// so results do not depend on timing) and applies the fused epilogue (GemmEpi): residual add with the
// next RMSNorm's statistics and activation planes, SwiGLU into activation planes, RoPE with the KV-cache
// write, or logits with per-tile argmax partials. Programmatic dependent launch: a GEMM starts streaming
// its weights while the kernel before it finishes and waits for it only before loading activations.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "common/check.h"
#include "kernels/batch.h"
#include "kernels/tcgen05.cuh"

namespace cudallm {
namespace {

constexpr int kGM = kGemmTileRows;  // weight rows per CTA (MMA M)
constexpr int kGN = kBatchMax;      // batch columns (MMA N)
constexpr int kGK = 64;             // K per stage: one 128-byte swizzled row
constexpr int kXRows = 2 * kGN;     // hi plane rows 0..63, lo plane rows 64..127
constexpr int kGStages = 7;        // deep ring: one CTA per SM
constexpr int kGStagesLogits = 3;  // shallow ring: two CTAs per SM, one's epilogue overlaps the other's stream
constexpr int kGThreads = 128;
constexpr int kMaxKsplit = 16;
constexpr int kWTileBytes = kGM * kGK * 2;     // 16 KiB
constexpr int kXTileBytes = kXRows * kGK * 2;  // 16 KiB
constexpr int kXPlaneBytes = kGN * kGK * 2;    // lo plane offset inside an X tile (1024-byte aligned)
constexpr int kCtrlBytes = 1024;  // barriers, TMEM slot, inv_rms[64], pos[64], inv_freq[32]
constexpr int ring_bytes(int stages) { return stages * (kWTileBytes + kXTileBytes); }
constexpr int smem_bytes(int stages) { return 1024 + ring_bytes(stages) + kCtrlBytes; }
constexpr uint64_t kGemmWaitNs = 1000000000ull;
static_assert(smem_bytes(kGStages) <= 232448, "GEMM shared memory above the per-block limit");
static_assert(2 * smem_bytes(kGStagesLogits) <= 228 * 1024 - 2 * 1024, "two lm_head CTAs must fit an SM");
static_assert(ring_bytes(kGStagesLogits) >= 2 * kGN * kGM * 4, "the epilogue scratch lives in the ring");

struct GemmArgs {
    int n, batch, chunks, ksplit, n_tiles;  // chunks: 64-column K chunks in total
    unsigned* err;                          // error word (set on a wait timeout)
    GemmEpi epi;
};

// Bounded wait on an mbarrier phase; false (and the error word set) after kGemmWaitNs.
__device__ bool gemm_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            const uint64_t t = global_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > kGemmWaitNs) {
                atomicOr(err, 1u);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void store_planes_g(__nv_bfloat16* p, size_t plane, size_t i, float v) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    p[i] = hi;
    p[plane + i] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

__device__ __forceinline__ float silu_g(float x) { return x / (1.f + __expf(-x)); }

template <typename KV>
__device__ __forceinline__ KV to_cache(float v);
template <>
__device__ __forceinline__ __half to_cache<__half>(float v) {
    return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 to_cache<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// The tile's accumulator in shared memory, column-major ([batch column][128 rows] fp32), summed over
// the cluster's K-split ranks in rank order. sum4 returns rows row..row+3 of one column: the loads from
// every rank are issued before any is added, so the distributed-shared-memory latency is paid once.
struct TileSum {
    const float* own;
    uint32_t own_saddr;
    uint32_t ks;
    __device__ __forceinline__ float4 sum4(int col, int row) const {
        const int idx = col * kGM + row;
        if (ks == 1) return *reinterpret_cast<const float4*>(own + idx);
        float4 part[kMaxKsplit];
#pragma unroll
        for (uint32_t r = 0; r < kMaxKsplit; ++r) {
            if (r < ks) part[r] = ld_peer_f32x4(peer_smem(own_saddr + 4u * idx, r));
        }
        float4 s = part[0];
#pragma unroll
        for (uint32_t r = 1; r < kMaxKsplit; ++r) {
            if (r < ks) {
                s.x += part[r].x;
                s.y += part[r].y;
                s.z += part[r].z;
                s.w += part[r].w;
            }
        }
        return s;
    }
};

__device__ __forceinline__ float f4get(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

__device__ __forceinline__ void argmax_better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// The fused epilogue of one tile (GemmEpi), run by all NT threads of the CTA once T holds this CTA's
// partial tile ([batch column][128 rows] fp32) and the cluster has synchronised. Every thread reaches
// every block and cluster barrier inside.
template <int EPI, typename KV, int NT>
__device__ __forceinline__ void fused_epilogue(const GemmArgs& a, float* T, const float* inv_rms, const int* pos_s,
                                               const float* freq_s, int tile, uint32_t ks, uint32_t rank, int tid) {
    const GemmEpi& e = a.epi;
    const int n0 = tile * kGM;
    const TileSum tsum{T, smem_addr(T), ks};
    auto sum = [&](int col, int row) { return tsum.sum4(col, row); };
    const int batch = a.batch;
    if constexpr (EPI == static_cast<int>(GemmEpilogue::STORE) || EPI == static_cast<int>(GemmEpilogue::LOGITS) ||
                  EPI == static_cast<int>(GemmEpilogue::ADD)) {
        // Slice `rank` of the tile's rows, in groups of 4 rows; items (row group, batch column) with
        // consecutive threads on consecutive row groups. Full groups use 16-byte accesses.
        const int g0 = static_cast<int>(rank) * (kGM / 4) / static_cast<int>(ks);
        const int len = (static_cast<int>(rank) + 1) * (kGM / 4) / static_cast<int>(ks) - g0;
        float* sq = T + kGN * kGM;  // ADD: squares per (batch column, row group) after T in the idle ring
        const size_t plane = static_cast<size_t>(kBatchMax) * a.n;
        for (int it = tid; it < kGN * len; it += NT) {
            const int el = it % len, b = it / len;
            const int row = 4 * (g0 + el), j = n0 + row;
            const size_t at = static_cast<size_t>(b) * a.n + j;
            const bool full4 = j + 3 < a.n && (at & 3) == 0;
            float sq4 = 0.f;
            if (b < batch && j < a.n) {
                float4 y4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (EPI == static_cast<int>(GemmEpilogue::ADD)) {
                    // The residual is fetched before the partial sums, so both latencies overlap.
                    if (full4) {
                        y4 = *reinterpret_cast<const float4*>(e.y + at);
                    } else {
                        y4.x = e.y[at];
                        if (j + 1 < a.n) y4.y = e.y[at + 1];
                        if (j + 2 < a.n) y4.z = e.y[at + 2];
                    }
                }
                const float4 s4 = sum(b, row);
                const float sc = inv_rms[b];
                float4 v4 = make_float4(s4.x * sc + y4.x, s4.y * sc + y4.y, s4.z * sc + y4.z, s4.w * sc + y4.w);
                if (full4) {
                    *reinterpret_cast<float4*>(e.y + at) = v4;
                } else {
                    for (int q = 0; q < 4 && j + q < a.n; ++q) e.y[at + q] = f4get(v4, q);
                }
                if constexpr (EPI == static_cast<int>(GemmEpilogue::ADD)) {
                    sq4 = v4.x * v4.x + v4.y * v4.y + v4.z * v4.z + v4.w * v4.w;
                    if (e.planes && !full4) {
                        for (int q = 0; q < 4 && j + q < a.n; ++q) {
                            store_planes_g(e.planes, plane, at + q, f4get(v4, q) * e.gain[j + q]);
                        }
                    } else if (e.planes) {
                        const float4 g4 = *reinterpret_cast<const float4*>(e.gain + j);
                        const float w0 = v4.x * g4.x, w1 = v4.y * g4.y, w2 = v4.z * g4.z, w3 = v4.w * g4.w;
                        const __nv_bfloat162 h01 = __floats2bfloat162_rn(w0, w1), h23 = __floats2bfloat162_rn(w2, w3);
                        const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                        const __nv_bfloat162 l01 = __floats2bfloat162_rn(w0 - f01.x, w1 - f01.y);
                        const __nv_bfloat162 l23 = __floats2bfloat162_rn(w2 - f23.x, w3 - f23.y);
                        uint2 hv, lv;
                        hv.x = *reinterpret_cast<const uint32_t*>(&h01);
                        hv.y = *reinterpret_cast<const uint32_t*>(&h23);
                        lv.x = *reinterpret_cast<const uint32_t*>(&l01);
                        lv.y = *reinterpret_cast<const uint32_t*>(&l23);
                        *reinterpret_cast<uint2*>(e.planes + at) = hv;
                        *reinterpret_cast<uint2*>(e.planes + plane + at) = lv;
                    }
                }
            }
            if constexpr (EPI == static_cast<int>(GemmEpilogue::ADD)) sq[b * len + el] = sq4;
        }
        if constexpr (EPI == static_cast<int>(GemmEpilogue::ADD)) {
            if (e.ssq_out) {
                // Per batch row: this rank's slice sum (in row order), then rank 0 adds the ranks in order,
                // one partial per tile.
                float* sqs = sq + kGN * (kGM / 4);
                __syncthreads();
                if (tid < kGN) {
                    float s = 0.f;
                    for (int el = 0; el < len; ++el) s += sq[tid * len + el];
                    sqs[tid] = s;
                }
                __syncthreads();
                if (ks > 1) cluster_sync();
                if (rank == 0 && tid < kGN) {
                    float s = 0.f;
                    if (ks == 1) {
                        s = sqs[tid];
                    } else {
                        for (uint32_t r = 0; r < ks; ++r) s += ld_peer_f32(peer_smem(smem_addr(sqs + tid), r));
                    }
                    e.ssq_out[static_cast<size_t>(tile) * kBatchMax + tid] = s;
                }
            }
        }
        if constexpr (EPI == static_cast<int>(GemmEpilogue::LOGITS)) {
            // ksplit is 1: the whole tile is local. Threads b and 64 + b: the largest scaled output of rows
            // 0-63 / 64-127 for batch row b; then merged.
            float* mv = T + kGN * kGM;
            int* mi = reinterpret_cast<int*>(mv + 2 * kGN);
            if (tid < 2 * kGN) {
                const int b = tid & 63, half = tid >> 6;
                float bv = -FLT_MAX;
                int bi = INT_MAX;
                const float sc = inv_rms[b];
                for (int row = 64 * half; row < 64 * half + 64 && n0 + row < a.n; ++row) {
                    argmax_better(bv, bi, T[b * kGM + row] * sc, n0 + row);
                }
                mv[tid] = bv;
                mi[tid] = bi;
            }
            __syncthreads();
            if (tid < batch) {
                float bv = mv[tid];
                int bi = mi[tid];
                argmax_better(bv, bi, mv[64 + tid], mi[64 + tid]);
                e.am_v[static_cast<size_t>(tid) * a.n_tiles + tile] = bv;
                e.am_i[static_cast<size_t>(tid) * a.n_tiles + tile] = bi;
            }
        }
    } else if constexpr (EPI == static_cast<int>(GemmEpilogue::SWIGLU)) {
        // Pairs (gate row p, up row 64 + p) of the interleaved layout -> output feature 64 * tile + p, in
        // groups of 4 pairs.
        const int g0 = static_cast<int>(rank) * (kGM / 8) / static_cast<int>(ks);
        const int len = (static_cast<int>(rank) + 1) * (kGM / 8) / static_cast<int>(ks) - g0;
        const int n_out = a.n / 2;
        const size_t plane = static_cast<size_t>(kBatchMax) * n_out;
        for (int it = tid; it < kGN * len; it += NT) {
            const int el = it % len, b = it / len;
            if (b >= batch) continue;
            const int p = 4 * (g0 + el);
            const float4 g4 = sum(b, p), u4 = sum(b, kGM / 2 + p);
            const float sc = inv_rms[b];
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = silu_g(f4get(g4, q) * sc) * (f4get(u4, q) * sc);
            const size_t idx = static_cast<size_t>(b) * n_out + tile * (kGM / 2) + p;
            if (e.y) *reinterpret_cast<float4*>(e.y + idx) = make_float4(v[0], v[1], v[2], v[3]);
            if (e.planes) {
                const __nv_bfloat162 h01 = __floats2bfloat162_rn(v[0], v[1]), h23 = __floats2bfloat162_rn(v[2], v[3]);
                const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                const __nv_bfloat162 l01 = __floats2bfloat162_rn(v[0] - f01.x, v[1] - f01.y);
                const __nv_bfloat162 l23 = __floats2bfloat162_rn(v[2] - f23.x, v[3] - f23.y);
                uint2 hv, lv;
                hv.x = *reinterpret_cast<const uint32_t*>(&h01);
                hv.y = *reinterpret_cast<const uint32_t*>(&h23);
                lv.x = *reinterpret_cast<const uint32_t*>(&l01);
                lv.y = *reinterpret_cast<const uint32_t*>(&l23);
                *reinterpret_cast<uint2*>(e.planes + idx) = hv;
                *reinterpret_cast<uint2*>(e.planes + plane + idx) = lv;
            }
        }
    } else {
        // QKV_ROPE: pairs (dim i, dim i + 32) of the tile's two heads, in groups of 4 pairs.
        const int g0 = static_cast<int>(rank) * (kGM / 8) / static_cast<int>(ks);
        const int len = (static_cast<int>(rank) + 1) * (kGM / 8) / static_cast<int>(ks) - g0;
        const int stride = (e.nh + 2 * e.nkv) * 64;
        for (int it = tid; it < kGN * len; it += NT) {
            const int el = it % len, b = it / len;
            if (b >= batch) continue;
            const int p = 4 * (g0 + el), hh = p >> 5, i0 = p & 31;
            const int ra = hh * 64 + i0, rb = ra + 32;
            const int gh = (n0 + ra) >> 6;  // global head: q < nh <= k < nh + nkv <= v
            const float4 a4 = sum(b, ra), b4 = sum(b, rb);
            const float sc = inv_rms[b];
            const int pos = pos_s[b];
            float y0[4], y1[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float x0 = f4get(a4, q) * sc, x1 = f4get(b4, q) * sc;
                if (gh < e.nh + e.nkv) {
                    float sn, cs;
                    sincosf(static_cast<float>(pos) * freq_s[i0 + q], &sn, &cs);
                    y0[q] = x0 * cs - x1 * sn;
                    y1[q] = x1 * cs + x0 * sn;
                } else {
                    y0[q] = x0;
                    y1[q] = x1;
                }
            }
            if (gh < e.nh) {
                float* qp = e.q_out + static_cast<size_t>(b) * stride + gh * 64 + i0;
                *reinterpret_cast<float4*>(qp) = make_float4(y0[0], y0[1], y0[2], y0[3]);
                *reinterpret_cast<float4*>(qp + 32) = make_float4(y1[0], y1[1], y1[2], y1[3]);
            } else {
                const bool is_k = gh < e.nh + e.nkv;
                KV* c = static_cast<KV*>(is_k ? e.k_cache : e.v_cache) + e.seq_stride * b +
                        (static_cast<size_t>(gh - e.nh - (is_k ? 0 : e.nkv)) * e.max_seq + pos) * 64 + i0;
                union Pack4 {
                    KV h[4];
                    uint2 u;
                } lo4, hi4;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    lo4.h[q] = to_cache<KV>(y0[q]);
                    hi4.h[q] = to_cache<KV>(y1[q]);
                }
                *reinterpret_cast<uint2*>(c) = lo4.u;
                *reinterpret_cast<uint2*>(c + 32) = hi4.u;
            }
        }
    }
}

template <int EPI, typename KV, int ST>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wt = smem;
    uint8_t* xt = smem + ST * kWTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_bytes(ST));
    uint64_t* empty = full + ST;
    uint64_t* done = empty + ST;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* inv_rms = reinterpret_cast<float*>(smem + ring_bytes(ST) + 256);
    int* pos_s = reinterpret_cast<int*>(smem + ring_bytes(ST) + 512);          // QKV_ROPE: pos[64]
    float* freq_s = reinterpret_cast<float*>(smem + ring_bytes(ST) + 768);     // QKV_ROPE: inv_freq[32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int tile = blockIdx.x;
    const int n0 = tile * kGM;
    const GemmEpi& e = a.epi;
    // This grid row's K chunks: [c0, c1), an even split of the chunks over the ksplit rows.
    const int c0 = static_cast<int>(static_cast<long long>(blockIdx.y) * a.chunks / a.ksplit);
    const int c1 = static_cast<int>(static_cast<long long>(blockIdx.y + 1) * a.chunks / a.ksplit);
    const int nch = c1 - c0;
    // CTAs start at different chunks of their K range (and wrap around), so that at any moment they read
    // different activation tiles instead of all hitting the same L2 lines.
    const int rot = static_cast<int>(blockIdx.x % static_cast<unsigned>(nch));
    auto chunk_x = [&](int i) { return (c0 + (i + rot) % nch) * kGK; };
    grid_dep_launch();
    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&wmap);
        prefetch_tensormap(&xmap);
    }
    if (warp == 0) tmem_alloc(tmem_slot, kGN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer: chunk i of this CTA's K range into stage i % ST. The weight tiles of the
        // first ring pass do not depend on the previous kernel and are issued before waiting for it.
        const uint64_t pol = l2_policy_evict_first();
        const int pre = nch < ST ? nch : ST;
        for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], kWTileBytes + kXTileBytes);
            tma_load_2d_hint(wt + i * kWTileBytes, &wmap, chunk_x(i), n0, &full[i], pol);
        }
        grid_dep_wait();
        for (int i = 0; i < pre; ++i) tma_load_2d(xt + i * kXTileBytes, &xmap, chunk_x(i), 0, &full[i]);
        int issued = pre;
        for (int i = pre; i < nch; ++i) {
            const int s = i % ST;
            if (!gemm_wait(&empty[s], ((i / ST) - 1) & 1, a.err)) break;
            mbar_arrive_expect_tx(&full[s], kWTileBytes + kXTileBytes);
            tma_load_2d_hint(wt + s * kWTileBytes, &wmap, chunk_x(i), n0, &full[s], pol);
            tma_load_2d(xt + s * kXTileBytes, &xmap, chunk_x(i), 0, &full[s]);
            issued = i + 1;
        }
        // Every load issued lands before the CTA may exit (the MMA thread consumes them; this only
        // matters when a wait gave up).
        for (int i = issued > ST ? issued - ST : 0; i < issued; ++i) {
            gemm_wait(&full[i % ST], (i / ST) & 1, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: per stage, 4 K steps of 16 (+32 bytes inside the swizzled 128-byte rows), each one
        // MMA with the hi plane and one with the lo plane into the same accumulator.
        constexpr uint32_t idesc = idesc_bf16_f32(kGM, kGN);
        for (int i = 0; i < nch; ++i) {
            const int s = i % ST;
            if (!gemm_wait(&full[s], (i / ST) & 1, a.err)) break;
            tc_fence_after();
            const uint64_t ad = smem_desc_sw128(smem_addr(wt + s * kWTileBytes));
            const uint64_t bh = smem_desc_sw128(smem_addr(xt + s * kXTileBytes));
            const uint64_t bl = smem_desc_sw128(smem_addr(xt + s * kXTileBytes + kXPlaneBytes));
#pragma unroll
            for (int kk = 0; kk < kGK / 16; ++kk) {
                mma_f16(tmem, ad + 2u * kk, bh + 2u * kk, idesc, i > 0 || kk > 0);
                mma_f16(tmem, ad + 2u * kk, bl + 2u * kk, idesc, true);
            }
            mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        mma_commit(done);
    } else if (warp >= 2) {
        // Idle during the mainloop: the RMSNorm scale of each batch row from the partial sums of squares.
        grid_dep_wait();
        const int b = tid - 64;
        float inv = 1.f;
        if (e.ssq_in) {
            // Up to 16 partials (one per 128-row tile of the producing GEMM): loads issued together, added in
            // order.
            float part[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) part[i] = i < e.ssq_count ? __ldcg(e.ssq_in + i * kBatchMax + b) : 0.f;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) s += part[i];
            inv = rsqrtf(s / static_cast<float>(e.norm_n) + e.eps);
        }
        inv_rms[b] = inv;
        if constexpr (EPI == static_cast<int>(GemmEpilogue::QKV_ROPE)) {
            pos_s[b] = b < a.batch ? e.pos[b] : 0;
            if (b < 32) freq_s[b] = e.inv_freq[b];
        }
    }
    __syncwarp();
    // Everything below may write buffers the previous kernel reads.
    grid_dep_wait();
    if (lane == 0) gemm_wait(done, 0, a.err);
    __syncwarp();
    tc_fence_after();
    // Accumulator -> shared memory T[col][row] (the ring is idle: every load landed and every MMA ended).
    float* T = reinterpret_cast<float*>(smem);
    {
        const int row = 32 * warp + lane;
#pragma unroll
        for (int c = 0; c < kGN; c += 32) {
            float v[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(c), v);
#pragma unroll
            for (int j = 0; j < 32; ++j) T[(c + j) * kGM + row] = v[j];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kGN);
    const uint32_t ks = static_cast<uint32_t>(a.ksplit);
    const uint32_t rank = ks > 1 ? cluster_rank() : 0u;
    if (ks > 1) cluster_sync();  // every rank's partial tile is in its shared memory
    fused_epilogue<EPI, KV, kGThreads>(a, T, inv_rms, pos_s, freq_s, tile, ks, rank, tid);
    __syncwarp();
    if (ks > 1) cluster_sync();  // peers read this CTA's tile until every rank is done
}


// ---- int4 weights ------------------------------------------------------------------------------------
// The same GEMM for the .cudallm int4 layout (two 4-bit codes u = q + 8 per byte, one fp16 scale per
// 128-column group of a row). The engine re-packs every 32-bit word of codes once (interleave_int4_codes)
// so that its low nibbles hold columns 0-3 and its high nibbles columns 4-7 of an 8-column chunk. Per
// stage the TMA brings the raw codes of 128 rows x 64 columns (4 KiB, no swizzle) and the activation
// tile; four converter warps turn the codes into exact bf16 q = u - 8 (byte permutes against the bf16
// exponent of 128, one bf16x2 subtraction of 136 per pair) in the 128-byte-swizzled layout the MMA reads.
// The tensor core accumulates each 128-column group into one of two TMEM buffers; four accumulator warps
// (one per TMEM lane quarter, one thread per weight row) add scale[row][group] x group sum into fp32
// registers while the MMAs of the next group run, so the scales are applied exactly as the reference's
// per-group dequantisation (fp32 products, no rounding of q * scale to 16 bits).
constexpr int kI4Threads = 384;     // warp 0 TMA, 1 MMA, 2-3 RMSNorm scale, 4-7 accumulators, 8-11 converters
constexpr int kI4Stages = 6;
constexpr int kRawTileBytes = kGM * kGK / 2;  // 4 KiB of codes
constexpr int kI4StageBytes = kRawTileBytes + kWTileBytes + kXTileBytes;
constexpr int kI4RingBytes = kI4Stages * kI4StageBytes;
constexpr int kI4SmemBytes = 1024 + kI4RingBytes + kCtrlBytes;
static_assert(kI4SmemBytes <= 232448, "int4 GEMM shared memory above the per-block limit");
static_assert(kI4RingBytes >= 2 * kGN * kGM * 4 + 2 * kGN * 4 * 2, "the epilogue scratch lives in the ring");

struct GemmI4Args {
    GemmArgs g;
    const __half* scales;  // [n][k / 128]
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// 8 codes of one re-packed word -> 8 bf16 values q = u - 8 (columns 0..7 of the chunk).
__device__ __forceinline__ uint4 codes_to_bf16(uint32_t w) {
    const uint32_t t = w & 0x0F0F0F0Fu, u = (w >> 4) & 0x0F0F0F0Fu;
    const uint32_t magic = 0x43434343u;  // bf16 0x43xx = 128 + xx for xx < 128
    uint32_t p[4] = {prmt(t, magic, 0x4140u), prmt(t, magic, 0x4342u), prmt(u, magic, 0x4140u), prmt(u, magic, 0x4342u)};
    const __nv_bfloat162 off = __floats2bfloat162_rn(136.f, 136.f);
    uint4 r;
    uint32_t* rr = &r.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 v = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&p[i]), off);
        rr[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    return r;
}

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int EPI, typename KV>
__global__ void __launch_bounds__(kI4Threads, 1)
    gemm_i4_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, const GemmI4Args ai) {
    const GemmArgs& a = ai.g;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // Stage s: bf16 W tile at s*16K, X tile after the W tiles, raw codes after the X tiles (all 1024-aligned).
    uint8_t* wt = smem;
    uint8_t* xt = smem + kI4Stages * kWTileBytes;
    uint8_t* rt = xt + kI4Stages * kXTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kI4RingBytes);  // codes + activations landed
    uint64_t* conv = full + kI4Stages;                                  // bf16 tile written (128 arrivals)
    uint64_t* empty = conv + kI4Stages;                                 // MMAs done with the stage
    uint64_t* gfull = empty + kI4Stages;                                // [2] group accumulated in TMEM
    uint64_t* gempty = gfull + 2;                                       // [2] TMEM buffer read (128 arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gempty + 2);
    float* inv_rms = reinterpret_cast<float*>(smem + kI4RingBytes + 256);
    int* pos_s = reinterpret_cast<int*>(smem + kI4RingBytes + 512);
    float* freq_s = reinterpret_cast<float*>(smem + kI4RingBytes + 768);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int tile = blockIdx.x;
    const int n0 = tile * kGM;
    const GemmEpi& e = a.epi;
    // This grid row's 128-column groups: an even split of the groups over the ksplit rows.
    const int groups = a.chunks / 2;
    const int g0 = static_cast<int>(static_cast<long long>(blockIdx.y) * groups / a.ksplit);
    const int g1 = static_cast<int>(static_cast<long long>(blockIdx.y + 1) * groups / a.ksplit);
    const int ng = g1 - g0, nch = 2 * ng, c0 = 2 * g0;
    grid_dep_launch();
    if (tid == 0) {
        for (int s = 0; s < kI4Stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 128);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&gfull[b], 1);
            mbar_init(&gempty[b], 128);
        }
        fence_barrier_init();
        prefetch_tensormap(&wmap);
        prefetch_tensormap(&xmap);
    }
    if (warp == 0) tmem_alloc(tmem_slot, 2 * kGN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer: codes (before the dependency: weights) and activations of chunk i.
        const uint64_t pol = l2_policy_evict_first();
        const int pre = nch < kI4Stages ? nch : kI4Stages;
        for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], kRawTileBytes + kXTileBytes);
            tma_load_2d_hint(rt + i * kRawTileBytes, &wmap, (c0 + i) * (kGK / 2), n0, &full[i], pol);
        }
        grid_dep_wait();
        for (int i = 0; i < pre; ++i) tma_load_2d(xt + i * kXTileBytes, &xmap, (c0 + i) * kGK, 0, &full[i]);
        int issued = pre;
        for (int i = pre; i < nch; ++i) {
            const int s = i % kI4Stages;
            if (!gemm_wait(&empty[s], ((i / kI4Stages) - 1) & 1, a.err)) break;
            mbar_arrive_expect_tx(&full[s], kRawTileBytes + kXTileBytes);
            tma_load_2d_hint(rt + s * kRawTileBytes, &wmap, (c0 + i) * (kGK / 2), n0, &full[s], pol);
            tma_load_2d(xt + s * kXTileBytes, &xmap, (c0 + i) * kGK, 0, &full[s]);
            issued = i + 1;
        }
        for (int i = issued > kI4Stages ? issued - kI4Stages : 0; i < issued; ++i) {
            gemm_wait(&full[i % kI4Stages], (i / kI4Stages) & 1, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: group j of this CTA's range accumulates into TMEM buffer j % 2.
        constexpr uint32_t idesc = idesc_bf16_f32(kGM, kGN);
        bool ok = true;
        for (int i = 0; i < nch && ok; ++i) {
            const int s = i % kI4Stages, j = i >> 1;
            const uint32_t buf = tmem + static_cast<uint32_t>((j & 1) * kGN);
            if ((i & 1) == 0 && j >= 2) ok = gemm_wait(&gempty[j & 1], ((j >> 1) - 1) & 1, a.err);
            if (ok) ok = gemm_wait(&full[s], (i / kI4Stages) & 1, a.err);
            if (ok) ok = gemm_wait(&conv[s], (i / kI4Stages) & 1, a.err);
            if (!ok) break;
            tc_fence_after();
            const uint64_t ad = smem_desc_sw128(smem_addr(wt + s * kWTileBytes));
            const uint64_t bh = smem_desc_sw128(smem_addr(xt + s * kXTileBytes));
            const uint64_t bl = smem_desc_sw128(smem_addr(xt + s * kXTileBytes + kXPlaneBytes));
#pragma unroll
            for (int kk = 0; kk < kGK / 16; ++kk) {
                mma_f16(buf, ad + 2u * kk, bh + 2u * kk, idesc, (i & 1) || kk > 0);
                mma_f16(buf, ad + 2u * kk, bl + 2u * kk, idesc, true);
            }
            mma_commit(&empty[s]);
            if (i & 1) mma_commit(&gfull[j & 1]);
        }
    } else if (warp == 2 || warp == 3) {
        grid_dep_wait();
        const int b = tid - 64;
        float inv = 1.f;
        if (e.ssq_in) {
            float part[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) part[i] = i < e.ssq_count ? __ldcg(e.ssq_in + i * kBatchMax + b) : 0.f;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) s += part[i];
            inv = rsqrtf(s / static_cast<float>(e.norm_n) + e.eps);
        }
        inv_rms[b] = inv;
        if constexpr (EPI == static_cast<int>(GemmEpilogue::QKV_ROPE)) {
            pos_s[b] = b < a.batch ? e.pos[b] : 0;
            if (b < 32) freq_s[b] = e.inv_freq[b];
        }
    } else if (warp >= 8) {
        // Converters: thread r converts row r of each stage's codes (32 bytes -> 8 swizzled 16-byte chunks).
        const int r = tid - 256;
        for (int i = 0; i < nch; ++i) {
            const int s = i % kI4Stages;
            if (!gemm_wait(&full[s], (i / kI4Stages) & 1, a.err)) break;
            const uint4* src = reinterpret_cast<const uint4*>(rt + s * kRawTileBytes + r * 32);
            const uint4 w0 = src[0], w1 = src[1];
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            uint8_t* dst = wt + s * kWTileBytes + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                *reinterpret_cast<uint4*>(dst + ((c ^ (r & 7)) << 4)) = codes_to_bf16(words[c]);
            }
            fence_async_shared();  // the tensor core reads the tile through the async proxy
            mbar_arrive(&conv[s]);
        }
    }
    // Accumulators (warps 4-7): TMEM lane quarter q = warp % 4, thread = weight row 32q + lane.
    float acc[kGN];
#pragma unroll
    for (int j = 0; j < kGN; ++j) acc[j] = 0.f;
    if (warp >= 4 && warp < 8) {
        const int q = warp & 3, row = 32 * q + lane;
        const int grow = min(n0 + row, a.n - 1);
        const __half* sc = ai.scales + static_cast<size_t>(grow) * groups + g0;
        float s_next = ng > 0 ? __half2float(sc[0]) : 0.f;
        for (int j = 0; j < ng; ++j) {
            const float s = s_next;
            if (j + 1 < ng) s_next = __half2float(sc[j + 1]);
            int ok = 1;
            if (lane == 0) ok = gemm_wait(&gfull[j & 1], (j >> 1) & 1, a.err) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            const uint32_t buf = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>((j & 1) * kGN);
#pragma unroll
            for (int c = 0; c < kGN; c += 32) {
                float v[32];
                tmem_ld32(buf + static_cast<uint32_t>(c), v);
#pragma unroll
                for (int t = 0; t < 32; ++t) acc[c + t] = fmaf(s, v[t], acc[c + t]);
            }
            tc_fence_before();
            mbar_arrive(&gempty[j & 1]);
        }
    }
    __syncwarp();
    // Everything below may write buffers the previous kernel reads; the ring is idle once every group was
    // accumulated (the accumulators waited for the last MMAs, which read the last stages).
    grid_dep_wait();
    __syncthreads();
    float* T = reinterpret_cast<float*>(smem);
    if (warp >= 4 && warp < 8) {
        const int row = 32 * (warp & 3) + lane;
#pragma unroll
        for (int j = 0; j < kGN; ++j) T[j * kGM + row] = acc[j];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 2 * kGN);
    const uint32_t ks = static_cast<uint32_t>(a.ksplit);
    const uint32_t rank = ks > 1 ? cluster_rank() : 0u;
    if (ks > 1) cluster_sync();
    fused_epilogue<EPI, KV, kI4Threads>(a, T, inv_rms, pos_s, freq_s, tile, ks, rank, tid);
    __syncwarp();
    if (ks > 1) cluster_sync();
}

}  // namespace
}  // namespace cudallm

namespace cudallm {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    CLLM_CHECK(fn != nullptr, "CUDA driver entry point cuTensorMapEncodeTiled unavailable");
    return fn;
}

// Row-major [rows][cols] bf16 matrix, tiles of box_rows x 64 columns, 128-byte swizzle, zero fill out of
// bounds. Cached per (address, shape): weights are encoded once, activation buffers once per engine.
const CUtensorMap* tensor_map(const void* base, int rows, int cols, int box_rows) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int>, CUtensorMap> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(base, rows, cols, box_rows);
    auto it = cache.find(key);
    if (it != cache.end()) return &it->second;
    CUtensorMap map{};
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CLLM_CHECK(r == CUDA_SUCCESS, "CUDA cuTensorMapEncodeTiled failed");
    return &cache.emplace(key, map).first->second;
}

// Row-major [rows][cols] bytes (the int4 codes, two per byte), tiles of 128 rows x 32 bytes, no swizzle.
const CUtensorMap* tensor_map_codes(const void* base, int rows, int col_bytes) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int>, CUtensorMap> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(base, rows, col_bytes);
    auto it = cache.find(key);
    if (it != cache.end()) return &it->second;
    CUtensorMap map{};
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(col_bytes), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(col_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGK / 2), static_cast<cuuint32_t>(kGM)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CLLM_CHECK(r == CUDA_SUCCESS, "CUDA cuTensorMapEncodeTiled failed (int4 codes)");
    return &cache.emplace(key, map).first->second;
}

using GemmI4Fn = void (*)(CUtensorMap, CUtensorMap, GemmI4Args);

GemmI4Fn gemm_i4_fn(GemmEpilogue kind, bool kv_bf16) {
    switch (kind) {
        case GemmEpilogue::STORE: return gemm_i4_kernel<0, __half>;
        case GemmEpilogue::ADD: return gemm_i4_kernel<1, __half>;
        case GemmEpilogue::SWIGLU: return gemm_i4_kernel<2, __half>;
        case GemmEpilogue::QKV_ROPE: return kv_bf16 ? gemm_i4_kernel<3, __nv_bfloat16> : gemm_i4_kernel<3, __half>;
        case GemmEpilogue::LOGITS: return gemm_i4_kernel<4, __half>;
    }
    return nullptr;
}

void configure_i4(GemmI4Fn fn) {
    static std::mutex mu;
    static std::map<std::pair<GemmI4Fn, int>, bool> done;
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({fn, dev})) return;
    CLLM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kI4SmemBytes));
    CLLM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    done[{fn, dev}] = true;
}

// In place: each 32-bit word of codes (byte j = columns 2j | 2j+1 << 4 of an 8-column chunk) becomes
// byte j = columns j | j+4 << 4.
__global__ void interleave_int4_codes_kernel(uint32_t* __restrict__ w, size_t words) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < words;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t v = w[i];
        uint32_t out = 0;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t code = (v >> (4 * c)) & 0xFu;  // column c sits at nibble c of the original word
            const int byte = c & 3, hi = c >> 2;
            out |= code << (8 * byte + 4 * hi);
        }
        w[i] = out;
    }
}

using GemmFn = void (*)(CUtensorMap, CUtensorMap, GemmArgs);

// Ring depth: 7 stages, one CTA per SM (measured 2-3 % faster over a batched step than 3 stages with two
// CTAs per SM). The lm_head uses 3: with 1002 tiles, two CTAs per SM let one CTA's epilogue overlap the
// other's stream.
constexpr bool deep_ring() { return true; }

template <int ST>
GemmFn gemm_fn_st(GemmEpilogue kind, bool kv_bf16) {
    switch (kind) {
        case GemmEpilogue::STORE: return gemm_kernel<0, __half, ST>;
        case GemmEpilogue::ADD: return gemm_kernel<1, __half, ST>;
        case GemmEpilogue::SWIGLU: return gemm_kernel<2, __half, ST>;
        case GemmEpilogue::QKV_ROPE: return kv_bf16 ? gemm_kernel<3, __nv_bfloat16, ST> : gemm_kernel<3, __half, ST>;
        case GemmEpilogue::LOGITS: return gemm_kernel<4, __half, ST>;
    }
    return nullptr;
}

int gemm_stages(GemmEpilogue kind) { return kind != GemmEpilogue::LOGITS && deep_ring() ? kGStages : kGStagesLogits; }

GemmFn gemm_fn(GemmEpilogue kind, bool kv_bf16) {
    return gemm_stages(kind) == kGStages ? gemm_fn_st<kGStages>(kind, kv_bf16) : gemm_fn_st<kGStagesLogits>(kind, kv_bf16);
}

int gemm_smem(GemmEpilogue kind) { return smem_bytes(gemm_stages(kind)); }

// Shared-memory size and cluster permission, once per (kernel, device).
void configure(GemmFn fn, int smem) {
    static std::mutex mu;
    static std::map<std::pair<GemmFn, int>, bool> done;
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({fn, dev})) return;
    CLLM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    CLLM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    done[{fn, dev}] = true;
}

__global__ void interleave_gate_up_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int inter, int row_u4) {
    // (row_u4: 16-byte units per row; bf16 weights, int4 codes and fp16 group scales alike.)
    // dst row r: tile t = r / 128, q = r % 128 -> gate row 64t + q (q < 64) or up row 64t + q - 64.
    const int r = blockIdx.x;
    const int t = r / kGM, q = r % kGM;
    const int s = q < kGM / 2 ? kGM / 2 * t + q : inter + kGM / 2 * t + (q - kGM / 2);
    for (int c = threadIdx.x; c < row_u4; c += blockDim.x) dst[static_cast<size_t>(r) * row_u4 + c] = src[static_cast<size_t>(s) * row_u4 + c];
}

}  // namespace

int gemm_pick_ksplit(int n, int k) {
    int dev = 0, sms = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    CLLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int mtiles = (n + kGM - 1) / kGM;
    const int chunks = k / kGK;
    GemmFn fn = gemm_fn(GemmEpilogue::STORE, false);
    configure(fn, gemm_smem(GemmEpilogue::STORE));
    for (int ks = std::min({kMaxKsplit, chunks, std::max(1, sms / mtiles)}); ks > 1; --ks) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(mtiles, ks);
        cfg.blockDim = dim3(kGThreads);
        cfg.dynamicSmemBytes = gemm_smem(GemmEpilogue::STORE);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = ks;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (clusters >= mtiles) return ks;
    }
    return 1;
}

namespace {

void check_epi(const GemmEpi& epi, int n, int ksplit) {
    CLLM_CHECK(!epi.ssq_in || (epi.ssq_count >= 1 && epi.ssq_count <= 16 && epi.norm_n >= 1),
               "launch_gemm: bad RMSNorm statistics");
    switch (epi.kind) {
        case GemmEpilogue::STORE: CLLM_CHECK(epi.y, "launch_gemm: STORE needs y"); break;
        case GemmEpilogue::LOGITS:
            CLLM_CHECK(epi.y && epi.am_v && epi.am_i && ksplit == 1, "launch_gemm: LOGITS needs y, am_v, am_i and ksplit 1");
            break;
        case GemmEpilogue::ADD: CLLM_CHECK(epi.y && (!epi.planes || epi.gain), "launch_gemm: ADD needs y (and gain with planes)"); break;
        case GemmEpilogue::SWIGLU:
            CLLM_CHECK((epi.y || epi.planes) && n % kGM == 0, "launch_gemm: SWIGLU needs an output and n % 128 == 0");
            break;
        case GemmEpilogue::QKV_ROPE:
            CLLM_CHECK(epi.q_out && epi.inv_freq && epi.k_cache && epi.v_cache && epi.pos && epi.nh > 0 && epi.nkv > 0 &&
                           n == (epi.nh + 2 * epi.nkv) * 64 && n % kGM == 0 && epi.max_seq > 0,
                       "launch_gemm: bad QKV_ROPE arguments");
            break;
    }
}

// cudaLaunchKernelEx with a (1, ksplit, 1) cluster when ksplit > 1 and the programmatic attribute.
template <typename Fn, typename Arg>
void launch_tiles(Fn fn, int mtiles, int ksplit, int threads, int smem, cudaStream_t stream, bool pdl, const CUtensorMap& wm,
                  const CUtensorMap& xm, const Arg& arg) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(mtiles, ksplit);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (ksplit > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = ksplit;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    CLLM_CUDA(cudaLaunchKernelEx(&cfg, fn, wm, xm, arg));
}

}  // namespace

void launch_gemm(const __nv_bfloat16* w, int n, int k, const __nv_bfloat16* x, int batch, int ksplit, const GemmEpi& epi,
                 unsigned* err, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(w && x && err, "launch_gemm: null pointer");
    CLLM_CHECK(batch >= 1 && batch <= kGN, "launch_gemm: batch must be 1..64");
    CLLM_CHECK(n >= 1 && k >= kGK && k % kGK == 0 && ksplit >= 1 && ksplit <= std::min(kMaxKsplit, k / kGK),
               "launch_gemm: k must be a multiple of 64 and ksplit in 1..min(16, k/64)");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               "launch_gemm: operands must be 16-byte aligned");
    check_epi(epi, n, ksplit);
    GemmFn fn = gemm_fn(epi.kind, epi.kv_bf16);
    const int smem = gemm_smem(epi.kind);
    configure(fn, smem);
    const CUtensorMap* wm = tensor_map(w, n, k, kGM);
    const CUtensorMap* xm = tensor_map(x, kXRows, k, kXRows);
    const int mtiles = (n + kGM - 1) / kGM;
    const GemmArgs a{n, batch, k / kGK, ksplit, mtiles, err, epi};
    launch_tiles(fn, mtiles, ksplit, kGThreads, smem, stream, pdl, *wm, *xm, a);
}

void launch_gemm_int4(const uint8_t* codes, const __half* scales, int n, int k, const __nv_bfloat16* x, int batch, int ksplit,
                      const GemmEpi& epi, unsigned* err, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(codes && scales && x && err, "launch_gemm_int4: null pointer");
    CLLM_CHECK(batch >= 1 && batch <= kGN, "launch_gemm_int4: batch must be 1..64");
    CLLM_CHECK(n >= 1 && k >= 2 * kGK && k % (2 * kGK) == 0 && ksplit >= 1 && ksplit <= std::min(kMaxKsplit, k / (2 * kGK)),
               "launch_gemm_int4: k must be a multiple of 128 and ksplit in 1..min(16, k/128)");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               "launch_gemm_int4: operands must be 16-byte aligned");
    check_epi(epi, n, ksplit);
    GemmI4Fn fn = gemm_i4_fn(epi.kind, epi.kv_bf16);
    configure_i4(fn);
    const CUtensorMap* wm = tensor_map_codes(codes, n, k / 2);
    const CUtensorMap* xm = tensor_map(x, kXRows, k, kXRows);
    const int mtiles = (n + kGM - 1) / kGM;
    const GemmI4Args a{GemmArgs{n, batch, k / kGK, ksplit, mtiles, err, epi}, scales};
    launch_tiles(fn, mtiles, ksplit, kI4Threads, kI4SmemBytes, stream, pdl, *wm, *xm, a);
}

void interleave_gate_up(const __nv_bfloat16* src, __nv_bfloat16* dst, int inter, int k, cudaStream_t stream) {
    interleave_gate_up_rows(src, dst, inter, k * 2, stream);
}

void interleave_gate_up_rows(const void* src, void* dst, int inter, int row_bytes, cudaStream_t stream) {
    CLLM_CHECK(src && dst && src != dst && inter % (kGM / 2) == 0 && row_bytes % 16 == 0, "interleave_gate_up: bad arguments");
    interleave_gate_up_kernel<<<2 * inter, 256, 0, stream>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), inter,
                                                          row_bytes / 16);
    CLLM_CUDA(cudaGetLastError());
}

void interleave_int4_codes(void* codes, size_t bytes, cudaStream_t stream) {
    CLLM_CHECK(codes && bytes % 4 == 0 && (reinterpret_cast<uintptr_t>(codes) & 3) == 0, "interleave_int4_codes: bad arguments");
    const size_t words = bytes / 4;
    const int blocks = static_cast<int>(std::min<size_t>((words + 255) / 256, 148 * 16));
    interleave_int4_codes_kernel<<<blocks, 256, 0, stream>>>(static_cast<uint32_t*>(codes), words);
    CLLM_CUDA(cudaGetLastError());
}

int gemm_pick_ksplit_int4(int n, int k) {
    int dev = 0, sms = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    CLLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int mtiles = (n + kGM - 1) / kGM;
    const int groups = k / (2 * kGK);
    GemmI4Fn fn = gemm_i4_fn(GemmEpilogue::STORE, false);
    configure_i4(fn);
    for (int ks = std::min({kMaxKsplit, groups, std::max(1, sms / mtiles)}); ks > 1; --ks) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(mtiles, ks);
        cfg.blockDim = dim3(kI4Threads);
        cfg.dynamicSmemBytes = kI4SmemBytes;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = ks;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (clusters >= mtiles) return ks;
    }
    return 1;
}

}  // namespace cudallm
