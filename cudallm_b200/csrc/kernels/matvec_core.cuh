// Device building blocks of every weight matvec (per-op stream kernel and persistent decode step).
//
// Work unit: a *tile* = up to R consecutive weight rows x one row segment, fetched by a single bulk
// copy (two for SWIGLU: R gate rows then the R matching up rows) into one 16 KiB shared-memory stage.
// One warp consumes a tile: lane l owns the 16-byte chunks l, l+32, l+64, ... of every row, so the
// per-row accumulation order (and therefore every result bit) is independent of the tile shape, the
// grid and the kernel that runs it.
//
// The input vector is staged once per operation into shared memory as "planes": float4 p of chunk c
// (its columns 4p..4p+3) is stored at plane p, slot c, so the 32 lanes of a warp read 32 consecutive
// float4 (no bank conflicts). Each float4 holds two (even, odd) column pairs, which are the operand
// pairs of the packed FMAs: a lane keeps two accumulation chains per row, one over the even and one
// over the odd columns of its chunks.
//   bf16: 8 cols/chunk, word k = cols (2k, 2k+1)
//   int8: 16 cols/chunk, word k = cols 4k..4k+3
//   int4: 32 cols/chunk, word k byte b = cols 8k+2b (low nibble), 8k+2b+1 (high nibble)
// Dequantisation follows the reference formats (wasiqnauman/cudallm python/cudallm/quantize.py:5-29,
// src/kernels/matvec_opt.cu:65-115) but not its arithmetic:
//   int8: q = byte value, one fp32 scale per row applied after the row reduction.
//   int4: a nibble n is placed in mantissa bits 16..19 of 0.5f by one PRMT, giving f = 0.5 + n/256;
//         per 32-column chunk sum_i q_i x_i = 256 * sum_i f_i x_i - 136 * sum_i x_i (q = n - 8), where
//         sum_i x_i of the chunk is precomputed while staging. Two instructions per weight.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "common/dtype.h"
#include "kernels/kernels.h"

namespace cudallm {

template <WeightType WT>
struct Chunk;
template <>
struct Chunk<WeightType::BF16> {
    static constexpr int kCols = 8, kPlanes = 2;
};
template <>
struct Chunk<WeightType::INT8> {
    static constexpr int kCols = 16, kPlanes = 4;
};
template <>
struct Chunk<WeightType::INT4> {
    static constexpr int kCols = 32, kPlanes = 8;
};

// Float offset of column j inside the plane layout (nc = number of chunks of the vector).
template <WeightType WT>
__device__ __forceinline__ int plane_offset(int j, int nc) {
    constexpr int C = Chunk<WT>::kCols;
    const int c = j / C;
    const int i = j % C;
    return ((i >> 2) * nc + c) * 4 + (i & 3);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }

// Stages the vector (optionally RMS-normalised with gain norm_w) into planes `xp`, and for int4 the
// per-chunk sums into `xc`. `src4(q)` returns columns 4q..4q+3 as a float4. Runs on `nthr` == 256
// threads with index tid (which fixes the sum-of-squares order); every thread issues all of its loads
// (K/1024 float4) before using any, so staging costs one memory round trip, not K/256 of them.
// `sync()` is a barrier over those threads; `red` is 32 floats of scratch.
constexpr int kMaxStageK = 8192;
constexpr int kStagePer = kMaxStageK / 4 / 256;  // float4 per thread at the largest K
// Gain float4s per thread a caller may load ahead of time (gain_pre): all of them at K = 2048, 256 threads.
constexpr int kGainPre = 2;
// Second half of stage_vector: v[i] holds columns 4q..4q+3 for q = tid + i * nthr (q < K/4). gain_pre, if
// given, holds the first kGainPre gain float4s of this thread (the same indices), loaded by the caller.
template <WeightType WT, typename Sync>
__device__ __forceinline__ void stage_commit(float4 (&v)[kStagePer], int K, const float* __restrict__ norm_w, float eps,
                                             float* xp, float* xc, float* red, int tid, int nthr, Sync sync,
                                             const float4* gain_pre = nullptr) {
    constexpr int C = Chunk<WT>::kCols;
    constexpr int kMaxPer = kStagePer;
    const int nc = K / C;
    const int n4 = K / 4;
    if (norm_w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
            if (tid + i * nthr < n4) {
                ss = fmaf(v[i].x, v[i].x, ss);
                ss = fmaf(v[i].y, v[i].y, ss);
                ss = fmaf(v[i].z, v[i].z, ss);
                ss = fmaf(v[i].w, v[i].w, ss);
            }
        }
        float4 g[kMaxPer];
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
            const int q = tid + i * nthr;
            if (q < n4) g[i] = (gain_pre != nullptr && i < kGainPre) ? gain_pre[i] : __ldg(reinterpret_cast<const float4*>(norm_w) + q);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        sync();
        if (tid < 32) {
            float t = (tid < nthr / 32) ? red[tid] : 0.f;
            t = warp_sum(t);
            if (tid == 0) red[0] = t;
        }
        sync();
        const float inv = rsqrtf(red[0] / static_cast<float>(K) + eps);
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
            v[i].x = v[i].x * inv * g[i].x;
            v[i].y = v[i].y * inv * g[i].y;
            v[i].z = v[i].z * inv * g[i].z;
            v[i].w = v[i].w * inv * g[i].w;
        }
    }
    float4* p4 = reinterpret_cast<float4*>(xp);
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        const int q = tid + i * nthr;
        if (q >= n4) continue;
        const int c = (4 * q) / C, i0 = (4 * q) % C;
        p4[(i0 >> 2) * nc + c] = v[i];
    }
    sync();
    if constexpr (WT == WeightType::INT4) {
        for (int c = tid; c < nc; c += nthr) {
            // Per word k: the even columns 8k, 8k+2, 8k+4, 8k+6, then the odd ones.
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 a = p4[(2 * k) * nc + c], b = p4[(2 * k + 1) * nc + c];
                s += a.x + a.z + b.x + b.z;
                s += a.y + a.w + b.y + b.w;
            }
            xc[c] = s;
        }
        sync();
    }
}

template <WeightType WT, typename Src4, typename Sync>
__device__ __forceinline__ void stage_vector(Src4 src4, int K, const float* __restrict__ norm_w, float eps, float* xp,
                                             float* xc, float* red, int tid, int nthr, Sync sync) {
    const int n4 = K / 4;
    float4 v[kStagePer];
#pragma unroll
    for (int i = 0; i < kStagePer; ++i) {
        const int q = tid + i * nthr;
        if (q < n4) v[i] = src4(q);
    }
    stage_commit<WT>(v, K, norm_w, eps, xp, xc, red, tid, nthr, sync);
}

// float4 source over a global fp32 vector, read through L2 (data written by other CTAs).
struct GlobalVec4 {
    const float* p;
    __device__ __forceinline__ float4 operator()(int q) const { return __ldcg(reinterpret_cast<const float4*>(p) + q); }
};

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// int8: biased byte (q + 128) in the mantissa of 2^23, minus 2^23 + 128 -> q (exact).
__device__ __forceinline__ float i8val(uint32_t wb, uint32_t sel) {
    return __uint_as_float(__byte_perm(wb, 0x4B000000u, sel)) - 8388736.f;
}
// The same before the subtraction (2^23 + q + 128), for packed subtraction of the bias.
__device__ __forceinline__ float i8raw(uint32_t wb, uint32_t sel) { return __uint_as_float(__byte_perm(wb, 0x4B000000u, sel)); }
// int4: nibble n (already isolated in byte b) -> 0.5 + n/256.
__device__ __forceinline__ float i4half(uint32_t v, uint32_t sel) { return __uint_as_float(__byte_perm(v, 0x3F000000u, sel)); }

// Rows of one stage. Stage layout is fixed whatever the number of valid rows: stage row i sits at
// byte i * seg_bytes; for SWIGLU the R gate rows come first and the R matching up rows start at stage
// row R. Rows past the end of the matrix are computed on stale shared memory and discarded, so the
// accumulation loop has no per-row branches.
struct TileRows {
    int r0;      // first output row of the tile
    int R;       // rows per half
    int up_off;  // global row offset of the up half (SWIGLU), else 0
    int last;    // last row of the weight matrix (scale loads are clamped to it)
    __device__ __forceinline__ int global_row(int i) const {
        const int r = i < R ? r0 + i : r0 + (i - R) + up_off;
        return r < last ? r : last;
    }
};

// Accumulates one tile (N stage rows x one row segment) into acc[0..N). Two independent FMA chains
// per row keep the dependency latency hidden. CPL > 0 fixes the chunks per lane (segment bytes / 512)
// at compile time so the chunk loop unrolls completely; CPL == 0 reads it from seg_bytes.
// Packed fp32 pair arithmetic (sm_100 FFMA2 / FADD2): each half is an ordinary round-to-nearest fp32
// operation, so pairing two independent accumulation chains changes no result bit.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// Rows i < HALF are read from `stage` (row i at i * seg_bytes), rows i >= HALF from `stage_hi` (row i at
// (i - HALF) * seg_bytes): a warp that takes some gate rows and the matching up rows of a shared SwiGLU
// stage reads two blocks. With HALF == N (the default) stage_hi is unused.
template <WeightType WT, int N, int CPL = 0, int HALF = N>
__device__ __forceinline__ void tile_dot(const uint8_t* stage, const TileRows& tr, int seg_bytes, int seg_chunk0,
                                         const float* xp, int nc, const float* xc, const void* scales, int K,
                                         float (&acc)[N], int lane, const uint8_t* stage_hi = nullptr) {
    const float4* p4 = reinterpret_cast<const float4*>(xp);
    auto row_at = [&](int i) { return i < HALF ? stage + i * seg_bytes : stage_hi + (i - HALF) * seg_bytes; };
    const int cpl = CPL > 0 ? CPL : (seg_bytes >> 9);  // chunks per lane per row
    if constexpr (CPL > 0) seg_bytes = CPL * 512;
    [[maybe_unused]] const int groups = K >> 7;
    if constexpr (WT == WeightType::INT4 && CPL > 0) {
        // Compile-time tile shape: one scalar chain per row, accumulated straight into acc (the group
        // scale is applied per chunk).
        const __half* sc = static_cast<const __half*>(scales);
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            const int gc = seg_chunk0 + c;
            const float xsum = xc[gc];
            float4 xa[4], xb[4];  // word k: columns 8k..8k+3 and 8k+4..8k+7
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                xa[k] = p4[(2 * k) * nc + gc];
                xb[k] = p4[(2 * k + 1) * nc + gc];
            }
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const uint4 w = *reinterpret_cast<const uint4*>(row_at(i) + c * 16);
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
                float2 pp = make_float2(0.f, 0.f);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t lo = words[k] & 0x0F0F0F0Fu;
                    const uint32_t hi = (words[k] >> 4) & 0x0F0F0F0Fu;
                    pp = fma2(make_float2(i4half(lo, 0x7044), i4half(hi, 0x7044)), make_float2(xa[k].x, xa[k].y), pp);
                    pp = fma2(make_float2(i4half(lo, 0x7144), i4half(hi, 0x7144)), make_float2(xa[k].z, xa[k].w), pp);
                    pp = fma2(make_float2(i4half(lo, 0x7244), i4half(hi, 0x7244)), make_float2(xb[k].x, xb[k].y), pp);
                    pp = fma2(make_float2(i4half(lo, 0x7344), i4half(hi, 0x7344)), make_float2(xb[k].z, xb[k].w), pp);
                }
                const float si = __half2float(__ldg(sc + static_cast<size_t>(tr.global_row(i)) * groups + (gc >> 2)));
                acc[i] = fmaf(si, fmaf(256.f, pp.x + pp.y, -136.f * xsum), acc[i]);
            }
        }
        return;
    } else {
        // Two accumulation chains per row (.x and .y), advanced together by one packed instruction.
        float2 a[N];
#pragma unroll
        for (int i = 0; i < N; ++i) a[i] = make_float2(0.f, 0.f);
#pragma unroll(CPL > 0 ? CPL : 2)
        for (int j = 0; j < cpl; ++j) {
            const int c = lane + 32 * j;
            const int gc = seg_chunk0 + c;
            if constexpr (WT == WeightType::BF16) {
                const float4 x0 = p4[gc], x1 = p4[nc + gc];
#pragma unroll
                for (int i = 0; i < N; ++i) {
                    const uint4 w = *reinterpret_cast<const uint4*>(row_at(i) + c * 16);
                    a[i] = fma2(make_float2(bf16lo(w.x), bf16hi(w.x)), make_float2(x0.x, x0.y), a[i]);
                    a[i] = fma2(make_float2(bf16lo(w.y), bf16hi(w.y)), make_float2(x0.z, x0.w), a[i]);
                    a[i] = fma2(make_float2(bf16lo(w.z), bf16hi(w.z)), make_float2(x1.x, x1.y), a[i]);
                    a[i] = fma2(make_float2(bf16lo(w.w), bf16hi(w.w)), make_float2(x1.z, x1.w), a[i]);
                }
            } else if constexpr (WT == WeightType::INT8) {
                const float4 x0 = p4[gc], x1 = p4[nc + gc], x2 = p4[2 * nc + gc], x3 = p4[3 * nc + gc];
                const float2 bias = make_float2(-8388736.f, -8388736.f);
#pragma unroll
                for (int i = 0; i < N; ++i) {
                    const uint4 w = *reinterpret_cast<const uint4*>(row_at(i) + c * 16);
                    const uint32_t b0 = w.x ^ 0x80808080u, b1 = w.y ^ 0x80808080u, b2 = w.z ^ 0x80808080u,
                                   b3 = w.w ^ 0x80808080u;
                    a[i] = fma2(add2(make_float2(i8raw(b0, 0x7540), i8raw(b0, 0x7541)), bias), make_float2(x0.x, x0.y), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b0, 0x7542), i8raw(b0, 0x7543)), bias), make_float2(x0.z, x0.w), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b1, 0x7540), i8raw(b1, 0x7541)), bias), make_float2(x1.x, x1.y), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b1, 0x7542), i8raw(b1, 0x7543)), bias), make_float2(x1.z, x1.w), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b2, 0x7540), i8raw(b2, 0x7541)), bias), make_float2(x2.x, x2.y), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b2, 0x7542), i8raw(b2, 0x7543)), bias), make_float2(x2.z, x2.w), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b3, 0x7540), i8raw(b3, 0x7541)), bias), make_float2(x3.x, x3.y), a[i]);
                    a[i] = fma2(add2(make_float2(i8raw(b3, 0x7542), i8raw(b3, 0x7543)), bias), make_float2(x3.z, x3.w), a[i]);
                }
            } else {
                const float xsum = xc[gc];
                const int g = gc >> 2;  // 128-column group of this chunk
                const __half* sc = static_cast<const __half*>(scales);
                float4 xa[4], xb[4];  // word k: columns 8k..8k+3 and 8k+4..8k+7
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    xa[k] = p4[(2 * k) * nc + gc];
                    xb[k] = p4[(2 * k + 1) * nc + gc];
                }
#pragma unroll
                for (int i = 0; i < N; ++i) {
                    const uint4 w = *reinterpret_cast<const uint4*>(row_at(i) + c * 16);
                    const float s = __half2float(__ldg(sc + static_cast<size_t>(tr.global_row(i)) * groups + g));
                    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
                    float2 pp = make_float2(0.f, 0.f);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t lo = words[k] & 0x0F0F0F0Fu;
                        const uint32_t hi = (words[k] >> 4) & 0x0F0F0F0Fu;
                        pp = fma2(make_float2(i4half(lo, 0x7044), i4half(hi, 0x7044)), make_float2(xa[k].x, xa[k].y), pp);
                        pp = fma2(make_float2(i4half(lo, 0x7144), i4half(hi, 0x7144)), make_float2(xa[k].z, xa[k].w), pp);
                        pp = fma2(make_float2(i4half(lo, 0x7244), i4half(hi, 0x7244)), make_float2(xb[k].x, xb[k].y), pp);
                        pp = fma2(make_float2(i4half(lo, 0x7344), i4half(hi, 0x7344)), make_float2(xb[k].z, xb[k].w), pp);
                    }
                    a[i].x = fmaf(s, fmaf(256.f, pp.x + pp.y, -136.f * xsum), a[i].x);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < N; ++i) acc[i] += a[i].x + a[i].y;
    }
}

// Register-staged form of tile_dot for bf16 and int8 tiles with a compile-time shape (N rows of CPL chunks per
// lane, rows contiguous at CPL * 512 bytes): load_tile_regs copies chunks j0 .. j0 + H - 1 of this lane's
// chunks of every row into registers, so the caller can release the stage before all the arithmetic is done
// and the ring refills while the warp computes; tile_dot_regs advances the two accumulation chains per row
// a[i] over those chunks. Called over consecutive chunk ranges from a[i] = 0 and followed by
// acc[i] += a[i].x + a[i].y, it performs exactly tile_dot's operations in tile_dot's order (bit-identical).
template <WeightType WT, int N, int H, int CPL>
__device__ __forceinline__ void load_tile_regs(const uint8_t* stage, uint4 (&w)[N][H], int lane, int j0) {
    static_assert(WT != WeightType::INT4, "int4 stages are shared between warps");
#pragma unroll
    for (int j = 0; j < H; ++j) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            w[i][j] = *reinterpret_cast<const uint4*>(stage + i * (CPL * 512) + (lane + 32 * (j0 + j)) * 16);
        }
    }
}

template <WeightType WT, int N, int H>
__device__ __forceinline__ void tile_dot_regs(const uint4 (&w)[N][H], int chunk0, const float* xp, int nc, float2 (&a)[N],
                                              int lane) {
    static_assert(WT != WeightType::INT4, "int4 stages are shared between warps");
    const float4* p4 = reinterpret_cast<const float4*>(xp);
#pragma unroll
    for (int j = 0; j < H; ++j) {
        const int gc = chunk0 + lane + 32 * j;
        if constexpr (WT == WeightType::BF16) {
            const float4 x0 = p4[gc], x1 = p4[nc + gc];
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const uint4 v = w[i][j];
                a[i] = fma2(make_float2(bf16lo(v.x), bf16hi(v.x)), make_float2(x0.x, x0.y), a[i]);
                a[i] = fma2(make_float2(bf16lo(v.y), bf16hi(v.y)), make_float2(x0.z, x0.w), a[i]);
                a[i] = fma2(make_float2(bf16lo(v.z), bf16hi(v.z)), make_float2(x1.x, x1.y), a[i]);
                a[i] = fma2(make_float2(bf16lo(v.w), bf16hi(v.w)), make_float2(x1.z, x1.w), a[i]);
            }
        } else {
            const float4 x0 = p4[gc], x1 = p4[nc + gc], x2 = p4[2 * nc + gc], x3 = p4[3 * nc + gc];
            const float2 bias = make_float2(-8388736.f, -8388736.f);
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const uint4 v = w[i][j];
                const uint32_t b0 = v.x ^ 0x80808080u, b1 = v.y ^ 0x80808080u, b2 = v.z ^ 0x80808080u, b3 = v.w ^ 0x80808080u;
                a[i] = fma2(add2(make_float2(i8raw(b0, 0x7540), i8raw(b0, 0x7541)), bias), make_float2(x0.x, x0.y), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b0, 0x7542), i8raw(b0, 0x7543)), bias), make_float2(x0.z, x0.w), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b1, 0x7540), i8raw(b1, 0x7541)), bias), make_float2(x1.x, x1.y), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b1, 0x7542), i8raw(b1, 0x7543)), bias), make_float2(x1.z, x1.w), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b2, 0x7540), i8raw(b2, 0x7541)), bias), make_float2(x2.x, x2.y), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b2, 0x7542), i8raw(b2, 0x7543)), bias), make_float2(x2.z, x2.w), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b3, 0x7540), i8raw(b3, 0x7541)), bias), make_float2(x3.x, x3.y), a[i]);
                a[i] = fma2(add2(make_float2(i8raw(b3, 0x7542), i8raw(b3, 0x7543)), bias), make_float2(x3.z, x3.w), a[i]);
            }
        }
    }
}

// Row result after the warp reduction (all lanes hold it); int8 applies its per-row scale here.
template <WeightType WT>
__device__ __forceinline__ float finish_row(float reduced, const void* scales, int global_row) {
    if constexpr (WT == WeightType::INT8) {
        return reduced * __ldg(static_cast<const float*>(scales) + global_row);
    } else {
        return reduced;
    }
}

}  // namespace cudallm
