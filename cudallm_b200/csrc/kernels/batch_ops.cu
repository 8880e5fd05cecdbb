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
// x[b][j] = emb[token][j] (bf16 weights), one block per row.
__global__ void embed_rows_kernel(const uint16_t* __restrict__ emb, const int* __restrict__ tok_in, const int* tok,
                                  float* __restrict__ x, int hidden) {
    grid_dep_launch();
    grid_dep_wait();
    const int b = blockIdx.x;
    const int t = tok_in[b] >= 0 ? tok_in[b] : tok[b];
    const uint16_t* row = emb + static_cast<size_t>(t) * hidden;
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) {
        x[static_cast<size_t>(b) * hidden + j] = __uint_as_float(static_cast<uint32_t>(row[j]) << 16);
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

// grid batch, block 1024: tok[b] = argmax of logits row b (lowest index on ties; all-NaN row -> 0),
// pos[b] += 1.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, int n, int* tok, int* pos_v) {
    grid_dep_launch();
    grid_dep_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int b = blockIdx.x;
    const float* row = logits + static_cast<size_t>(b) * n;
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int j = threadIdx.x; j < n; j += 1024) {
        const float v = row[j];
        if (v > bv || (v == bv && j < bi)) {
            bv = v;
            bi = j;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = sv[0];
        int i = si[0];
        for (int w = 1; w < 32; ++w) {
            if (sv[w] > v || (sv[w] == v && si[w] < i)) {
                v = sv[w];
                i = si[w];
            }
        }
        tok[b] = i == INT_MAX ? 0 : i;
        pos_v[b] += 1;
    }
}

}  // namespace

void launch_embed_rows(const uint16_t* emb, const int* tok_in, const int* tok, float* x, int batch, int hidden, cudaStream_t stream,
                       bool pdl) {
    CLLM_CHECK(emb && tok_in && tok && x && batch >= 1, "launch_embed_rows: bad arguments");
    launch_kernel(embed_rows_kernel, dim3(batch), dim3(256), 0, stream, pdl, emb, tok_in, tok, x, hidden);
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

void launch_argmax_rows(const float* logits, int n, int* tok, int* pos, int batch, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(logits && tok && pos && batch >= 1 && n >= 1, "launch_argmax_rows: bad arguments");
    launch_kernel(argmax_rows_kernel, dim3(batch), dim3(1024), 0, stream, pdl, logits, n, tok, pos);
}

template void launch_rope_kv_rows<__nv_bfloat16>(float*, const float*, __nv_bfloat16*, __nv_bfloat16*, size_t, const int*, int,
                                                 int, int, int, int, cudaStream_t, bool);
template void launch_rope_kv_rows<__half>(float*, const float*, __half*, __half*, size_t, const int*, int, int, int, int, int,
                                          cudaStream_t, bool);
template void launch_attention_rows<__nv_bfloat16>(const float*, const __nv_bfloat16*, const __nv_bfloat16*, size_t, const int*,
                                                   int, float*, float*, __nv_bfloat16*, int, int, int, int, cudaStream_t, bool);
template void launch_attention_rows<__half>(const float*, const __half*, const __half*, size_t, const int*, int, float*, float*,
                                            __nv_bfloat16*, int, int, int, int, cudaStream_t, bool);

}  // namespace cudallm
