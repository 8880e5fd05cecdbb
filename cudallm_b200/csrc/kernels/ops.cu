// Per-operation kernels other than the weight matvec: embedding gather, RMSNorm, RoPE / KV-cache
// write, decode attention (naive and split-K), elementwise ops, deterministic argmax and the DRAM
// bandwidth probes. Each one mirrors the semantics of the same-named launcher of
// wasiqnauman/cudallm src/kernels/*.cu (cited per kernel); the KV cache is templated on its element
// type (fp16, the reference's, or bf16).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>

#include "common/check.h"
#include "kernels/attention_core.cuh"
#include "kernels/kernels.h"
#include "kernels/matvec_core.cuh"

namespace cudallm {

namespace {

// ---- embedding (reference src/kernels/embedding.cu:14-29): x = dequant(emb[*d_token]) ----------
template <WeightType WT>
__global__ void embedding_kernel(const void* __restrict__ w, const void* __restrict__ scales, const int* __restrict__ d_token,
                                 float* __restrict__ x, int cols, int group_size) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    const size_t tok = static_cast<size_t>(*d_token);
    if constexpr (WT == WeightType::BF16) {
        x[j] = __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(w)[tok * cols + j]) << 16);
    } else if constexpr (WT == WeightType::INT8) {
        x[j] = static_cast<float>(static_cast<const int8_t*>(w)[tok * cols + j]) * static_cast<const float*>(scales)[tok];
    } else {
        const uint8_t b = static_cast<const uint8_t*>(w)[tok * (cols / 2) + j / 2];
        const int q = ((j & 1) ? (b >> 4) : (b & 0x0F)) - 8;
        x[j] = static_cast<float>(q) *
               __half2float(static_cast<const __half*>(scales)[tok * (cols / group_size) + j / group_size]);
    }
}

// ---- RMSNorm (reference src/kernels/rmsnorm.cu:12-20): y = x * rsqrt(mean(x^2) + eps) * w ------
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps, float* __restrict__ y,
                               int n) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) ss = fmaf(x[j], x[j], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / static_cast<float>(n) + eps);
    for (int j = threadIdx.x; j < n; j += blockDim.x) y[j] = x[j] * inv * w[j];
}

// ---- RoPE / KV write (reference src/kernels/rope_kv.cu:13-79) ----------------------------------
__device__ __forceinline__ void rotate_pair(float x0, float x1, float ang, float& r0, float& r1) {
    float s, c;
    sincosf(ang, &s, &c);
    r0 = x0 * c - x1 * s;
    r1 = x1 * c + x0 * s;
}

// grid nh + nkv, block hd/2: rotates q head b (b < nh) or k head b - nh in place.
__global__ void rope_inplace_kernel(float* __restrict__ qkv, const float* __restrict__ inv_freq, const int* __restrict__ d_pos,
                                    int hd) {
    const int half = hd / 2, i = threadIdx.x;
    float* v = qkv + static_cast<size_t>(blockIdx.x) * hd;
    float r0, r1;
    rotate_pair(v[i], v[i + half], static_cast<float>(*d_pos) * inv_freq[i], r0, r1);
    v[i] = r0;
    v[i + half] = r1;
}

// grid 2*nkv, block hd: copies k head b (b < nkv) or v head b - nkv into its cache row at pos.
template <typename KV>
__global__ void kv_write_kernel(const float* __restrict__ qkv, KV* __restrict__ k_cache, KV* __restrict__ v_cache,
                                const int* __restrict__ d_pos, int nh, int nkv, int hd, int max_seq) {
    const int b = blockIdx.x, d = threadIdx.x, pos = *d_pos;
    const bool is_k = b < nkv;
    const int head = is_k ? b : b - nkv;
    const float* src = qkv + static_cast<size_t>(nh + (is_k ? 0 : nkv) + head) * hd;
    KV* cache = is_k ? k_cache : v_cache;
    cache[(static_cast<size_t>(head) * max_seq + pos) * hd + d] = to_kv<KV>(src[d]);
}

// grid nh + 2*nkv, block hd/2: q heads rotated in place; k heads rotated into the cache (the k part
// of qkv is left as is); v heads copied into the cache.
template <typename KV>
__global__ void rope_kv_fused_kernel(float* __restrict__ qkv, const float* __restrict__ inv_freq, KV* __restrict__ k_cache,
                                     KV* __restrict__ v_cache, const int* __restrict__ d_pos, int nh, int nkv, int hd,
                                     int max_seq) {
    const int b = blockIdx.x, i = threadIdx.x, half = hd / 2, pos = *d_pos;
    if (b < nh + nkv) {
        float* v = qkv + static_cast<size_t>(b) * hd;
        float r0, r1;
        rotate_pair(v[i], v[i + half], static_cast<float>(pos) * inv_freq[i], r0, r1);
        if (b < nh) {
            v[i] = r0;
            v[i + half] = r1;
        } else {
            KV* dst = k_cache + (static_cast<size_t>(b - nh) * max_seq + pos) * hd;
            dst[i] = to_kv<KV>(r0);
            dst[i + half] = to_kv<KV>(r1);
        }
    } else {
        const int head = b - nh - nkv;
        const float* src = qkv + static_cast<size_t>(nh + nkv + head) * hd;
        KV* dst = v_cache + (static_cast<size_t>(head) * max_seq + pos) * hd;
        dst[2 * i] = to_kv<KV>(src[2 * i]);
        dst[2 * i + 1] = to_kv<KV>(src[2 * i + 1]);
    }
}

// ---- attention ---------------------------------------------------------------------------------
// Naive (reference src/kernels/attention_naive.cu:18-68): one block per query head over the whole
// context, scores in shared memory; every query head re-reads its KV head (the deliberate GQA
// inefficiency of the matvec/attn=naive baseline).
template <typename KV>
__global__ void attention_naive_kernel(const float* __restrict__ q, const KV* __restrict__ k_cache,
                                       const KV* __restrict__ v_cache, const int* __restrict__ d_pos, float* __restrict__ out,
                                       int nh, int nkv, int hd, int max_seq) {
    extern __shared__ float sc[];
    float* red = sc + max_seq;
    const int h = blockIdx.x, kvh = h / (nh / nkv), ctx = *d_pos + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float* qh = q + static_cast<size_t>(h) * hd;
    const KV* K = k_cache + static_cast<size_t>(kvh) * max_seq * hd;
    const KV* V = v_cache + static_cast<size_t>(kvh) * max_seq * hd;
    float mx = -INFINITY;
    for (int t = threadIdx.x; t < ctx; t += blockDim.x) {
        float dot = 0.f;
        for (int d = 0; d < hd; ++d) dot = fmaf(qh[d], kv_to_float(K[static_cast<size_t>(t) * hd + d]), dot);
        sc[t] = 0.125f * dot;
        mx = fmaxf(mx, sc[t]);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (warp == 0) {
        float m = lane < nw ? red[lane] : -INFINITY;
        m = warp_max(m);
        if (lane == 0) red[0] = m;
    }
    __syncthreads();
    const float m = red[0];
    __syncthreads();
    float sum = 0.f;
    for (int t = threadIdx.x; t < ctx; t += blockDim.x) {
        sc[t] = expf(sc[t] - m);
        sum += sc[t];
    }
    sum = warp_sum(sum);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (warp == 0) {
        float s = lane < nw ? red[lane] : 0.f;
        s = warp_sum(s);
        if (lane == 0) red[0] = s;
    }
    __syncthreads();
    const float total = red[0];
    if (threadIdx.x < hd) {
        const int d = threadIdx.x;
        float acc = 0.f;
        for (int t = 0; t < ctx; ++t) acc = fmaf(sc[t], kv_to_float(V[static_cast<size_t>(t) * hd + d]), acc);
        out[static_cast<size_t>(h) * hd + d] = acc / total;
    }
}

// Split-K partial: grid (nkv, max_seq / kAttnTile), 256 threads; tiles past the context exit at once
// so the grid is fixed (graph-capturable) while the work follows the context length.
template <typename KV>
__global__ void __launch_bounds__(kAttThreads) attention_partial_kernel(const float* __restrict__ q, const KV* k_cache,
                                                                        const KV* v_cache, const int* __restrict__ d_pos,
                                                                        float* part_o, float* part_ml, int nh, int max_seq) {
    __shared__ AttSmem<KV> sm;
    const int ctx = *d_pos + 1;
    const int tile = blockIdx.y;
    if (tile * kAttnTile >= ctx) return;
    attend_tile<KV, false>(PlainSrc{q}, nh, 0, nullptr, const_cast<KV*>(k_cache), const_cast<KV*>(v_cache), max_seq, blockIdx.x, tile,
                           ctx, max_seq / kAttnTile, part_o, part_ml, sm, threadIdx.x, [] { __syncthreads(); });
}

// Split-K combine: grid nkv, 256 threads (4 query heads x 64 dims).
__global__ void __launch_bounds__(kAttThreads) attention_combine_kernel(const float* part_o, const float* part_ml,
                                                                        const int* __restrict__ d_pos, float* out,
                                                                        int max_seq) {
    const int ctx = *d_pos + 1;
    combine_head(part_o, part_ml, blockIdx.x, (ctx + kAttnTile - 1) / kAttnTile, max_seq / kAttnTile, PlainDst{out},
                 threadIdx.x);
}

// ---- elementwise (reference src/kernels/elementwise.cu:10-24) ---------------------------------
__global__ void add_inplace_kernel(float* __restrict__ x, const float* __restrict__ y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += y[i];
}

__global__ void silu_mul_kernel(const float* __restrict__ gu, float* __restrict__ act, int inter) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < inter) act[i] = silu_f(gu[i]) * gu[i + inter];
}

__global__ void set_token_kernel(int* d_token, int token) { *d_token = token; }

// ---- argmax (reference src/kernels/argmax.cu:13-73) ------------------------------------------
// "Better" = larger value, or equal value and lower index. It is a total order, so any reduction
// tree gives the same winner.
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

__device__ __forceinline__ void block_argmax(float& v, int& i, float* sv, int* si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    warp_argmax(v, i);
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = i;
    }
    __syncthreads();
    if (warp == 0) {
        v = lane < nw ? sv[lane] : -INFINITY;
        i = lane < nw ? si[lane] : INT_MAX;
        warp_argmax(v, i);
    }
}

__global__ void argmax_partial_kernel(const float* __restrict__ logits, int n, float* __restrict__ part_v,
                                      int* __restrict__ part_i) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    block_argmax(bv, bi, sv, si);
    if (threadIdx.x == 0) {
        part_v[blockIdx.x] = bv;
        part_i[blockIdx.x] = bi;
    }
}

__global__ void argmax_final_kernel(const float* __restrict__ part_v, const int* __restrict__ part_i, int n_part,
                                    int* __restrict__ d_token, int* __restrict__ d_pos) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int k = threadIdx.x; k < n_part; k += blockDim.x) {
        if (better(part_v[k], part_i[k], bv, bi)) {
            bv = part_v[k];
            bi = part_i[k];
        }
    }
    block_argmax(bv, bi, sv, si);
    if (threadIdx.x == 0) {
        // Every logit NaN (never "better"): fall back to index 0 like a scan that keeps its start.
        *d_token = bi == INT_MAX ? 0 : bi;
        *d_pos += 1;
    }
}

// ---- DRAM bandwidth probes (reference src/kernels/bandwidth.cu:14-47) -------------------------
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

void launch_embedding(const Linear& emb, const int* d_token, float* x, int hidden, int group_size, cudaStream_t stream) {
    CLLM_CHECK(emb.w && d_token && x, "launch_embedding: null pointer");
    CLLM_CHECK(emb.cols == hidden && hidden % 256 == 0, "launch_embedding: hidden must equal emb.cols and be a multiple of 256");
    const dim3 grid(hidden / 256), block(256);
    switch (emb.wtype) {
        case WeightType::BF16:
            embedding_kernel<WeightType::BF16><<<grid, block, 0, stream>>>(emb.w, emb.scales, d_token, x, emb.cols, group_size);
            break;
        case WeightType::INT8:
            CLLM_CHECK(emb.scales, "launch_embedding: int8 needs scales");
            embedding_kernel<WeightType::INT8><<<grid, block, 0, stream>>>(emb.w, emb.scales, d_token, x, emb.cols, group_size);
            break;
        case WeightType::INT4:
            CLLM_CHECK(emb.scales && group_size > 0 && hidden % group_size == 0,
                       "launch_embedding: int4 needs scales and a valid group size");
            embedding_kernel<WeightType::INT4><<<grid, block, 0, stream>>>(emb.w, emb.scales, d_token, x, emb.cols, group_size);
            break;
    }
    CLLM_CUDA(cudaGetLastError());
}

void launch_rmsnorm(const float* x, const float* w, float eps, float* y, int n, cudaStream_t stream) {
    CLLM_CHECK(x && w && y, "launch_rmsnorm: null pointer");
    CLLM_CHECK(n > 0 && n % 256 == 0, "launch_rmsnorm: n must be a positive multiple of 256");
    rmsnorm_kernel<<<1, 256, 0, stream>>>(x, w, eps, y, n);
    CLLM_CUDA(cudaGetLastError());
}

template <typename KV>
void launch_rope_inplace(float* qkv, const float* inv_freq, const int* d_pos, int nh, int nkv, int hd, cudaStream_t stream) {
    CLLM_CHECK(qkv && inv_freq && d_pos, "launch_rope_inplace: null pointer");
    CLLM_CHECK(nh > 0 && nkv > 0 && hd > 0 && hd % 2 == 0 && hd <= 2048, "launch_rope_inplace: bad dimensions");
    rope_inplace_kernel<<<nh + nkv, hd / 2, 0, stream>>>(qkv, inv_freq, d_pos, hd);
    CLLM_CUDA(cudaGetLastError());
}

template <typename KV>
void launch_kv_write(const float* qkv, KV* k_cache_l, KV* v_cache_l, const int* d_pos, int nh, int nkv, int hd, int max_seq,
                     cudaStream_t stream) {
    CLLM_CHECK(qkv && k_cache_l && v_cache_l && d_pos, "launch_kv_write: null pointer");
    CLLM_CHECK(nh > 0 && nkv > 0 && hd > 0 && hd <= 1024 && max_seq > 0, "launch_kv_write: bad dimensions");
    kv_write_kernel<KV><<<2 * nkv, hd, 0, stream>>>(qkv, k_cache_l, v_cache_l, d_pos, nh, nkv, hd, max_seq);
    CLLM_CUDA(cudaGetLastError());
}

template <typename KV>
void launch_rope_kv_fused(float* qkv, const float* inv_freq, KV* k_cache_l, KV* v_cache_l, const int* d_pos, int nh, int nkv,
                          int hd, int max_seq, cudaStream_t stream) {
    CLLM_CHECK(qkv && inv_freq && k_cache_l && v_cache_l && d_pos, "launch_rope_kv_fused: null pointer");
    CLLM_CHECK(nh > 0 && nkv > 0 && hd > 0 && hd % 2 == 0 && hd <= 2048 && max_seq > 0, "launch_rope_kv_fused: bad dimensions");
    rope_kv_fused_kernel<KV><<<nh + 2 * nkv, hd / 2, 0, stream>>>(qkv, inv_freq, k_cache_l, v_cache_l, d_pos, nh, nkv, hd,
                                                                  max_seq);
    CLLM_CUDA(cudaGetLastError());
}

template <typename KV>
void launch_attention_naive(const float* q, const KV* k_l, const KV* v_l, const int* d_pos, float* out, int nh, int nkv,
                            int hd, int max_seq, cudaStream_t stream) {
    CLLM_CHECK(q && k_l && v_l && d_pos && out, "launch_attention_naive: null pointer");
    CLLM_CHECK(nh > 0 && nkv > 0 && nh % nkv == 0, "launch_attention_naive: nh must be a multiple of nkv");
    CLLM_CHECK(hd > 0 && hd <= 256 && max_seq > 0, "launch_attention_naive: bad dimensions");
    const size_t smem = (static_cast<size_t>(max_seq) + 32) * sizeof(float);
    CLLM_CHECK(smem <= 200 * 1024, "launch_attention_naive: max_seq too large for shared-memory scores");
    auto kernel = attention_naive_kernel<KV>;
    CLLM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    kernel<<<nh, 256, smem, stream>>>(q, k_l, v_l, d_pos, out, nh, nkv, hd, max_seq);
    CLLM_CUDA(cudaGetLastError());
}

template <typename KV>
void launch_attention_split(const float* q, const KV* k_l, const KV* v_l, const int* d_pos, float* part_o, float* part_ml,
                            float* out, int nh, int nkv, int hd, int max_seq, cudaStream_t stream) {
    CLLM_CHECK(q && k_l && v_l && d_pos && part_o && part_ml && out, "launch_attention_split: null pointer");
    CLLM_CHECK(nkv > 0 && nh == nkv * kGqa, "launch_attention_split: requires nh/nkv == 4");
    CLLM_CHECK(hd == kHd, "launch_attention_split: requires hd == 64");
    CLLM_CHECK(max_seq > 0 && max_seq % kAttnTile == 0, "launch_attention_split: max_seq must be a multiple of 64");
    CLLM_CHECK(aligned16(k_l) && aligned16(v_l), "launch_attention_split: caches must be 16-byte aligned");
    attention_partial_kernel<KV><<<dim3(nkv, max_seq / kAttnTile), kAttThreads, 0, stream>>>(q, k_l, v_l, d_pos, part_o,
                                                                                             part_ml, nh, max_seq);
    CLLM_CUDA(cudaGetLastError());
    attention_combine_kernel<<<nkv, kAttThreads, 0, stream>>>(part_o, part_ml, d_pos, out, max_seq);
    CLLM_CUDA(cudaGetLastError());
}

void launch_add_inplace(float* x, const float* y, int n, cudaStream_t stream) {
    CLLM_CHECK(x && y && n > 0, "launch_add_inplace: bad arguments");
    add_inplace_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, y, n);
    CLLM_CUDA(cudaGetLastError());
}

void launch_silu_mul(const float* gu, float* act, int inter, cudaStream_t stream) {
    CLLM_CHECK(gu && act && inter > 0, "launch_silu_mul: bad arguments");
    silu_mul_kernel<<<(inter + 255) / 256, 256, 0, stream>>>(gu, act, inter);
    CLLM_CUDA(cudaGetLastError());
}

void launch_set_token(int* d_token, int token, cudaStream_t stream) {
    CLLM_CHECK(d_token && token >= 0, "launch_set_token: bad arguments");
    set_token_kernel<<<1, 1, 0, stream>>>(d_token, token);
    CLLM_CUDA(cudaGetLastError());
}

void launch_argmax(const float* logits, int n, float* part_v, int* part_i, int* d_token, int* d_pos, cudaStream_t stream) {
    CLLM_CHECK(logits && part_v && part_i && d_token && d_pos, "launch_argmax: null pointer");
    CLLM_CHECK(n > 0, "launch_argmax: n must be positive");
    argmax_partial_kernel<<<kArgmaxBlocks, 256, 0, stream>>>(logits, n, part_v, part_i);
    CLLM_CUDA(cudaGetLastError());
    argmax_final_kernel<<<1, 256, 0, stream>>>(part_v, part_i, kArgmaxBlocks, d_token, d_pos);
    CLLM_CUDA(cudaGetLastError());
}

#define CLLM_INSTANTIATE_KV(KV)                                                                                            \
    template void launch_rope_inplace<KV>(float*, const float*, const int*, int, int, int, cudaStream_t);                  \
    template void launch_kv_write<KV>(const float*, KV*, KV*, const int*, int, int, int, int, cudaStream_t);               \
    template void launch_rope_kv_fused<KV>(float*, const float*, KV*, KV*, const int*, int, int, int, int, cudaStream_t); \
    template void launch_attention_naive<KV>(const float*, const KV*, const KV*, const int*, float*, int, int, int, int,   \
                                             cudaStream_t);                                                                \
    template void launch_attention_split<KV>(const float*, const KV*, const KV*, const int*, float*, float*, float*, int,  \
                                             int, int, int, cudaStream_t);
CLLM_INSTANTIATE_KV(__half)
CLLM_INSTANTIATE_KV(__nv_bfloat16)
#undef CLLM_INSTANTIATE_KV

}  // namespace cudallm
