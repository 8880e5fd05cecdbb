// Batched decode GEMM on the sm_100a tensor cores: part[ks][b][n] = sum over the ks-th K range of
// X[b][k] * W[n][k], W the [N][K] bf16 weight matrix (row-major, as stored in the .cudallm file), X the
// fp32 activations of up to 64 sequences carried as two bf16 planes, X = hi + lo (hi = bf16(X), lo =
// bf16(X - hi)), so the product keeps ~16 mantissa bits of the fp32 activation, like the batch-1 path's
// fp32 vectors. Weight rows are the MMA's M side: a CTA computes 128 weight rows x 64 batch columns
// (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 64, K = 16 per instruction; one MMA per plane into the
// same accumulator) in a 64-column fp32 TMEM accumulator, so every weight element is read from HBM once
// per step and used for the whole batch. Operands arrive by 2D TMA tensor loads (128-byte swizzle, no
// multicast) through a 7-stage ring of (W 128 x 64, X 2 x 64 x 64) tiles; one thread issues the loads,
// one thread the MMAs, and the 4 warps read the accumulator back (warp w owns TMEM lanes 32w..32w+31).
// K ranges per grid row (blockIdx.y) spread short operations over the SMs; gemm_reduce adds the ranges in
// order. The kernels take part in programmatic dependent launch: a GEMM starts streaming its weights
// while the kernel before it finishes and waits for it only before loading the activations.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

#include "common/check.h"
#include "kernels/batch.h"
#include "kernels/launch.cuh"
#include "kernels/tcgen05.cuh"

namespace cudallm {
namespace {

constexpr int kGM = 128;            // weight rows per CTA (MMA M)
constexpr int kGN = kBatchMax;      // batch columns (MMA N)
constexpr int kGK = 64;             // K per stage: one 128-byte swizzled row
constexpr int kXRows = 2 * kGN;     // hi plane rows 0..63, lo plane rows 64..127
constexpr int kGStages = 7;
constexpr int kGThreads = 128;
constexpr int kWTileBytes = kGM * kGK * 2;     // 16 KiB
constexpr int kXTileBytes = kXRows * kGK * 2;  // 16 KiB
constexpr int kXPlaneBytes = kGN * kGK * 2;    // lo plane offset inside an X tile (1024-byte aligned)
constexpr int kGSmemBytes = 1024 + kGStages * (kWTileBytes + kXTileBytes) + 256;
constexpr uint64_t kGemmWaitNs = 1000000000ull;

struct GemmArgs {
    float* part;                // [ksplit][batch][n]
    int n, batch, chunks, ksplit;  // chunks: 64-column K chunks in total
    unsigned* err;              // error word (set on a wait timeout)
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

__global__ void __launch_bounds__(kGThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* wt = smem;
    uint8_t* xt = smem + kGStages * kWTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(xt + kGStages * kXTileBytes);
    uint64_t* empty = full + kGStages;
    uint64_t* done = empty + kGStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kGM;
    // This grid row's K chunks: [c0, c1), an even split of the chunks over the ksplit rows.
    const int c0 = static_cast<int>(static_cast<long long>(blockIdx.y) * a.chunks / a.ksplit);
    const int c1 = static_cast<int>(static_cast<long long>(blockIdx.y + 1) * a.chunks / a.ksplit);
    const int nch = c1 - c0;
    // CTAs of one grid row start at different chunks of their K range (and wrap around), so that at any
    // moment they read different activation tiles instead of all hitting the same L2 lines.
    const int rot = static_cast<int>(blockIdx.x % static_cast<unsigned>(nch));
    auto chunk_x = [&](int i) { return (c0 + (i + rot) % nch) * kGK; };
    grid_dep_launch();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
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
        // TMA producer: chunk i of this CTA's K range into stage i % kGStages. The weight tiles of the
        // first ring pass do not depend on the previous kernel and are issued before waiting for it.
        const uint64_t pol = l2_policy_evict_first();
        const int pre = nch < kGStages ? nch : kGStages;
        for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], kWTileBytes + kXTileBytes);
            tma_load_2d_hint(wt + i * kWTileBytes, &wmap, chunk_x(i), n0, &full[i], pol);
        }
        grid_dep_wait();
        for (int i = 0; i < pre; ++i) tma_load_2d(xt + i * kXTileBytes, &xmap, chunk_x(i), 0, &full[i]);
        int issued = pre;
        for (int i = pre; i < nch; ++i) {
            const int s = i % kGStages;
            if (!gemm_wait(&empty[s], ((i / kGStages) - 1) & 1, a.err)) break;
            mbar_arrive_expect_tx(&full[s], kWTileBytes + kXTileBytes);
            tma_load_2d_hint(wt + s * kWTileBytes, &wmap, chunk_x(i), n0, &full[s], pol);
            tma_load_2d(xt + s * kXTileBytes, &xmap, chunk_x(i), 0, &full[s]);
            issued = i + 1;
        }
        // Every load issued lands before the CTA may exit (the MMA thread consumes them; this only
        // matters when a wait gave up).
        for (int i = issued > kGStages ? issued - kGStages : 0; i < issued; ++i) {
            gemm_wait(&full[i % kGStages], (i / kGStages) & 1, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: per stage, 4 K steps of 16 (+32 bytes inside the swizzled 128-byte rows), each one
        // MMA with the hi plane and one with the lo plane into the same accumulator.
        constexpr uint32_t idesc = idesc_bf16_f32(kGM, kGN);
        for (int i = 0; i < nch; ++i) {
            const int s = i % kGStages;
            if (!gemm_wait(&full[s], (i / kGStages) & 1, a.err)) break;
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
    }
    __syncwarp();
    // Epilogue: TMEM lane m = weight row n0 + m, column b = batch row b. The partials buffer may still be
    // read by the kernel before this one until it has completed.
    grid_dep_wait();
    if (lane == 0) gemm_wait(done, 0, a.err);
    __syncwarp();
    tc_fence_after();
    const int n = n0 + 32 * warp + lane;
#pragma unroll
    for (int c = 0; c < kGN; c += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(c), v);
        if (n < a.n) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int b = c + j;
                if (b < a.batch) a.part[(static_cast<size_t>(blockIdx.y) * a.batch + b) * a.n + n] = v[j];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kGN);
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

__device__ __forceinline__ float silu_g(float x) { return x / (1.f + __expf(-x)); }

// out[b][j] from sum over ks of part[ks][b][j] (added in ks order): STORE / ADD (residual) / SWIGLU
// (j < n/2: silu(s[j]) * s[n/2 + j]); outb (optional) gets the value as hi/lo bf16 planes.
__global__ void gemm_reduce_kernel(const float* __restrict__ part, int ksplit, int batch, int n, int ep, float* out,
                                   __nv_bfloat16* outb) {
    grid_dep_launch();
    grid_dep_wait();
    const int n_out = ep == static_cast<int>(GemmEpilogue::SWIGLU) ? n / 2 : n;
    const size_t total = static_cast<size_t>(batch) * n_out;
    const size_t plane = static_cast<size_t>(kBatchMax) * n_out;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(idx / n_out), j = static_cast<int>(idx % n_out);
        float v;
        if (ep == static_cast<int>(GemmEpilogue::SWIGLU)) {
            float g = 0.f, u = 0.f;
            for (int ks = 0; ks < ksplit; ++ks) {
                const float* pr = part + (static_cast<size_t>(ks) * batch + b) * n;
                g += pr[j];
                u += pr[n_out + j];
            }
            v = silu_g(g) * u;
        } else {
            float s = 0.f;
            for (int ks = 0; ks < ksplit; ++ks) s += part[(static_cast<size_t>(ks) * batch + b) * n + j];
            v = ep == static_cast<int>(GemmEpilogue::ADD) ? out[idx] + s : s;
        }
        if (out) out[idx] = v;
        if (outb) {
            const __nv_bfloat16 hi = __float2bfloat16_rn(v);
            outb[idx] = hi;
            outb[plane + idx] = __float2bfloat16_rn(v - __bfloat162float(hi));
        }
    }
}

}  // namespace

int gemm_smem_bytes() { return kGSmemBytes; }

void launch_gemm_bf16(const __nv_bfloat16* w, int n, int k, const __nv_bfloat16* x, int batch, int ksplit, float* part,
                      unsigned* err, cudaStream_t stream, bool pdl) {
    CLLM_CHECK(w && x && part && err, "launch_gemm_bf16: null pointer");
    CLLM_CHECK(batch >= 1 && batch <= kGN, "launch_gemm_bf16: batch must be 1..64");
    CLLM_CHECK(n >= 1 && k >= kGK && k % kGK == 0 && ksplit >= 1 && ksplit <= k / kGK,
               "launch_gemm_bf16: k must be a multiple of 64 with at least ksplit 64-column chunks");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
               "launch_gemm_bf16: operands must be 16-byte aligned");
    static bool configured[64] = {};
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || !configured[dev]) {
        CLLM_CUDA(cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmemBytes));
        if (dev < 64) configured[dev] = true;
    }
    const CUtensorMap* wm = tensor_map(w, n, k, kGM);
    const CUtensorMap* xm = tensor_map(x, kXRows, k, kXRows);
    GemmArgs a{part, n, batch, k / kGK, ksplit, err};
    launch_kernel(gemm_bf16_kernel, dim3((n + kGM - 1) / kGM, ksplit), dim3(kGThreads), kGSmemBytes, stream, pdl, *wm, *xm,
                  a);
}

void launch_gemm_reduce(const float* part, int ksplit, int batch, int n, GemmEpilogue ep, float* out, __nv_bfloat16* outb,
                        cudaStream_t stream, bool pdl) {
    CLLM_CHECK(part && (out || outb) && batch >= 1 && batch <= kBatchMax && n >= 1 && ksplit >= 1,
               "launch_gemm_reduce: bad arguments");
    CLLM_CHECK(ep != GemmEpilogue::ADD || out, "launch_gemm_reduce: ADD needs out");
    const size_t total = static_cast<size_t>(batch) * (ep == GemmEpilogue::SWIGLU ? n / 2 : n);
    const int blocks = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 8));
    launch_kernel(gemm_reduce_kernel, dim3(blocks), dim3(256), 0, stream, pdl, part, ksplit, batch, n, static_cast<int>(ep), out,
                  outb);
}

}  // namespace cudallm
