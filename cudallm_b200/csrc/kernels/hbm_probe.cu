// HBM bandwidth probes behind cudallm_bandwidth (the counterpart of wasiqnauman/cudallm
// src/kernels/bandwidth.cu, whose read figure is the "measured peak" the reference divides by).
//
// Each probe moves a buffer larger than L2 once per launch:
//   * read: every thread keeps four independent 16-byte streaming loads in flight per iteration and folds
//     them into an XOR that is stored once per thread (so the loads cannot be dropped);
//   * write / copy: the same unrolled pattern with streaming stores;
//   * bulk read: the decode step's own way of reading weights. Each CTA streams its slice of the buffer
//     through a ring of shared-memory stages with 1-D bulk copies (cp.async.bulk + mbarrier), one lane
//     issuing, all threads touching one word per stage so the data is consumed.
#include <cuda_runtime.h>

#include <cstdint>

#include "common/check.h"
#include "kernels/kernels.h"
#include "kernels/ptx.cuh"

namespace cudallm {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(kProbeThreads) probe_read(const uint4* __restrict__ src, size_t n, unsigned* __restrict__ sink) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kProbeThreads;
    size_t i = blockIdx.x * static_cast<size_t>(kProbeThreads) + threadIdx.x;
    unsigned acc = 0;
    for (; i + (kUnroll - 1) * stride < n; i += kUnroll * stride) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    for (; i < n; i += stride) {
        const uint4 v = __ldcs(src + i);
        acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    sink[blockIdx.x * kProbeThreads + threadIdx.x] = acc;
}

__global__ void __launch_bounds__(kProbeThreads) probe_write(uint4* __restrict__ dst, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kProbeThreads;
    size_t i = blockIdx.x * static_cast<size_t>(kProbeThreads) + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < n; i += kUnroll * stride) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const unsigned w = static_cast<unsigned>(i + u * stride);
            __stcs(dst + i + u * stride, make_uint4(w, ~w, w, ~w));
        }
    }
    for (; i < n; i += stride) {
        const unsigned w = static_cast<unsigned>(i);
        __stcs(dst + i, make_uint4(w, ~w, w, ~w));
    }
}

__global__ void __launch_bounds__(kProbeThreads) probe_copy(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kProbeThreads;
    size_t i = blockIdx.x * static_cast<size_t>(kProbeThreads) + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < n; i += kUnroll * stride) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) __stcs(dst + i + u * stride, v[u]);
    }
    for (; i < n; i += stride) __stcs(dst + i, __ldcs(src + i));
}

constexpr int kBulkStages = 8;
constexpr uint32_t kBulkStageBytes = 16 * 1024;
constexpr unsigned long long kBulkWaitLimitNs = 1000000000ull;

// Every wait is bounded (1 s); a CTA that gives up records it in *err and stops issuing, and first lets
// every copy it issued land.
__global__ void __launch_bounds__(kProbeThreads) probe_bulk_read(const uint8_t* __restrict__ src, size_t chunks,
                                                                 unsigned* __restrict__ sink, unsigned* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t probe_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(probe_smem);
    uint8_t* ring = probe_smem + 128;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // Chunks c = blockIdx.x, blockIdx.x + gridDim.x, ...: chunk j of this CTA goes to stage j % kBulkStages.
    const size_t mine = chunks > blockIdx.x ? (chunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    size_t issued = 0;  // thread 0: chunks issued so far
    auto issue = [&](size_t j) {
        const size_t c = blockIdx.x + j * gridDim.x;
        const int s = static_cast<int>(j % kBulkStages);
        mbar_arrive_expect_tx(&full[s], kBulkStageBytes);
        bulk_load(ring + s * kBulkStageBytes, src + c * kBulkStageBytes, kBulkStageBytes, &full[s], l2_policy_evict_first());
        issued = j + 1;
    };
    if (threadIdx.x == 0) {
        for (size_t j = 0; j < mine && j < kBulkStages; ++j) issue(j);
    }
    unsigned acc = 0;
    bool ok = true;
    for (size_t j = 0; j < mine; ++j) {
        const int s = static_cast<int>(j % kBulkStages);
        const uint32_t parity = static_cast<uint32_t>((j / kBulkStages) & 1);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(&full[s], parity)) {
            if (global_ns() - t0 > kBulkWaitLimitNs) {
                ok = false;
                break;
            }
        }
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }
        acc ^= reinterpret_cast<const unsigned*>(ring + s * kBulkStageBytes)[threadIdx.x * 16];
        __syncthreads();  // the stage is consumed before it is refilled
        if (threadIdx.x == 0 && j + kBulkStages < mine) issue(j + kBulkStages);
    }
    if (!ok && threadIdx.x == 0) {
        atomicOr(err, 1u);
        // The last copy issued into each stage lands before the CTA exits (bounded as well).
        for (size_t j = issued > kBulkStages ? issued - kBulkStages : 0; j < issued; ++j) {
            const int s = static_cast<int>(j % kBulkStages);
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(&full[s], static_cast<uint32_t>((j / kBulkStages) & 1)) && global_ns() - t0 < kBulkWaitLimitNs) {
            }
        }
    }
    sink[blockIdx.x * kProbeThreads + threadIdx.x] = acc;
}

// Ring probe: 1-D bulk copies into 12 shared-memory stages of 16 KiB, one producer lane per stage (warp 0)
// and 8 consumer warps that touch a word of each stage and release it at once, with no block barrier per
// stage: the copy rate a weight ring like the decode step's can reach. Chunk j of a CTA is buffer chunk
// (blockIdx.x + j * gridDim.x) % chunks and goes to stage j % 12, so a buffer smaller than L2 is re-read from
// L2. A per-stage word holds the chunk last issued into the stage, so a consumer's parity test cannot pass
// on an older phase. Every wait is bounded (1 s); a CTA that gives up sets *err, and the producer lanes let
// their last copies land before the CTA exits.
constexpr int kRingStages = 12;
constexpr int kRingThreads = 384;

__device__ __forceinline__ void bulk_load_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__global__ void __launch_bounds__(kRingThreads, 1) probe_bulk_ring(const uint8_t* __restrict__ src, size_t chunks, int per_cta,
                                                                   unsigned* __restrict__ sink, unsigned* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t ring_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(ring_smem);
    uint64_t* empty = full + kRingStages;
    volatile int* stile = reinterpret_cast<volatile int*>(ring_smem + 256);
    volatile int* gave_up = reinterpret_cast<volatile int*>(ring_smem + 320);
    uint8_t* ring = ring_smem + 1024;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRingStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            stile[s] = -1;
        }
        *gave_up = 0;
        fence_barrier_init();
    }
    __syncthreads();
    auto chunk = [&](int j) { return src + ((blockIdx.x + static_cast<size_t>(j) * gridDim.x) % chunks) * kBulkStageBytes; };
    if (warp == 0) {
        if (lane < kRingStages) {
            int k = 0;  // copies issued into this lane's stage
            for (int j = lane; j < per_cta; j += kRingStages, ++k) {
                if (k > 0) {
                    const uint64_t t0 = global_ns();
                    while (!mbar_test_wait(&empty[lane], (k - 1) & 1)) {
                        if (*gave_up || global_ns() - t0 > kBulkWaitLimitNs) {
                            *gave_up = 1;
                            break;
                        }
                    }
                    if (*gave_up) break;
                }
                stile[lane] = j;
                mbar_arrive_expect_tx(&full[lane], kBulkStageBytes);
                bulk_load_plain(ring + lane * kBulkStageBytes, chunk(j), kBulkStageBytes, &full[lane]);
            }
            if (k > 0) {
                const uint64_t t0 = global_ns();
                while (!mbar_test_wait(&full[lane], (k - 1) & 1) && global_ns() - t0 < kBulkWaitLimitNs) {
                }
            }
        }
    } else if (warp >= 4) {
        const int cw = warp - 4;
        unsigned acc = 0;
        for (int j = cw; j < per_cta; j += 8) {
            const int s = j % kRingStages;
            const uint32_t parity = static_cast<uint32_t>((j / kRingStages) & 1);
            const uint64_t t0 = global_ns();
            bool ok = true;
            while (!__all_sync(0xffffffffu, stile[s] == j && mbar_test_wait(&full[s], parity))) {
                if (__any_sync(0xffffffffu, *gave_up != 0) || global_ns() - t0 > kBulkWaitLimitNs) {
                    ok = false;
                    break;
                }
            }
            if (!ok) {
                if (lane == 0) *gave_up = 1;
                break;
            }
            acc ^= reinterpret_cast<const unsigned*>(ring + s * kBulkStageBytes)[lane * 128];
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        sink[blockIdx.x * 256 + cw * 32 + lane] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0 && *gave_up) atomicOr(err, 1u);
}

}  // namespace

int probe_grid() { return num_sms() * 8; }

void launch_bw_read(const uint4* src, size_t n_uint4, unsigned* sink, int grid, cudaStream_t stream) {
    CLLM_CHECK(src && sink && n_uint4 > 0 && grid > 0, "launch_bw_read: bad arguments");
    probe_read<<<grid, kProbeThreads, 0, stream>>>(src, n_uint4, sink);
    CLLM_CUDA(cudaGetLastError());
}

void launch_bw_write(uint4* dst, size_t n_uint4, int grid, cudaStream_t stream) {
    CLLM_CHECK(dst && n_uint4 > 0 && grid > 0, "launch_bw_write: bad arguments");
    probe_write<<<grid, kProbeThreads, 0, stream>>>(dst, n_uint4);
    CLLM_CUDA(cudaGetLastError());
}

void launch_bw_copy(const uint4* src, uint4* dst, size_t n_uint4, int grid, cudaStream_t stream) {
    CLLM_CHECK(src && dst && n_uint4 > 0 && grid > 0, "launch_bw_copy: bad arguments");
    probe_copy<<<grid, kProbeThreads, 0, stream>>>(src, dst, n_uint4);
    CLLM_CUDA(cudaGetLastError());
}

size_t bulk_probe_chunk_bytes() { return kBulkStageBytes; }

size_t launch_bw_bulk_ring(const void* src, size_t bytes, int reps, unsigned* sink, unsigned* err, cudaStream_t stream) {
    CLLM_CHECK(src && sink && err && bytes >= kBulkStageBytes && reps >= 1, "launch_bw_bulk_ring: bad arguments");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(src) & 15u) == 0, "launch_bw_bulk_ring: source must be 16-byte aligned");
    const int smem = 1024 + kRingStages * static_cast<int>(kBulkStageBytes);
    static bool configured = false;
    if (!configured) {
        CLLM_CUDA(cudaFuncSetAttribute(probe_bulk_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured = true;
    }
    const size_t chunks = bytes / kBulkStageBytes;
    const int per_cta = static_cast<int>(chunks * static_cast<size_t>(reps) / static_cast<size_t>(num_sms()));
    CLLM_CHECK(per_cta >= 1, "launch_bw_bulk_ring: buffer too small for the grid");
    probe_bulk_ring<<<num_sms(), kRingThreads, smem, stream>>>(static_cast<const uint8_t*>(src), chunks, per_cta, sink, err);
    CLLM_CUDA(cudaGetLastError());
    return static_cast<size_t>(per_cta) * static_cast<size_t>(num_sms()) * kBulkStageBytes;
}

void launch_bw_bulk_read(const void* src, size_t bytes, unsigned* sink, unsigned* err, cudaStream_t stream) {
    CLLM_CHECK(src && sink && err && bytes >= kBulkStageBytes, "launch_bw_bulk_read: bad arguments");
    CLLM_CHECK((reinterpret_cast<uintptr_t>(src) & 15u) == 0, "launch_bw_bulk_read: source must be 16-byte aligned");
    const int smem = 128 + kBulkStages * kBulkStageBytes;
    static bool configured = false;
    if (!configured) {
        CLLM_CUDA(cudaFuncSetAttribute(probe_bulk_read, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured = true;
    }
    // One CTA per SM (the ring takes 128 KiB of shared memory).
    probe_bulk_read<<<num_sms(), kProbeThreads, smem, stream>>>(static_cast<const uint8_t*>(src), bytes / kBulkStageBytes,
                                                                 sink, err);
    CLLM_CUDA(cudaGetLastError());
}

}  // namespace cudallm
