// Per-operation weight matvec for sm_100a: y = W x with optional fused RMSNorm prologue and
// STORE / ADD / SWIGLU epilogues (semantics of wasiqnauman/cudallm src/kernels/matvec_opt.cu:127-157,
// re-designed): each CTA owns a contiguous range of output rows; warp 0 streams that range's weight
// tiles into a ring of 16 KiB shared-memory stages with bulk (TMA) copies tracked by mbarriers, while
// 8 consumer warps stage the input vector once and then consume whole tiles (matvec_core.cuh).
// Also holds the deliberately naive bf16 matvec used by the matvec_impl=0 option.
#include <cuda_bf16.h>

#include <algorithm>

#include "common/check.h"
#include "kernels/kernels.h"
#include "kernels/matvec_core.cuh"
#include "kernels/ptx.cuh"

namespace cudallm {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kStreamThreads = 32 + kConsumerThreads;
constexpr int kStreamStages = 4;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

__host__ __device__ constexpr int align128(int v) { return (v + 127) & ~127; }

struct StreamLayout {
    int bars, tiles, red, xp, xc, scratch, ring, total;
};

__host__ __device__ inline StreamLayout stream_layout(int cols, int stages) {
    StreamLayout L;
    L.bars = 0;
    L.tiles = 2 * stages * 8;
    L.red = align128(L.tiles + stages * 4);
    L.xp = L.red + 128;
    L.xc = align128(L.xp + cols * 4);
    L.scratch = align128(L.xc + (cols / 32) * 4);
    L.ring = align128(L.scratch + kConsumerWarps * 32 * 4);
    L.total = L.ring + stages * kStageBytes;
    return L;
}

// Bounded wait on an mbarrier phase. Returns false (after recording *err) if it did not complete.
// With `tile_word`, first waits until the producer has published tile `tile` into that stage: a
// parity wait is only meaningful for the barrier's current or previous phase, and a consumer warp
// can be more than one phase ahead of a stage it does not consume every round.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, unsigned* err,
                                           const volatile int* tile_word = nullptr, int tile = 0) {
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        if ((tile_word == nullptr || *tile_word == tile) && mbar_try_wait(bar, parity)) return true;
        if ((it & 255) == 0) {
            const uint64_t t = global_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > kWaitLimitNs) {
                if (err) atomicOr(err, 1u);
                return false;
            }
        }
    }
}

// Consumer warp loop: row groups cw, cw+8, ... of this CTA's range, N = rows_per_tile * halves stage rows.
template <WeightType WT, Epilogue EP, int N>
__device__ __forceinline__ void consume_groups(const MatvecArgs& a, const TileGeom& g, int lo, int hi, const uint8_t* ring,
                                               uint64_t* full, uint64_t* empty, const volatile int* stage_tile,
                                               const float* xp, const float* xc, float* scratch, unsigned* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cw = warp - 1;
    const int R = g.rows_per_tile;
    const int n_groups = (hi - lo + R - 1) / R;
    const int nc = g.cols / Chunk<WT>::kCols;
    const int seg_chunks = g.seg_bytes / 16;
    float* my = scratch + cw * 32;
    for (int grp = cw; grp < n_groups; grp += kConsumerWarps) {
        const int r0 = lo + grp * R;
        const int nr = min(R, hi - r0);
        const TileRows tr{r0, R, g.halves == 2 ? g.out_rows : 0, g.out_rows * g.halves - 1};
        float acc[N];
#pragma unroll
        for (int i = 0; i < N; ++i) acc[i] = 0.f;
        for (int sg = 0; sg < g.n_seg; ++sg) {
            const int t = grp * g.n_seg + sg;
            const int s = t % kStreamStages;
            if (!wait_phase(&full[s], (t / kStreamStages) & 1, err, &stage_tile[s], t)) return;
            tile_dot<WT, N>(ring + s * kStageBytes, tr, g.seg_bytes, sg * seg_chunks, xp, nc, xc, a.scales, g.cols, acc, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const float v = warp_sum(acc[i]);
            if (lane == 0) my[i] = finish_row<WT>(v, a.scales, tr.global_row(i));
        }
        __syncwarp();
        if (lane < nr) {
            const int r = r0 + lane;
            if constexpr (EP == Epilogue::SWIGLU) {
                a.y[r] = silu_f(my[lane]) * my[R + lane];
            } else if constexpr (EP == Epilogue::ADD) {
                a.y[r] += my[lane];
            } else {
                a.y[r] = my[lane];
            }
        }
        __syncwarp();
    }
}

template <WeightType WT, Epilogue EP, bool NORM>
__global__ void __launch_bounds__(kStreamThreads) matvec_stream_kernel(const MatvecArgs a, const TileGeom g, unsigned* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const StreamLayout L = stream_layout(g.cols, kStreamStages);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + kStreamStages;
    volatile int* stage_tile = reinterpret_cast<volatile int*>(smem + L.tiles);
    float* red = reinterpret_cast<float*>(smem + L.red);
    float* xp = reinterpret_cast<float*>(smem + L.xp);
    float* xc = reinterpret_cast<float*>(smem + L.xc);
    float* scratch = reinterpret_cast<float*>(smem + L.scratch);
    uint8_t* ring = smem + L.ring;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lo = static_cast<int>(static_cast<long long>(blockIdx.x) * g.out_rows / gridDim.x);
    const int hi = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * g.out_rows / gridDim.x);
    const int R = g.rows_per_tile;
    const int n_groups = (hi - lo + R - 1) / R;
    const int n_tiles = n_groups * g.n_seg;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStreamStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            stage_tile[s] = -1;
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            const uint8_t* w = static_cast<const uint8_t*>(a.w);
            int issued = 0;
            for (int t = 0; t < n_tiles; ++t) {
                const int s = t % kStreamStages;
                const int k = t / kStreamStages;
                if (k > 0 && !wait_phase(&empty[s], (k - 1) & 1, err)) break;
                ++issued;
                const int grp = t / g.n_seg, sg = t % g.n_seg;
                const int r0 = lo + grp * R;
                const int nr = min(R, hi - r0);
                stage_tile[s] = t;
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nr * g.seg_bytes * g.halves));
                uint8_t* dst = ring + s * kStageBytes;
                for (int h = 0; h < g.halves; ++h) {
                    const size_t row = static_cast<size_t>(r0) + static_cast<size_t>(h) * g.out_rows;
                    if (g.n_seg == 1) {
                        bulk_load(dst + h * R * g.seg_bytes, w + row * g.row_bytes, static_cast<uint32_t>(nr * g.row_bytes),
                                  &full[s], pol);
                    } else {
                        for (int i = 0; i < nr; ++i) {
                            bulk_load(dst + (h * R + i) * g.seg_bytes,
                                      w + (row + i) * g.row_bytes + static_cast<size_t>(sg) * g.seg_bytes,
                                      static_cast<uint32_t>(g.seg_bytes), &full[s], pol);
                        }
                    }
                }
            }
            // Drain: every issued copy must land before the CTA may exit.
            for (int t = max(0, issued - kStreamStages); t < issued; ++t) {
                wait_phase(&full[t % kStreamStages], (t / kStreamStages) & 1, err);
            }
        }
        return;
    }

    const int tid = threadIdx.x - 32;
    stage_vector<WT>(GlobalVec4{a.x}, g.cols, NORM ? a.norm_w : nullptr, a.eps, xp, xc, red, tid,
                     kConsumerThreads, [] { named_barrier(1, kConsumerThreads); });

    switch (R * g.halves) {
        case 1: consume_groups<WT, EP, 1>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
        case 2: consume_groups<WT, EP, 2>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
        case 4: consume_groups<WT, EP, 4>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
        case 8: consume_groups<WT, EP, 8>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
        case 16: consume_groups<WT, EP, 16>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
        default: consume_groups<WT, EP, 32>(a, g, lo, hi, ring, full, empty, stage_tile, xp, xc, scratch, err); break;
    }
}

// One thread per output row, columns in order, uncoalesced on purpose: the baseline of the
// matvec_impl=0 option (reference src/kernels/matvec_naive.cu:13-21 semantics).
__global__ void matvec_naive_kernel(const uint16_t* __restrict__ w, const float* __restrict__ x, float* __restrict__ y,
                                    int rows, int cols) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const uint16_t* wr = w + static_cast<size_t>(row) * cols;
    float acc = 0.f;
    for (int j = 0; j < cols; ++j) acc += __uint_as_float(static_cast<uint32_t>(wr[j]) << 16) * x[j];
    y[row] = acc;
}

unsigned* hook_error_word() {
    // One process-wide device word for kernels launched outside an engine; never freed.
    static unsigned* p = [] {
        unsigned* q = nullptr;
        CLLM_CUDA(cudaMalloc(&q, sizeof(unsigned)));
        CLLM_CUDA(cudaMemset(q, 0, sizeof(unsigned)));
        return q;
    }();
    return p;
}

template <WeightType WT, Epilogue EP, bool NORM>
void launch_instance(const MatvecArgs& a, const TileGeom& g, cudaStream_t stream, unsigned* err) {
    auto kernel = matvec_stream_kernel<WT, EP, NORM>;
    const int smem = stream_layout(g.cols, kStreamStages).total;
    static int configured_smem[64] = {};
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || configured_smem[dev] < smem) {
        CLLM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        if (dev < 64) configured_smem[dev] = smem;
    }
    const int groups = (g.out_rows + g.rows_per_tile - 1) / g.rows_per_tile;
    const int grid = std::max(1, std::min(groups, 2 * num_sms()));
    kernel<<<grid, kStreamThreads, smem, stream>>>(a, g, err ? err : hook_error_word());
    CLLM_CUDA(cudaGetLastError());
}

template <WeightType WT, Epilogue EP>
void dispatch_norm(bool norm, const MatvecArgs& a, const TileGeom& g, cudaStream_t s, unsigned* err) {
    if (norm) {
        launch_instance<WT, EP, true>(a, g, s, err);
    } else {
        launch_instance<WT, EP, false>(a, g, s, err);
    }
}

template <WeightType WT>
void dispatch_ep(Epilogue ep, bool norm, const MatvecArgs& a, const TileGeom& g, cudaStream_t s, unsigned* err) {
    switch (ep) {
        case Epilogue::STORE: dispatch_norm<WT, Epilogue::STORE>(norm, a, g, s, err); return;
        case Epilogue::ADD: dispatch_norm<WT, Epilogue::ADD>(norm, a, g, s, err); return;
        case Epilogue::SWIGLU: dispatch_norm<WT, Epilogue::SWIGLU>(norm, a, g, s, err); return;
    }
    throw InternalError("launch_matvec_stream: unknown epilogue");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

void check_kernel_error() {
    unsigned v = 0;
    CLLM_CUDA(cudaMemcpy(&v, hook_error_word(), sizeof(v), cudaMemcpyDeviceToHost));
    if (v != 0) {
        CLLM_CUDA(cudaMemset(hook_error_word(), 0, sizeof(unsigned)));
        throw StateError("device: a bounded in-kernel wait gave up (code " + std::to_string(v) + ")");
    }
}

int num_sms() {
    static int n = [] {
        int dev = 0, v = 0;
        CLLM_CUDA(cudaGetDevice(&dev));
        CLLM_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
        return v;
    }();
    return n;
}

int default_rpb(WeightType) { return kMaxTileRows; }

TileGeom make_tile_geom(WeightType wt, Epilogue ep, int rows, int cols, int rpb, int seg_cap) {
    TileGeom g{};
    g.halves = ep == Epilogue::SWIGLU ? 2 : 1;
    g.out_rows = rows / g.halves;
    g.cols = cols;
    g.row_bytes = static_cast<int>(row_bytes(wt, static_cast<uint64_t>(cols)));
    const int stage_limit = kStageBytes / g.halves;
    const int limit = seg_cap > 0 ? std::min(seg_cap, stage_limit) : stage_limit;
    int seg = g.row_bytes;
    if (seg > limit) {
        const int units = g.row_bytes / 512;
        int best = 1;
        for (int d = 1; d <= units; ++d) {
            if (units % d == 0 && 512 * d <= limit) best = d;
        }
        seg = 512 * best;
    }
    g.seg_bytes = seg;
    g.n_seg = g.row_bytes / seg;
    const int cap = rpb > 0 ? std::min(rpb, kMaxTileRows) : kMaxTileRows;
    g.rows_per_tile = std::max(1, std::min(cap, stage_limit / seg));
    return g;
}

void launch_matvec_stream(WeightType wt, Epilogue ep, bool fuse_norm, const MatvecArgs& a, int rpb, cudaStream_t stream,
                          unsigned* err) {
    CLLM_CHECK(a.w && a.x && a.y, "launch_matvec_stream: null pointer");
    CLLM_CHECK(a.rows > 0 && a.cols > 0, "launch_matvec_stream: bad shape");
    CLLM_CHECK(a.cols % 1024 == 0, "launch_matvec_stream: cols must be a multiple of 1024");
    CLLM_CHECK(a.cols <= 16384, "launch_matvec_stream: cols must be at most 16384");
    CLLM_CHECK(ep != Epilogue::SWIGLU || a.rows % 2 == 0, "launch_matvec_stream: SWIGLU needs an even row count");
    CLLM_CHECK(rpb == 0 || rpb == 1 || rpb == 2 || rpb == 4 || rpb == 8 || rpb == 16,
               "launch_matvec_stream: rpb must be 0, 1, 2, 4, 8 or 16");
    CLLM_CHECK(aligned16(a.w) && aligned16(a.x) && aligned16(a.y), "launch_matvec_stream: pointers must be 16-byte aligned");
    CLLM_CHECK(!fuse_norm || a.norm_w, "launch_matvec_stream: fuse_norm needs norm_w");
    CLLM_CHECK(wt == WeightType::BF16 || a.scales, "launch_matvec_stream: quantized weights need scales");
    CLLM_CHECK(static_cast<const void*>(a.x) != static_cast<const void*>(a.y), "launch_matvec_stream: x and y alias");
    const TileGeom g = make_tile_geom(wt, ep, a.rows, a.cols, rpb);
    switch (wt) {
        case WeightType::BF16: dispatch_ep<WeightType::BF16>(ep, fuse_norm, a, g, stream, err); return;
        case WeightType::INT8: dispatch_ep<WeightType::INT8>(ep, fuse_norm, a, g, stream, err); return;
        case WeightType::INT4: dispatch_ep<WeightType::INT4>(ep, fuse_norm, a, g, stream, err); return;
    }
    throw InternalError("launch_matvec_stream: unknown weight type");
}

void launch_matvec_naive(const MatvecArgs& a, cudaStream_t stream) {
    CLLM_CHECK(a.w && a.x && a.y, "launch_matvec_naive: null pointer");
    CLLM_CHECK(a.rows > 0 && a.cols > 0, "launch_matvec_naive: bad shape");
    CLLM_CHECK(a.norm_w == nullptr, "launch_matvec_naive: fused norm not supported");
    CLLM_CHECK(static_cast<const void*>(a.x) != static_cast<const void*>(a.y), "launch_matvec_naive: x and y alias");
    matvec_naive_kernel<<<(a.rows + 255) / 256, 256, 0, stream>>>(static_cast<const uint16_t*>(a.w), a.x, a.y, a.rows,
                                                                  a.cols);
    CLLM_CUDA(cudaGetLastError());
}

}  // namespace cudallm
