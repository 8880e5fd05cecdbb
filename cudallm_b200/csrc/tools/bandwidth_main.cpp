// cudallm_bandwidth: measured HBM bandwidth of this GPU, the denominator of "% of peak" in the decode
// benchmarks. Flags and JSON keys are those of wasiqnauman/cudallm src/tools/cudallm_bandwidth.cpp (its
// bench/bench_bandwidth.py reads read_gbps_best as the measured peak).
//
// Buffers of 1 GiB (8x the L2) are read, written and copied by the probes in kernels/hbm_probe.cu, 3
// untimed and 20 timed launches each, with CUDA events; GB/s counts the bytes moved (a copy counts its read
// and its write). Added keys: bulk_read_gbps_best / _median, the read rate of 1-D bulk (TMA) copies into
// shared memory, which is how the decode step streams its weights; bulk_read_l2_gbps_best / _median, the same
// copies from a 48 MiB buffer resident in L2 (how fast the ring can refill from L2-prefetched weights).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "common/check.h"
#include "kernels/kernels.h"
#include "tools/cli.h"

using cudallm::tools::JsonValue;
using cudallm::tools::Options;

namespace {

constexpr size_t kBytes = size_t{1} << 30;
constexpr size_t kL2Bytes = size_t{48} << 20;
constexpr int kUntimed = 3;
constexpr int kTimed = 20;

struct Rate {
    double best, median;
};

Rate time_rate(const std::function<void()>& launch, double bytes) {
    for (int i = 0; i < kUntimed; ++i) launch();
    CLLM_CUDA(cudaDeviceSynchronize());
    cudaEvent_t a, b;
    CLLM_CUDA(cudaEventCreate(&a));
    CLLM_CUDA(cudaEventCreate(&b));
    std::vector<double> gbs;
    for (int i = 0; i < kTimed; ++i) {
        CLLM_CUDA(cudaEventRecord(a, 0));
        launch();
        CLLM_CUDA(cudaEventRecord(b, 0));
        CLLM_CUDA(cudaEventSynchronize(b));
        float ms = 0.f;
        CLLM_CUDA(cudaEventElapsedTime(&ms, a, b));
        gbs.push_back(bytes / (ms * 1e-3) / 1e9);
    }
    CLLM_CUDA(cudaEventDestroy(a));
    CLLM_CUDA(cudaEventDestroy(b));
    std::sort(gbs.begin(), gbs.end());
    return {gbs.back(), 0.5 * (gbs[kTimed / 2 - 1] + gbs[kTimed / 2])};
}

}  // namespace

int main(int argc, char** argv) {
    Options opt("cudallm_bandwidth", "[--json PATH]");
    opt.add("json", "", "write the result here");
    opt.parse(argc, argv);
    uint4 *src = nullptr, *dst = nullptr;
    unsigned *sink = nullptr, *err = nullptr;
    int status = 0;
    try {
        using namespace cudallm;
        int dev = 0;
        CLLM_CUDA(cudaGetDevice(&dev));
        cudaDeviceProp prop{};
        CLLM_CUDA(cudaGetDeviceProperties(&prop, dev));
        const int grid = probe_grid();
        const size_t n = kBytes / sizeof(uint4);
        CLLM_CUDA(cudaMalloc(&src, kBytes));
        CLLM_CUDA(cudaMalloc(&dst, kBytes));
        CLLM_CUDA(cudaMalloc(&sink, sizeof(unsigned) * static_cast<size_t>(std::max(grid, num_sms())) * 256));
        CLLM_CUDA(cudaMalloc(&err, sizeof(unsigned)));
        CLLM_CUDA(cudaMemset(src, 0x5a, kBytes));
        CLLM_CUDA(cudaMemset(dst, 0, kBytes));
        CLLM_CUDA(cudaMemset(err, 0, sizeof(unsigned)));
        const Rate rd = time_rate([&] { launch_bw_read(src, n, sink, grid, 0); }, kBytes);
        const Rate wr = time_rate([&] { launch_bw_write(dst, n, grid, 0); }, kBytes);
        const Rate cp = time_rate([&] { launch_bw_copy(src, dst, n, grid, 0); }, 2.0 * kBytes);
        const Rate mc = time_rate([&] { CLLM_CUDA(cudaMemcpyAsync(dst, src, kBytes, cudaMemcpyDeviceToDevice, 0)); }, 2.0 * kBytes);
        const Rate bk = time_rate([&] { launch_bw_bulk_read(src, kBytes, sink, err, 0); }, kBytes);
        // Bulk copies through a decode-step-like ring (12 stages per SM, per-stage producer lanes, consumers
        // releasing stages at once) from a 48 MiB buffer that stays resident in L2, re-read 16 times per launch:
        // the rate at which the weight ring can refill from L2-prefetched data.
        const double l2_moved = static_cast<double>(16 * (kL2Bytes / bulk_probe_chunk_bytes()) / num_sms()) * num_sms() *
                                bulk_probe_chunk_bytes();  // what launch_bw_bulk_ring reports it moves
        const Rate bl2 = time_rate([&] { launch_bw_bulk_ring(src, kL2Bytes, 16, sink, err, 0); }, l2_moved);
        unsigned gave_up = 0;
        CLLM_CUDA(cudaMemcpy(&gave_up, err, sizeof(unsigned), cudaMemcpyDeviceToHost));
        if (gave_up) throw StateError("bulk read probe: a bounded wait gave up");
        std::printf("gpu: %s  grid=%d x 256\n", prop.name, grid);
        std::printf("read   best %.1f GB/s  median %.1f GB/s\n", rd.best, rd.median);
        std::printf("write  best %.1f GB/s  median %.1f GB/s\n", wr.best, wr.median);
        std::printf("copy   best %.1f GB/s  median %.1f GB/s (read+write)\n", cp.best, cp.median);
        std::printf("memcpy best %.1f GB/s (read+write)\n", mc.best);
        std::printf("bulk   best %.1f GB/s  median %.1f GB/s (1-D bulk copies to shared memory)\n", bk.best, bk.median);
        std::printf("bulk from L2 best %.1f GB/s  median %.1f GB/s (48 MiB buffer resident in L2)\n", bl2.best, bl2.median);
        if (opt.given("json")) {
            JsonValue j = JsonValue::object();
            j["tool"] = "cudallm_bandwidth";
            j["read_gbps_best"] = rd.best;
            j["read_gbps_median"] = rd.median;
            j["write_gbps_best"] = wr.best;
            j["write_gbps_median"] = wr.median;
            j["copy_gbps_best"] = cp.best;
            j["copy_gbps_median"] = cp.median;
            j["memcpy_d2d_gbps_best"] = mc.best;
            j["bulk_read_gbps_best"] = bk.best;
            j["bulk_read_gbps_median"] = bk.median;
            j["bulk_read_l2_gbps_best"] = bl2.best;
            j["bulk_read_l2_gbps_median"] = bl2.median;
            j["bytes"] = static_cast<unsigned long long>(kBytes);
            j["gpu_name"] = prop.name;
            if (!j.write_file(opt.str("json"))) throw std::runtime_error("cannot write " + opt.str("json"));
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "cudallm_bandwidth: %s\n", e.what());
        status = 1;
    }
    cudaFree(src);
    cudaFree(dst);
    cudaFree(sink);
    cudaFree(err);
    return status;
}
