// cudallm_kernelbench: per-kernel microbenchmarks of the per-operation path. Flags and JSON keys are those
// of wasiqnauman/cudallm src/tools/cudallm_kernelbench.cpp:21-27,174-300 (its bench/sweep_matvec.py runs
// `--op shapes` per weight type and rpb and reads weighted_us).
//
//   --op matvec    one weight matvec (the streaming tile kernel, or the naive one)
//   --op shapes    the five Llama-3.2-1B projections with the fused engine's epilogues;
//                  weighted_us = 16 * (qkv + wo + gate_up + down) + lm_head
//   --op attention split-K (opt) or one-block-per-head (naive) decode attention at --ctx
//
// Timing: 20 untimed launches, then --iters launches each bracketed by CUDA events; the median in us.
// On B200 every projection but the lm_head fits in the 126 MB L2, and so do the KV caches of short
// contexts; back-to-back launches on one buffer would time L2, not HBM. So the launches rotate over enough
// copies of the operands to exceed 256 MiB (--rotate 0 turns this off), and GB/s counts the weight bytes.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "common/check.h"
#include "kernels/kernels.h"
#include "tools/cli.h"

using cudallm::tools::JsonValue;
using cudallm::tools::Options;
using namespace cudallm;

namespace {

constexpr int kUntimed = 20;
constexpr size_t kRotateBytes = size_t{256} << 20;
constexpr int kNh = 32, kNkv = 8, kHd = 64;

struct DeviceBlock {
    void* p = nullptr;
    explicit DeviceBlock(size_t bytes) { CLLM_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 16))); }
    ~DeviceBlock() { cudaFree(p); }
    DeviceBlock(const DeviceBlock&) = delete;
    DeviceBlock& operator=(const DeviceBlock&) = delete;
    template <typename T>
    T* at(size_t byte_off = 0) const {
        return reinterpret_cast<T*>(static_cast<uint8_t*>(p) + byte_off);
    }
};

int copies_for(size_t bytes_per_copy, bool rotate) {
    if (!rotate || bytes_per_copy == 0) return 1;
    return static_cast<int>(std::min<size_t>(64, std::max<size_t>(1, (kRotateBytes + bytes_per_copy - 1) / bytes_per_copy)));
}

double median_us(const std::function<void(int)>& launch, int iters) {
    for (int i = 0; i < kUntimed; ++i) launch(i);
    CLLM_CUDA(cudaDeviceSynchronize());
    cudaEvent_t a, b;
    CLLM_CUDA(cudaEventCreate(&a));
    CLLM_CUDA(cudaEventCreate(&b));
    std::vector<double> us;
    for (int i = 0; i < iters; ++i) {
        CLLM_CUDA(cudaEventRecord(a, 0));
        launch(kUntimed + i);
        CLLM_CUDA(cudaEventRecord(b, 0));
        CLLM_CUDA(cudaEventSynchronize(b));
        float ms = 0.f;
        CLLM_CUDA(cudaEventElapsedTime(&ms, a, b));
        us.push_back(ms * 1e3);
    }
    CLLM_CUDA(cudaEventDestroy(a));
    CLLM_CUDA(cudaEventDestroy(b));
    check_kernel_error();
    std::sort(us.begin(), us.end());
    return iters % 2 ? us[iters / 2] : 0.5 * (us[iters / 2 - 1] + us[iters / 2]);
}

const char* wname(WeightType w) { return to_string(w); }
const char* ename(Epilogue e) { return e == Epilogue::STORE ? "store" : e == Epilogue::ADD ? "add" : "swiglu"; }

struct MatvecRun {
    std::string name;
    int rows, cols;
    bool opt;
    WeightType wt;
    Epilogue ep;
    bool fuse_norm;
    int rpb;
    int copies;
    double us, gbps;
    unsigned long long bytes;
};

// Random operands (fixed seed) for one shape, `copies` copies of the weights and scales.
MatvecRun run_matvec(const std::string& name, bool opt, WeightType wt, Epilogue ep, bool fuse_norm, int rpb, int rows, int cols,
                     int iters, bool rotate) {
    std::mt19937_64 rng(20240917);
    const size_t w_bytes = static_cast<size_t>(rows) * row_bytes(wt, static_cast<uint64_t>(cols));
    const size_t s_bytes = wt == WeightType::INT8 ? sizeof(float) * rows
                           : wt == WeightType::INT4 ? sizeof(__half) * static_cast<size_t>(rows) * (cols / 128) : 0;
    std::vector<uint8_t> w(w_bytes), s(s_bytes);
    if (wt == WeightType::BF16) {
        std::normal_distribution<float> d(0.f, 0.02f);
        for (size_t i = 0; i < w_bytes / 2; ++i) {
            const float f = d(rng);
            uint32_t u;
            std::memcpy(&u, &f, 4);
            const uint16_t h = static_cast<uint16_t>(u >> 16);
            std::memcpy(&w[2 * i], &h, 2);
        }
    } else {
        std::uniform_int_distribution<int> byte(0, 255);
        for (auto& b : w) b = static_cast<uint8_t>(byte(rng));
        if (wt == WeightType::INT8) {
            std::uniform_real_distribution<float> d(0.004f, 0.012f);
            for (size_t r = 0; r < static_cast<size_t>(rows); ++r) {
                const float f = d(rng);
                std::memcpy(&s[4 * r], &f, 4);
            }
        } else {
            std::uniform_real_distribution<float> d(0.001f, 0.004f);
            for (size_t i = 0; i < s_bytes / 2; ++i) {
                const __half h = __float2half(d(rng));
                std::memcpy(&s[2 * i], &h, 2);
            }
        }
    }
    std::vector<float> x(cols), g(cols);
    std::normal_distribution<float> xd(0.f, 1.f);
    std::uniform_real_distribution<float> gd(0.5f, 1.5f);
    for (auto& v : x) v = xd(rng);
    for (auto& v : g) v = gd(rng);
    const int outs = ep == Epilogue::SWIGLU ? rows / 2 : rows;
    const int copies = copies_for(w_bytes + s_bytes, rotate);
    const size_t wpad = (w_bytes + 255) / 256 * 256, spad = (s_bytes + 255) / 256 * 256;
    DeviceBlock dw(wpad * copies), ds(spad * copies), dx(sizeof(float) * cols), dg(sizeof(float) * cols), dy(sizeof(float) * outs);
    for (int c = 0; c < copies; ++c) {
        CLLM_CUDA(cudaMemcpy(dw.at<uint8_t>(wpad * c), w.data(), w_bytes, cudaMemcpyHostToDevice));
        if (s_bytes) CLLM_CUDA(cudaMemcpy(ds.at<uint8_t>(spad * c), s.data(), s_bytes, cudaMemcpyHostToDevice));
    }
    CLLM_CUDA(cudaMemcpy(dx.p, x.data(), sizeof(float) * cols, cudaMemcpyHostToDevice));
    CLLM_CUDA(cudaMemcpy(dg.p, g.data(), sizeof(float) * cols, cudaMemcpyHostToDevice));
    CLLM_CUDA(cudaMemset(dy.p, 0, sizeof(float) * outs));
    const double us = median_us(
        [&](int i) {
            const int c = i % copies;
            MatvecArgs a;
            a.w = dw.at<uint8_t>(wpad * c);
            a.scales = s_bytes ? ds.at<uint8_t>(spad * c) : nullptr;
            a.x = dx.at<float>();
            a.norm_w = fuse_norm ? dg.at<float>() : nullptr;
            a.eps = 1e-5f;
            a.y = dy.at<float>();
            a.rows = rows;
            a.cols = cols;
            if (opt) {
                launch_matvec_stream(wt, ep, fuse_norm, a, rpb, 0);
            } else {
                launch_matvec_naive(a, 0);
            }
        },
        iters);
    const unsigned long long bytes = w_bytes + s_bytes;
    return {name, rows, cols, opt, wt, ep, fuse_norm, rpb, copies, us, bytes / (us * 1e-6) / 1e9, bytes};
}

void report(const MatvecRun& r, JsonValue& arr) {
    std::printf("%-8s %6d x %-5d %-5s %-4s %-6s fuse_norm=%d rpb=%d: %10.2f us  %7.1f GB/s  (%d copies)\n", r.name.c_str(), r.rows,
                r.cols, r.opt ? "opt" : "naive", wname(r.wt), ename(r.ep), r.fuse_norm ? 1 : 0, r.rpb, r.us, r.gbps, r.copies);
    JsonValue& o = arr.push(JsonValue::object());
    o["name"] = r.name;
    o["rows"] = r.rows;
    o["cols"] = r.cols;
    o["impl"] = r.opt ? "opt" : "naive";
    o["wtype"] = wname(r.wt);
    o["epilogue"] = ename(r.ep);
    o["fuse_norm"] = r.fuse_norm;
    o["rpb"] = r.rpb;
    o["bytes"] = r.bytes;
    o["median_us"] = r.us;
    o["gbps"] = r.gbps;
    o["copies"] = r.copies;
}

double run_attention(bool opt, int ctx, int max_seq, int iters, bool rotate) {
    std::mt19937_64 rng(777);
    std::normal_distribution<float> d(0.f, 1.f);
    const size_t cache_n = static_cast<size_t>(kNkv) * max_seq * kHd;
    std::vector<float> q(kNh * kHd);
    std::vector<__half> kv(2 * cache_n);
    for (auto& e : q) e = d(rng);
    for (auto& e : kv) e = __float2half(d(rng));
    const size_t kv_bytes = 2 * cache_n * sizeof(__half);
    const int copies = copies_for(static_cast<size_t>(ctx) * kNkv * kHd * 4, rotate);
    const size_t slots = static_cast<size_t>(max_seq) / kAttnTile;
    DeviceBlock dkv(kv_bytes * copies), dq(sizeof(float) * q.size()), dpos(sizeof(int)), dout(sizeof(float) * kNh * kHd),
        dpo(sizeof(float) * kNh * slots * kHd), dpm(sizeof(float) * kNh * slots * 2);
    for (int c = 0; c < copies; ++c) CLLM_CUDA(cudaMemcpy(dkv.at<uint8_t>(kv_bytes * c), kv.data(), kv_bytes, cudaMemcpyHostToDevice));
    CLLM_CUDA(cudaMemcpy(dq.p, q.data(), sizeof(float) * q.size(), cudaMemcpyHostToDevice));
    const int pos = ctx - 1;
    CLLM_CUDA(cudaMemcpy(dpos.p, &pos, sizeof(int), cudaMemcpyHostToDevice));
    return median_us(
        [&](int i) {
            const __half* k = dkv.at<__half>(kv_bytes * (i % copies));
            const __half* v = k + cache_n;
            if (opt) {
                launch_attention_split<__half>(dq.at<float>(), k, v, dpos.at<int>(), dpo.at<float>(), dpm.at<float>(), dout.at<float>(),
                                               kNh, kNkv, kHd, max_seq, 0);
            } else {
                launch_attention_naive<__half>(dq.at<float>(), k, v, dpos.at<int>(), dout.at<float>(), kNh, kNkv, kHd, max_seq, 0);
            }
        },
        iters);
}

}  // namespace

int main(int argc, char** argv) {
    Options opt("cudallm_kernelbench", "--op matvec|shapes|attention [options]");
    opt.add("op", "", "matvec | shapes | attention")
        .add("wtype", "bf16", "bf16|int8|int4")
        .add("rows", "", "matvec rows")
        .add("cols", "", "matvec cols")
        .add("rpb", "0", "rows per consumer tile (0 = default, else 1, 2, 4, 8)")
        .add("epilogue", "store", "store|add|swiglu")
        .add("fuse-norm", "0", "0|1")
        .add("impl", "opt", "opt|naive")
        .add("iters", "200", "timed launches")
        .add("ctx", "", "attention context length")
        .add("max-seq", "4096", "attention cache length (a multiple of 128)")
        .add("rotate", "1", "rotate over operand copies larger than L2 (0|1)")
        .add("json", "", "write the result here");
    opt.parse(argc, argv);
    const std::string op = opt.choice("op", {"matvec", "shapes", "attention"});
    const int iters = static_cast<int>(opt.integer("iters"));
    if (iters < 1) opt.die("--iters must be >= 1");
    const bool rotate = opt.flag("rotate");
    const std::string impl = opt.choice("impl", {"opt", "naive"});
    // Every argument is checked before the first CUDA call.
    int ctx = 0, max_seq = 0, rpb = 0, rows = 0, cols = 0;
    bool fuse_norm = false;
    WeightType wt = WeightType::BF16;
    Epilogue ep = Epilogue::STORE;
    std::string wname_arg;
    if (op == "attention") {
        if (!opt.given("ctx")) opt.die("--ctx is required for --op attention");
        ctx = static_cast<int>(opt.integer("ctx"));
        max_seq = static_cast<int>(opt.integer("max-seq"));
        if (max_seq < 128 || max_seq % 128 != 0) opt.die("--max-seq must be a positive multiple of 128");
        if (ctx < 1 || ctx > max_seq) opt.die("--ctx must be in [1, max-seq]");
    } else {
        wname_arg = opt.choice("wtype", {"bf16", "int8", "int4"});
        wt = wname_arg == "bf16" ? WeightType::BF16 : wname_arg == "int8" ? WeightType::INT8 : WeightType::INT4;
        rpb = static_cast<int>(opt.integer("rpb"));
        if (rpb != 0 && rpb != 1 && rpb != 2 && rpb != 4 && rpb != 8) opt.die("--rpb must be 0, 1, 2, 4 or 8");
        if (impl == "naive" && wt != WeightType::BF16) opt.die("--impl naive needs --wtype bf16");
        if (op == "matvec") {
            if (!opt.given("rows") || !opt.given("cols")) opt.die("--rows and --cols are required for --op matvec");
            rows = static_cast<int>(opt.integer("rows"));
            cols = static_cast<int>(opt.integer("cols"));
            if (rows < 1 || cols < 1) opt.die("--rows and --cols must be positive");
            const std::string e = opt.choice("epilogue", {"store", "add", "swiglu"});
            ep = e == "store" ? Epilogue::STORE : e == "add" ? Epilogue::ADD : Epilogue::SWIGLU;
            fuse_norm = opt.flag("fuse-norm");
            if (impl == "naive" && (ep != Epilogue::STORE || fuse_norm)) opt.die("--impl naive has no epilogue or fused norm");
        }
    }
    int status = 0;
    try {
        int dev = 0;
        CLLM_CUDA(cudaGetDevice(&dev));
        cudaDeviceProp prop{};
        CLLM_CUDA(cudaGetDeviceProperties(&prop, dev));
        JsonValue j = JsonValue::object();
        j["tool"] = "cudallm_kernelbench";
        j["op"] = op;
        j["gpu_name"] = prop.name;
        j["iters"] = iters;
        j["rotate"] = rotate;
        j["impl"] = impl;
        if (op == "attention") {
            const double us = run_attention(impl == "opt", ctx, max_seq, iters, rotate);
            std::printf("attention %-5s ctx=%d: %.2f us\n", impl.c_str(), ctx, us);
            j["ctx"] = ctx;
            j["max_seq"] = max_seq;
            j["median_us"] = us;
        } else {
            j["wtype"] = wname_arg;
            j["rpb"] = rpb;
            JsonValue& results = j["results"] = JsonValue::array();
            if (op == "matvec") {
                report(run_matvec("matvec", impl == "opt", wt, ep, fuse_norm, rpb, rows, cols, iters, rotate), results);
            } else {
                struct Shape {
                    const char* name;
                    int rows, cols;
                    Epilogue ep;
                    bool norm;
                };
                const Shape shapes[] = {{"qkv", 3072, 2048, Epilogue::STORE, true},
                                        {"wo", 2048, 2048, Epilogue::ADD, false},
                                        {"gate_up", 16384, 2048, Epilogue::SWIGLU, true},
                                        {"down", 2048, 8192, Epilogue::ADD, false},
                                        {"lm_head", 128256, 2048, Epilogue::STORE, true}};
                double us[5];
                for (int i = 0; i < 5; ++i) {
                    const Shape& s = shapes[i];
                    const bool o = impl == "opt";  // the naive kernel: STORE, no fused norm
                    const MatvecRun r = run_matvec(s.name, o, wt, o ? s.ep : Epilogue::STORE, o && s.norm, rpb, s.rows, s.cols, iters, rotate);
                    report(r, results);
                    us[i] = r.us;
                }
                const double weighted = 16.0 * (us[0] + us[1] + us[2] + us[3]) + us[4];
                std::printf("weighted_us = 16*(qkv+wo+gate_up+down) + lm_head = %.2f\n", weighted);
                j["weighted_us"] = weighted;
            }
        }
        if (opt.given("json") && !j.write_file(opt.str("json"))) throw std::runtime_error("cannot write " + opt.str("json"));
    } catch (const std::exception& e) {
        std::fprintf(stderr, "cudallm_kernelbench: %s\n", e.what());
        status = 1;
    }
    return status;
}
