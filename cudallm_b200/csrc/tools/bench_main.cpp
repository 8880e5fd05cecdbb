// cudallm_bench: end-to-end batch-1 decode benchmark through the public C ABI (include/cudallm.h).
//
// Flags and JSON keys are those of wasiqnauman/cudallm src/tools/cudallm_bench.cpp:20-22,94-124 (read by
// its bench/bench_decode.py); the measurement is the same: per repetition, reset, step the prompt one
// token at a time, drain, then time `gen` decode steps that feed back the device argmax; report the
// median tok/s and bytes/token = weight bytes + KV bytes at the mean context (cudallm_bench.cpp:82-87).
// Timing here uses CUDA events recorded on the engine's own stream around the queued steps.
//
// Additions: --prompt-seed S (uniform random prompt tokens in [0, vocab) from a seeded mt19937_64) or
// --prompt-file PATH (little-endian int32 token ids) instead of the reference's fixed token formula;
// --kv fp16|bf16, --path auto|persistent|per_op, --max-seq-len.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "cudallm.h"
#include "tools/cli.h"

using cudallm::tools::JsonValue;
using cudallm::tools::Options;

namespace {

// The reference bench's prompt (cudallm_bench.cpp:24): BOS, then a fixed arithmetic sequence.
int formula_token(int i) { return i == 0 ? 128000 : (i * 7919) % 120000 + 1000; }

void ok(int rc, const char* what) {
    if (rc != CUDALLM_OK) throw std::runtime_error(std::string(what) + ": " + cudallm_last_error());
}

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": CUDA " + cudaGetErrorString(e));
}

double median(std::vector<double> v) {
    std::sort(v.begin(), v.end());
    const size_t n = v.size();
    return n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}

const char* dtype_name(int code) { return code == 1 ? "bf16" : code == 3 ? "int8" : code == 4 ? "int4" : "?"; }

}  // namespace

int main(int argc, char** argv) {
    Options opt("cudallm_bench", "--model PATH [options]");
    opt.add("model", "", "the .cudallm file")
        .add("prompt-len", "128", "prompt tokens stepped before the timed decode")
        .add("gen", "256", "timed decode steps")
        .add("reps", "5", "timed repetitions (median reported)")
        .add("warmup", "1", "untimed repetitions first")
        .add("matvec", "opt", "opt|naive")
        .add("attn", "opt", "opt|naive")
        .add("fuse", "1", "0|1")
        .add("graph", "1", "0|1")
        .add("rpb", "0", "0 (default) or 1, 2, 4, 8")
        .add("max-seq-len", "0", "0 = the file's")
        .add("kv", "fp16", "fp16|bf16 KV cache")
        .add("path", "auto", "auto|persistent|per_op")
        .add("prompt-seed", "", "random prompt from this seed instead of the reference formula")
        .add("prompt-file", "", "prompt token ids (int32) from this file")
        .add("json", "", "write the result here");
    opt.parse(argc, argv);
    if (!opt.given("model")) opt.die("--model is required");
    const int prompt_len = static_cast<int>(opt.integer("prompt-len"));
    const int gen = static_cast<int>(opt.integer("gen"));
    const int reps = static_cast<int>(opt.integer("reps"));
    const int warmup = static_cast<int>(opt.integer("warmup"));
    if (prompt_len < 1) opt.die("--prompt-len must be >= 1");
    if (gen < 1 || reps < 1 || warmup < 0) opt.die("--gen and --reps must be >= 1, --warmup >= 0");
    const std::string matvec = opt.choice("matvec", {"opt", "naive"});
    const std::string attn = opt.choice("attn", {"opt", "naive"});
    const std::string kv = opt.choice("kv", {"fp16", "bf16"});
    const std::string path_kind = opt.choice("path", {"auto", "persistent", "per_op"});

    cudallm_engine* eng = nullptr;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    int status = 0;
    try {
        cudallm_options o;
        cudallm_default_options(&o);
        o.matvec_impl = matvec == "opt";
        o.attn_impl = attn == "opt";
        o.fuse = opt.flag("fuse");
        o.cuda_graph = opt.flag("graph");
        o.matvec_rpb = static_cast<int>(opt.integer("rpb"));
        o.max_seq_len = static_cast<int>(opt.integer("max-seq-len"));
        cudallm_options_ex ex;
        cudallm_default_options_ex(&ex);
        ex.kv_dtype = kv == "bf16" ? CUDALLM_KV_BF16 : CUDALLM_KV_FP16;
        ex.path = path_kind == "persistent" ? CUDALLM_PATH_PERSISTENT : path_kind == "per_op" ? CUDALLM_PATH_PER_OP : CUDALLM_PATH_AUTO;
        const std::string model = opt.str("model");
        ok(cudallm_create_ex(model.c_str(), &o, &ex, &eng), "cudallm_create");
        cudallm_config_info c;
        ok(cudallm_get_config(eng, &c), "cudallm_get_config");
        if (prompt_len + gen > c.max_seq_len) throw std::runtime_error("prompt-len + gen exceeds max_seq_len");

        std::vector<int> prompt(prompt_len);
        std::string prompt_kind = "formula";
        if (opt.given("prompt-file")) {
            std::ifstream f(opt.str("prompt-file"), std::ios::binary);
            std::vector<int32_t> ids(static_cast<size_t>(prompt_len));
            if (!f.read(reinterpret_cast<char*>(ids.data()), static_cast<std::streamsize>(ids.size() * 4))) {
                throw std::runtime_error("--prompt-file holds fewer than prompt-len int32 token ids");
            }
            for (int i = 0; i < prompt_len; ++i) prompt[i] = ids[i];
            prompt_kind = "file";
        } else if (opt.given("prompt-seed")) {
            std::mt19937_64 rng(static_cast<uint64_t>(opt.integer("prompt-seed")));
            std::uniform_int_distribution<int> tok(0, c.vocab - 1);
            for (int& t : prompt) t = tok(rng);
            prompt_kind = "seed " + opt.str("prompt-seed");
        } else {
            for (int i = 0; i < prompt_len; ++i) prompt[i] = formula_token(i);
        }

        auto* stream = static_cast<cudaStream_t>(cudallm_engine_stream(eng));
        cuda_ok(cudaEventCreate(&t0), "cudaEventCreate");
        cuda_ok(cudaEventCreate(&t1), "cudaEventCreate");
        std::vector<double> tok_s, ms_tok;
        for (int r = 0; r < warmup + reps; ++r) {
            ok(cudallm_reset(eng), "cudallm_reset");
            for (int t : prompt) ok(cudallm_step(eng, t, nullptr, nullptr), "cudallm_step");
            ok(cudallm_synchronize(eng), "cudallm_synchronize");
            cuda_ok(cudaEventRecord(t0, stream), "cudaEventRecord");
            for (int i = 0; i < gen; ++i) ok(cudallm_step(eng, -1, nullptr, nullptr), "cudallm_step");
            cuda_ok(cudaEventRecord(t1, stream), "cudaEventRecord");
            ok(cudallm_synchronize(eng), "cudallm_synchronize");
            float ms = 0.f;
            cuda_ok(cudaEventElapsedTime(&ms, t0, t1), "cudaEventElapsedTime");
            if (r >= warmup) {
                tok_s.push_back(gen / (ms / 1e3));
                ms_tok.push_back(ms / gen);
            }
        }
        const unsigned long long weight_bytes = c.weight_bytes;
        const unsigned long long kv_bytes = static_cast<unsigned long long>(c.n_layers) * 2 * c.n_kv_heads * c.head_dim * 2 *
                                            (static_cast<unsigned long long>(prompt_len) + (gen + 1) / 2);
        const unsigned long long bytes = weight_bytes + kv_bytes;
        const double tps = median(tok_s);
        const double gbps = static_cast<double>(bytes) * tps / 1e9;
        const int decode_path = cudallm_engine_path(eng);
        cudaDeviceProp prop{};
        cuda_ok(cudaGetDeviceProperties(&prop, cudallm_engine_device(eng)), "cudaGetDeviceProperties");
        std::printf("%s %s matvec=%s attn=%s fuse=%d graph=%d rpb=%d prompt=%d gen=%d: %.2f tok/s (median of %d), "
                    "%.3f ms/token, %.1f GB/s [%s path, %s KV]\n",
                    model.c_str(), dtype_name(c.weight_dtype), matvec.c_str(), attn.c_str(), o.fuse, o.cuda_graph,
                    o.matvec_rpb, prompt_len, gen, tps, reps, median(ms_tok), gbps,
                    decode_path == CUDALLM_PATH_PERSISTENT ? "persistent" : "per-op", kv.c_str());
        if (opt.given("json")) {
            JsonValue j = JsonValue::object();
            j["tool"] = "cudallm_bench";
            j["model"] = model;
            j["weight_dtype"] = dtype_name(c.weight_dtype);
            JsonValue& op = j["options"] = JsonValue::object();
            op["matvec"] = matvec;
            op["attn"] = attn;
            op["fuse"] = o.fuse != 0;
            op["graph"] = o.cuda_graph != 0;
            op["rpb"] = o.matvec_rpb;
            op["kv"] = kv;
            op["path"] = decode_path == CUDALLM_PATH_PERSISTENT ? "persistent" : "per_op";
            j["prompt_len"] = prompt_len;
            j["prompt"] = prompt_kind;
            j["gen"] = gen;
            j["reps"] = reps;
            JsonValue& arr = j["decode_tok_s"] = JsonValue::array();
            for (double v : tok_s) arr.push(v);
            j["decode_tok_s_median"] = tps;
            j["ms_per_token_median"] = median(ms_tok);
            j["weight_bytes"] = weight_bytes;
            j["kv_bytes_per_token_avg"] = kv_bytes;
            j["bytes_per_token"] = bytes;
            j["achieved_gbps_median"] = gbps;
            j["max_seq_len"] = c.max_seq_len;
            j["gpu_name"] = prop.name;
            if (!j.write_file(opt.str("json"))) throw std::runtime_error("cannot write " + opt.str("json"));
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "cudallm_bench: %s\n", e.what());
        status = 1;
    }
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    cudallm_destroy(eng);
    return status;
}
