// Split-K decode attention for callers that cannot allocate device memory.
//
// Some callers of this library must not call cudaMalloc: code running inside a CUDA graph capture that
// forbids allocation, real-time loops that must not touch the driver's allocator, or hosts whose
// device memory is owned and pooled by another runtime. cudallm_kernel_attention allocates its
// buffers (and its split-K partials) on every call, so it is unusable there. This entry point runs the
// same kernels on buffers the caller already owns (device pointers) and keeps the partial results
// in a file-scope device array instead of allocated scratch.
//
// The scratch array g_attn_scratch holds the split-K partials (o, m, l) of at most kMaxHeads query
// heads x kMaxSeq cached positions and the position word the kernels read. Every GPU that loads the
// library holds it (1.03 MiB) until the process exits. All calls on a device share it and it keeps
// the last call's contents, so calls whose GPU work overlaps (different streams, or host threads)
// race; serialise them on one stream. Nothing in it has to start at zero: every partial the kernels
// read is written earlier in the same call, and the position word is set by the call itself.
//
// In host code g_attn_scratch is only a host-side stand-in for the symbol, not a device address: the
// first call on each device (with that device current) resolves the address with
// cudaGetSymbolAddress and caches it; later calls reuse it. Because that first call performs this
// set-up, it should be made before any stream capture that includes the entry point.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <exception>
#include <mutex>

#include "common/check.h"
#include "cudallm.h"
#include "kernels/kernels.h"

namespace cudallm {
int capi_report(const std::exception& ex);  // capi.cpp: sets cudallm_last_error, returns the code

namespace {

constexpr int kMaxHeads = 32;
constexpr int kMaxSeq = 8192;
constexpr int kMaxSlots = kMaxSeq / kAttnTile;
constexpr size_t kPartOFloats = static_cast<size_t>(kMaxHeads) * kMaxSlots * 64;
constexpr size_t kPartMlFloats = static_cast<size_t>(kMaxHeads) * kMaxSlots * 2;
constexpr size_t kScratchFloats = kPartOFloats + kPartMlFloats + 64;  // + the position word (own 256 B)

static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device (resolved once per device).
float* scratch_address() {
    int dev = 0;
    CLLM_CUDA(cudaGetDevice(&dev));
    CLLM_REQUIRE(dev >= 0 && dev < kMaxDevices, "cudallm_attention_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        CLLM_CUDA(cudaGetSymbolAddress(&ptr, g_attn_scratch));
        g_scratch_ptr[dev] = static_cast<float*>(ptr);
    }
    return g_scratch_ptr[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace cudallm

extern "C" int cudallm_attention_noalloc(const float* q, const unsigned short* k_cache, const unsigned short* v_cache, int ctx,
                                         float* out, int nh, int nkv, int hd, int max_seq, void* stream) {
    using namespace cudallm;
    try {
        CLLM_REQUIRE(q && k_cache && v_cache && out, "cudallm_attention_noalloc: null argument");
        CLLM_REQUIRE(nh > 0 && nkv > 0 && nh == 4 * nkv && hd == 64,
                     "cudallm_attention_noalloc: needs nh == 4*nkv and hd == 64");
        CLLM_REQUIRE(max_seq > 0 && max_seq % kAttnAbiChunk == 0, "cudallm_attention_noalloc: max_seq must be a multiple of 128");
        CLLM_REQUIRE(ctx >= 1 && ctx <= max_seq, "cudallm_attention_noalloc: ctx must be in [1, max_seq]");
        CLLM_REQUIRE(nh <= kMaxHeads && max_seq <= kMaxSeq,
                     "cudallm_attention_noalloc: at most 32 query heads and max_seq 8192 (fixed scratch of 1.03 MiB)");
        CLLM_REQUIRE(aligned16(k_cache) && aligned16(v_cache), "cudallm_attention_noalloc: caches must be 16-byte aligned");
        float* scratch = scratch_address();
        const size_t slots = static_cast<size_t>(max_seq) / kAttnTile;
        float* part_o = scratch;
        float* part_ml = scratch + static_cast<size_t>(nh) * slots * 64;
        int* d_pos = reinterpret_cast<int*>(scratch + kPartOFloats + kPartMlFloats);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        launch_set_token(d_pos, ctx - 1, s);  // the kernels read the context length from the device
        launch_attention_split<__half>(q, reinterpret_cast<const __half*>(k_cache), reinterpret_cast<const __half*>(v_cache),
                                       d_pos, part_o, part_ml, out, nh, nkv, hd, max_seq, s);
        return CUDALLM_OK;
    } catch (const std::exception& ex) {
        return capi_report(ex);
    }
}
