// Top-k / top-p sampling of the next token from the lm_head logits, fused into the persistent decode
// step (the reference decodes greedily only: wasiqnauman/cudallm src/kernels/argmax.cu). Every CTA selects
// the top kMaxTopK of its own vocabulary rows; the last CTA through the lm_head selects the top k of those
// candidates, applies the temperature and the nucleus (top-p) cut and draws with a counter-based random
// number (seed, position), so a given (seed, position, logits) always yields the same token.
//
// Order: candidates are ranked by the 64-bit key (order-preserving bits of the logit) << 32 | ~index, i.e.
// by logit, then lowest index first on ties (the reference argmax's tie rule), which makes the top-k set
// unique. Selection is a most-significant-digit radix select over those keys (8 passes of 8 bits,
// histograms in shared memory), after which the k winners are placed by rank.
#pragma once

#include <cstdint>
#include <cstring>

namespace cudallm {

constexpr int kMaxTopK = 64;

// Order-preserving map of an fp32 value to an unsigned key (larger value -> larger key).
__host__ __device__ __forceinline__ uint32_t float_order_key(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float float_from_order_key(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    float v;
    memcpy(&v, &u, 4);
    return v;
}
__host__ __device__ __forceinline__ uint64_t candidate_key(float v, int index) {
    return (static_cast<uint64_t>(float_order_key(v)) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(index));
}
__host__ __device__ __forceinline__ float candidate_value(uint64_t key) { return float_from_order_key(static_cast<uint32_t>(key >> 32)); }
__host__ __device__ __forceinline__ int candidate_index(uint64_t key) { return static_cast<int>(~static_cast<uint32_t>(key)); }

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014): the
// draw for position pos is the finaliser of seed + (pos + 1) * golden gamma; u = top 24 bits / 2^24.
__host__ __device__ __forceinline__ float sample_uniform(unsigned long long seed, int pos) {
    uint64_t z = seed + static_cast<uint64_t>(pos + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

#ifdef __CUDACC__
// Shared-memory scratch of select_top_k.
struct TopKScratch {
    unsigned hist[256];
    unsigned count;
    uint64_t found[kMaxTopK];
};

// Writes the k largest of the n unique keys in shared memory `keys` to out[0..k) in descending order
// (out in shared memory, k <= kMaxTopK, k <= n). nthr threads with index tid; sync() is a barrier over them.
// Radix select, most significant byte first: each pass histograms the bytes of the keys that still match
// the prefix found so far, and every warp locates (redundantly, without a further barrier) the bin that
// holds the need-th largest of them. After 8 passes the prefix is the k-th largest key itself; the k keys
// >= it are gathered (in any order) and placed by rank.
template <typename Sync>
__device__ void select_top_k(const uint64_t* keys, int n, int k, uint64_t* out, TopKScratch& sc, int tid, int nthr,
                             Sync sync) {
    const int lane = tid & 31;
    uint64_t prefix = 0, mask = 0;
    unsigned need = static_cast<unsigned>(k);
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int b = tid; b < 256; b += nthr) sc.hist[b] = 0u;
        sync();
        for (int i = tid; i < n; i += nthr) {
            const uint64_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&sc.hist[(key >> shift) & 255u], 1u);
        }
        sync();
        // Lane l holds bins 8l .. 8l+7; s = count in lanes l..31 (the bins at or above 8l).
        unsigned own = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) own += sc.hist[8 * lane + j];
        unsigned s = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned t = __shfl_down_sync(0xffffffffu, s, o);
            if (lane + o < 32) s += t;
        }
        const unsigned ok = __ballot_sync(0xffffffffu, s >= need);
        const int L = 31 - __clz(static_cast<int>(ok));  // highest lane whose bins reach need (lane 0 always does)
        int bin = 0;
        unsigned above = 0;
        if (lane == L) {
            above = s - own;  // bins above lane L's
            for (int j = 7; j >= 0; --j) {
                const unsigned h = sc.hist[8 * lane + j];
                if (above + h >= need || j == 0) {
                    bin = 8 * lane + j;
                    break;
                }
                above += h;
            }
        }
        bin = __shfl_sync(0xffffffffu, bin, L);
        above = __shfl_sync(0xffffffffu, above, L);
        prefix |= static_cast<uint64_t>(bin) << shift;
        mask |= 255ull << shift;
        need -= above;
        sync();  // the histogram is cleared by the next pass
    }
    if (tid == 0) sc.count = 0u;
    sync();
    for (int i = tid; i < n; i += nthr) {
        const uint64_t key = keys[i];
        if (key >= prefix) sc.found[atomicAdd(&sc.count, 1u)] = key;
    }
    sync();
    if (tid < k) {
        const uint64_t key = sc.found[tid];
        int rank = 0;
        for (int j = 0; j < k; ++j) rank += sc.found[j] > key ? 1 : 0;
        out[rank] = key;
    }
    sync();
}

// One thread: the token drawn from the k candidates top[0..k) (descending). Weights w_i =
// exp((v_i - v_0) / temperature) accumulate in candidate order into S_i; the nucleus is candidates 0..m
// with m the first index where S_m >= top_p * S_{k-1}; the token is the first candidate i <= m with
// S_i > u * S_m.
__device__ __forceinline__ int draw_from_top_k(const uint64_t* top, int k, float temperature, float top_p, float u) {
    const float v0 = candidate_value(top[0]);
    float total = 0.f;
    for (int i = 0; i < k; ++i) total += expf((candidate_value(top[i]) - v0) / temperature);
    const float cut = top_p * total;
    float s = 0.f, s_m = 0.f;
    int m = k - 1;
    for (int i = 0; i < k; ++i) {
        s += expf((candidate_value(top[i]) - v0) / temperature);
        if (s >= cut) {
            m = i;
            s_m = s;
            break;
        }
    }
    if (s_m == 0.f) s_m = s;
    const float target = u * s_m;
    s = 0.f;
    for (int i = 0; i <= m; ++i) {
        s += expf((candidate_value(top[i]) - v0) / temperature);
        if (s > target) return candidate_index(top[i]);
    }
    return candidate_index(top[m]);
}
#endif  // __CUDACC__

}  // namespace cudallm
