// Batched decode: tensor-core GEMM and the per-row kernels around it (batch of independent sequences).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace cudallm {

constexpr int kBatchMax = 64;

enum class GemmEpilogue : int { STORE = 0, ADD = 1, SWIGLU = 2 };

// part[ks][b][j] = sum over the ks-th of ksplit even ranges of 64-column K chunks of x[b][k] * w[j][k] (fp32
// accumulation, tcgen05 tensor cores). w: [n][k] bf16 row-major; x: activation planes [2][kBatchMax][k] bf16,
// hi (x rounded to bf16) then lo (the remainder rounded to bf16), rows >= batch ignored; batch 1..64;
// k % 64 == 0, ksplit <= k / 64. err: device word, bit 0 set if a bounded wait gave up. pdl: launch with
// the programmatic-dependent-launch attribute (the weight stream starts before the previous kernel ends).
void launch_gemm_bf16(const __nv_bfloat16* w, int n, int k, const __nv_bfloat16* x, int batch, int ksplit, float* part,
                      unsigned* err, cudaStream_t stream, bool pdl = false);
int gemm_smem_bytes();
// Adds the ksplit partials in order and applies the epilogue: out[b][j] = s (STORE), out[b][j] += s
// (ADD), or, for j < n/2, silu(s[j]) * s[n/2 + j] (SWIGLU, out is [batch][n/2]); outb (may be null) gets
// the value as the next GEMM's activation planes [2][kBatchMax][n_out] (hi, lo). out may be null for STORE /
// SWIGLU when only outb is wanted.
void launch_gemm_reduce(const float* part, int ksplit, int batch, int n, GemmEpilogue ep, float* out, __nv_bfloat16* outb,
                        cudaStream_t stream, bool pdl = false);

}  // namespace cudallm
