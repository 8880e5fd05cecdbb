// sm_100a tensor-core building blocks for the batched GEMMs: TMEM allocation, tcgen05.mma (kind::f16,
// single CTA), commits to mbarriers, TMEM loads, 2D TMA tensor loads (no multicast) and the shared-
// memory / instruction descriptors, written from the PTX ISA descriptions of these instructions.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "kernels/ptx.cuh"

namespace cudallm {

// ---- Tensor memory --------------------------------------------------------------------------------
// One warp allocates `cols` columns (a power of two >= 32) and writes the TMEM base address to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, both operands K-major bf16/f16, fp32 accumulator.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// Arrives once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane i of the warp reads TMEM lane
// base_lane + i): v[j] = column col + j.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// ---- Descriptors ----------------------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major operand tile whose rows are 128 bytes (64 bf16) stored
// with the 128-byte swizzle (as a TMA tensor load with CU_TENSOR_MAP_SWIZZLE_128B writes it): 8-row
// groups 1024 bytes apart (stride byte offset), the leading byte offset unused, descriptor version 1
// (bits 46-47), layout 2 = 128-byte swizzle (bits 61-63). The tile must start on a 1024-byte boundary;
// the K offset inside the 128-byte row is added to the start address (16-byte units).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;                 // leading byte offset (ignored for this layout)
    d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version
    d |= static_cast<uint64_t>(2u) << 61;                 // 128-byte swizzle
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, fp32 D, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4)                                     // D format: f32
           | (1u << 7)                                   // A format: bf16
           | (1u << 10)                                  // B format: bf16
           | (static_cast<uint32_t>(n >> 3) << 17)       // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);      // M / 16
}

// ---- TMA ------------------------------------------------------------------------------------------
// 2D tiled tensor load (no multicast) into shared memory, completing on `bar` (transaction bytes).
// x is the inner (contiguous) coordinate in elements; x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
        "[%4], %5;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

}  // namespace cudallm
