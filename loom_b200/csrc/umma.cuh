// umma.cuh -- 5th-generation tensor-core primitives (tcgen05, sm_100a):
// TMEM allocation, shared-memory matrix descriptors, the bf16 MMA with an f32
// accumulator in TMEM, its completion barrier, and TMEM -> register loads.
//
// Operand layout used everywhere here: "K-major, no swizzle". A tile of R rows
// (M or N) by K bf16 values is stored as [K/8 chunks][R rows][8 values]: each
// 8-row x 16-byte core matrix is 128 contiguous bytes. For the MMA step that
// covers chunks 2s and 2s+1 the descriptor has
//   start = tile + 2s * R * 16 bytes
//   leading-dimension byte offset (next K chunk)  = R * 16 bytes
//   stride-dimension byte offset (next 8 rows)    = 128 bytes.
// Field positions follow the sm_100 shared-memory descriptor: start >> 4 in
// bits [0,14), LBO >> 4 in [16,30), SBO >> 4 in [32,46), version 1 at bit 46,
// base offset 0, layout type 0 (no swizzle) in [61,64).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "tma.cuh"

namespace loom {

__device__ __forceinline__ uint64_t umma_desc_kmajor(const void *tile, uint32_t rows) {
    const uint64_t start = (smem_u32(tile) >> 4) & 0x3FFFu;
    const uint64_t lbo = ((rows * 16u) >> 4) & 0x3FFFu;
    const uint64_t sbo = (128u >> 4) & 0x3FFFu;
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46);
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, both
// K-major, f32 accumulator, M x N (bits: c_format [4,6) = 1, a_format [7,10)
// = 1, b_format [10,13) = 1, N >> 3 in [17,23), M >> 4 in [24,29)).
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// One warp, converged: allocate `ncols` TMEM columns (a power of two >= 32);
// the base address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[desc] * B[desc]^T, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The MMAs this thread issued so far arrive on *bar once they complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy writes of shared memory -> visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Warp w of the (4-warp) group reads TMEM lanes [32w, 32w+32), 16 consecutive
// 32-bit columns starting at `taddr`'s column: thread t gets lane 32w+t.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

}  // namespace loom
