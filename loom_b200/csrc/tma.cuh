// tma.cuh -- bulk asynchronous copies (TMA, cp.async.bulk) into shared memory
// with an mbarrier transaction count, and a bounded wait on it.
#pragma once
#include <stdint.h>

namespace loom {

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// init without the fence: the caller issues one fence.mbarrier_init after several
__device__ __forceinline__ void mbar_init_nf(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// global -> this CTA's shared memory, `bytes` a multiple of 16, both addresses 16-byte aligned
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Wait for phase `parity` of the barrier; gives up after `max_polls` polls and
// returns false (the caller records the failure and carries on: no trap, no
// endless spin).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t max_polls) {
    for (uint32_t i = 0; i < max_polls; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// As mbar_wait, with a suspend-time hint: a waiting thread sleeps until the
// phase completes or about `ns` nanoseconds pass, instead of re-polling (a
// polling warp takes issue slots from the warps doing the work).
__device__ __forceinline__ bool mbar_wait_hint(uint64_t *bar, uint32_t parity, uint32_t max_polls, uint32_t ns) {
    for (uint32_t i = 0; i < max_polls; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Wait for phase `parity` with non-blocking tests (mbarrier.test_wait) and a
// short sleep between them: for barriers several warps wait on at once, where
// a suspended try_wait may not be woken promptly. Gives up after `max_polls`.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity, uint32_t max_polls) {
    for (uint32_t i = 0; i < max_polls; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        __nanosleep(20);
    }
    return false;
}

}  // namespace loom
