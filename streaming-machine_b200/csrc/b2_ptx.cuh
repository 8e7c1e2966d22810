// b2_ptx.cuh -- the few PTX wrappers the kernels share: mbarriers with bounded waits, 1-D bulk async copies.
#pragma once
#include <stdint.h>
#include "b2_epi.cuh"

namespace b2 {

B2_DEV uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

B2_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
B2_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
B2_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
B2_DEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// bounded wait: gives up after WAIT_NS of wall time (%globaltimer), sets DERR_TIMEOUT and returns false
constexpr uint64_t WAIT_NS = 500ull * 1000 * 1000;
B2_DEV uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
B2_DEV bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t* err) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = gtime();
    for (;;) {
        for (int i = 0; i < 256; i++)
            if (mbar_try_wait(bar, phase)) return true;
        if (gtime() - t0 > WAIT_NS || (*(volatile uint32_t*)err & DERR_TIMEOUT)) break;
    }
    atomicOr(err, DERR_TIMEOUT);
    return false;
}
// bring `bytes` of global memory into L2 (no shared memory, no completion; address 16-byte aligned, bytes % 16 == 0)
B2_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((uint64_t)src), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> shared, completing on an mbarrier (both addresses 16-byte aligned, bytes % 16 == 0)
B2_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
                 "l"((uint64_t)src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}

}  // namespace b2
