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
// bounded waits: each gives up after a limit of wall time (%globaltimer), sets DERR_TIMEOUT and returns false.
// The limit lives beside the handle's error word (err[2..3], a uint64 in ns; 0 = WAIT_NS), so a caller can shorten it
// (b2_set_scalar "wait_ns") without rebuilding; every kernel that waits gets the handle's error word.
constexpr uint64_t WAIT_NS = 500ull * 1000 * 1000;
B2_DEV uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
B2_DEV uint64_t wait_limit(const uint32_t* err) {
    const uint64_t v = *(const volatile uint64_t*)(err + 2);
    return v ? v : WAIT_NS;
}
B2_DEV bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t* err) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = gtime(), lim = wait_limit(err);
    for (;;) {
        for (int i = 0; i < 256; i++)
            if (mbar_try_wait(bar, phase)) return true;
        if (gtime() - t0 > lim || (*(volatile uint32_t*)err & DERR_TIMEOUT)) break;
    }
    atomicOr(err, DERR_TIMEOUT);
    return false;
}
// b2_profile mode 2 (in-kernel stamps): a kernel that takes a stamp slot records when its dependent work starts (the
// first CTA out of griddepcontrol.wait); the unit of work's accumulate kernel turns consecutive starts into durations.
// Costs one atomic per CTA and leaves the launches, graph and programmatic overlap as they are.
B2_DEV void stamp_begin(uint64_t* slot) {
    if (slot && threadIdx.x == 0 && threadIdx.y == 0) atomicMin((unsigned long long*)slot, (unsigned long long)gtime());
}
// thread-block clusters: rank, barrier (all threads), another CTA's shared memory (DSMEM)
B2_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
B2_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
B2_DEV uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
B2_DEV int64_t ld_dsmem(uint32_t addr) {
    uint64_t v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(addr));
    return (int64_t)v;
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
