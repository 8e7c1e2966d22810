// b2_tcgen05.cuh -- PTX wrappers for the 5th-generation tensor cores (tcgen05 MMA kind::i8, TMEM), 2-D TMA tile
// loads, thread-block clusters (DSMEM) and the shared-memory operand layout (K-major, SWIZZLE_128B), shared by the
// bank kernels (b2_tc.cu). Every function is inline.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "b2_epi.cuh"
#include "b2_ptx.cuh"

namespace b2 {

// ---- PTX wrappers ---------------------------------------------------------------------------------------------------
B2_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            saddr(dst)),
        "l"((uint64_t)map), "r"(saddr(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// the same with an L2 eviction-priority hint (a policy from l2_evict_first / l2_evict_normal)
B2_DEV void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
        "[%2], %5;" ::"r"(saddr(dst)),
        "l"((uint64_t)map), "r"(saddr(bar)), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}
// L2 policies: data read once per step (a decode step's weights) goes first, so that what is reused (code, tables,
// activations, recent keys) stays
B2_DEV uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
B2_DEV uint64_t l2_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
B2_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
B2_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
B2_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
B2_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row core groups 1024 bytes apart (sm100 version 1)
B2_DEV uint64_t sdesc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset
    d |= (uint64_t)1 << 46;                 // descriptor version
    d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
    return d;
}
B2_DEV void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
B2_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar)) : "memory");
}
B2_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
B2_DEV void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
B2_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// cluster helpers
B2_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

constexpr int BN = 64;                               // rows per MMA (the MMA's N)
constexpr int A_BYTES = 128 * 128;                   // one weight plane of a 128-byte K block
constexpr int B_BYTES = BN * 128;                    // one row plane of a K block
constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;     // 48 KB
// kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, N = 64, M = 128
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr int MAX_STAGES = 4;
constexpr int MAX_SPLIT = 8;      // portable cluster size
constexpr int MAX_KPS = 3;        // K blocks held by one split CTA

// the 16 MMAs of one K block: 4 K steps x {wh.xh -> A1, wh.xl + wl.xh -> A2, wl.xl -> A3}; the A planes at abase
// (wh, then wl A_BYTES on), the B planes at bbase (xh, then xl B_BYTES on)
B2_DEV void mma_kblock2(uint32_t abase, uint32_t bbase, uint32_t tacc, bool first) {
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        uint64_t ah = sdesc(abase + kk * 32), al = sdesc(abase + A_BYTES + kk * 32);
        uint64_t bh = sdesc(bbase + kk * 32), bl = sdesc(bbase + B_BYTES + kk * 32);
        uint32_t acc = (!first || kk) ? 1u : 0u;
        mma_i8(tacc + 0 * BN, ah, bh, IDESC, acc);
        mma_i8(tacc + 1 * BN, ah, bl, IDESC, acc);
        mma_i8(tacc + 1 * BN, al, bh, IDESC, 1);
        mma_i8(tacc + 2 * BN, al, bl, IDESC, acc);
    }
}

// 65536*A1 + 256*A2 + A3 for 16 rows from TMEM (this warp's lane quadrant, columns n0..n0+15 of each accumulator)
B2_DEV void tmem_piles16(uint32_t taddr, int64_t (&p)[16]) {
    uint32_t r1[16], r2[16], r3[16];
    tmem_ld16(taddr + 0 * BN, r1);
    tmem_ld16(taddr + 1 * BN, r2);
    tmem_ld16(taddr + 2 * BN, r3);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 16; q++)
        p[q] = (int64_t)(int32_t)r1[q] * 65536 + (int64_t)(int32_t)r2[q] * 256 + (int64_t)(int32_t)r3[q];
}

// the same for 4 rows (columns n0..n0+3 of each accumulator)
B2_DEV void tmem_piles4(uint32_t taddr, int64_t (&p)[4]) {
    uint32_t r1[4], r2[4], r3[4];
    tmem_ld4(taddr + 0 * BN, r1);
    tmem_ld4(taddr + 1 * BN, r2);
    tmem_ld4(taddr + 2 * BN, r3);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 4; q++)
        p[q] = (int64_t)(int32_t)r1[q] * 65536 + (int64_t)(int32_t)r2[q] * 256 + (int64_t)(int32_t)r3[q];
}

B2_DEV uint32_t sw128(int row, int chunk) { return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4)); }
B2_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
B2_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace b2
