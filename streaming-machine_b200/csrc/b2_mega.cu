// b2_mega.cu -- the GPT-2 decode step (<= 64 streams) as ONE persistent kernel.
//
// A decode step as separate kernels is ~126 dependent launches whose fixed costs (launch, ramp-up and drain, the
// wait on the previous grid) are several microseconds each, far more than their work. Here one launch of MEGA_CS-CTA
// thread-block clusters (one CTA per SM, as many clusters as can be resident at once) runs every phase of the step,
// with a grid-wide barrier between phases:
//   embed       each row's word and position, R = wte + wpe, the OR of |R| per row; the other OR slots cleared
//   per layer   qkv    bank (the gauge folded in) -> q16 / k16 / v of each head and the key/value append
//               arrival over each (row, head)          -> ATT and the OR of |ATT| per row
//               proj   bank                             -> R += ..., OR of |R|
//               fc     bank (the gauge) and the bend    -> HID, OR of |HID|
//               mproj  bank                             -> R += ..., OR of |R| (not after the last layer)
// The head, the race and the bookkeeping run after it as ordinary launches.
//
// A bank phase: a cluster takes tpc output tiles of 128 columns, each tile's K range split over ks CTAs (tpc x ks =
// MEGA_CS). A CTA reads its rows' slice of the producer's int64 output, to16's it with the row's shift (from the OR the
// producer published with atomicOr) into the two signed-byte planes in SWIZZLE_128B shared memory, sums S1/S2 (the
// gauge) over its slice, runs the tcgen05 MMAs against weight planes that arrived by TMA during the previous phase,
// and parks its corrected partial piles in shared memory. After a cluster barrier each CTA sums a slice of the rows
// over DSMEM and finishes them (gauge power, bias, bend, residual add, heads16), then issues the TMA loads of its part
// of the NEXT bank's weights, which land while the grid barrier and the next prologue run.
// The arrival phase: each CTA takes (row, head) units in turn, the stream's keys, values and their metadata brought
// into shared memory by bulk copies a few units ahead, scored and summed by all 8 warps.
//
// Data written inside the kernel is read with ld.global.cg (L2) only, never through the non-coherent path, and the
// key/value append is made visible to the bulk copies with a proxy fence. Every wait is bounded (0.5 s of
// %globaltimer): a timeout sets DERR_TIMEOUT, after which every barrier and wait returns at once and no new copy is
// issued, so the kernel still meets every cluster barrier, drains its own copies and MMAs, frees its TMEM and ends
// (the call reports B2_ERR_DEVICE).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <vector>

#include "b2_mega.cuh"
#include "b2_tcgen05.cuh"

namespace b2 {

namespace {

constexpr int NT = 512;                              // threads per CTA (16 warps: latency-bound code needs them)
constexpr int WST = 2 * A_BYTES;                     // weight planes of one 128-input K block: 32 KB
constexpr int XST = 2 * B_BYTES;                     // activation planes of one K block: 16 KB
constexpr int MAXKPS = 4;                            // K blocks per CTA (mproj: 24 blocks over 6 CTAs)
constexpr int ATT_BASE = WST + XST;                  // the arrival's buffers start above a 1-block bank (proj's
                                                     // weights are in flight during the arrival)
constexpr int DYN = 208 * 1024;                      // dynamic shared memory in use (after 1 KB alignment)
constexpr int MAX_SLOTS = 4;
constexpr int KEY_BYTES = 128 + 256 + 8 + 4 + 8 + 4;  // k16, v, +32768 mask, exponent, score, arrival weight
constexpr uint64_t DRAIN_NS = 20ull * 1000 * 1000;   // final drain of our own copies / MMAs after a timeout

B2_DEV uint32_t ldv(const uint32_t* p) { return *(const volatile uint32_t*)p; }
B2_DEV bool is_dead(const uint32_t* err) { return (ldv(err) & DERR_TIMEOUT) != 0; }
B2_DEV uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
B2_DEV void red_release(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B2_DEV void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
B2_DEV int64_t ldcg(const int64_t* p) { return (int64_t)__ldcg((const long long*)p); }
B2_DEV uint64_t ldcgu(const uint64_t* p) { return (uint64_t)__ldcg((const unsigned long long*)p); }
B2_DEV int32_t ldcg_i32(const int32_t* p) { return __ldcg(p); }

// profiling aid: thread 0 stamps the time of step k of phase ph
B2_DEV void stamp(const MegaArgs& a, int ph, int k) {
    if (a.trace && threadIdx.x == 0 && ph < MEGA_MAX_PHASES) {
        a.trace[((size_t)blockIdx.x * MEGA_MAX_PHASES + ph) * MEGA_STAMPS + k] = gtime();
        if (k == 0) a.trace[((size_t)blockIdx.x * MEGA_MAX_PHASES + ph) * MEGA_STAMPS + 7] = clock64();
    }
}

// bounded wait ignoring the error word: the final drain of our own copies and MMAs
B2_DEV void mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = gtime();
    while (!mbar_try_wait(bar, parity))
        if (gtime() - t0 > DRAIN_NS) return;
}

// every CTA of the grid: arrive, then wait (bounded) until all have arrived `target / gridDim` times
B2_DEV void grid_sync(uint32_t* bar, uint32_t target, uint32_t* err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release(bar, 1);
        if (!is_dead(err)) {
            const uint64_t t0 = gtime(), lim = wait_limit(err);
            while (ld_acquire(bar) < target) {
                if (gtime() - t0 > lim) { atomicOr(err, DERR_TIMEOUT); break; }
                if (is_dead(err)) break;
            }
        }
        __threadfence();
    }
    __syncthreads();
}

struct Sh {
    uint64_t wbar[MAXKPS], accbar, abar[MAX_SLOTS], rbar;
    uint32_t tmem;
    int sh[BN];
    int32_t pos[BN], slot[BN];       // the rows' positions and stream slots (fixed for the whole step)
    alignas(16) int64_t S12[BN][2];  // partial S1, S2 per row (sent to the peers as 16-byte rows)
    int64_t rowc[BN], LS[BN], e2[BN];
    uint32_t sat[BN][MAXKPS * 4];
    unsigned long long satrows;
    uint64_t hor[16][2];
    int32_t qs[MAX_SLOTS][64];
    int64_t red[2][8][66];           // the arrival: per warp group, per warp
    int nslots, slot_bytes;
};

// per-thread bookkeeping of the asynchronous work this CTA has in flight (meaningful in the thread that owns it)
struct Track {
    uint32_t warm[MAXKPS];     // tid 0: times wbar[kb] was armed
    uint32_t wwait;            // MMA thread: parity bits of the next wbar waits
    uint32_t acc;              // all threads: completed accbar phases
    uint32_t aarm[MAX_SLOTS];  // tid 0: times abar[s] was armed
    uint32_t await_;           // all threads: parity bits of the next abar waits
    uint32_t rpar;             // all threads: completed rbar phases (the reduction's incoming slices)
};

struct Unit {
    int mt, kk, g;
    bool on;
};
B2_DEV Unit unit_of(const MegaBank& bk, int cluster, int crank, int round, int nclusters) {
    Unit u;
    u.g = crank / bk.ks;
    u.kk = crank % bk.ks;
    u.mt = (round * nclusters + cluster) * bk.tpc + u.g;
    u.on = u.g < bk.tpc && u.mt < bk.ntiles;
    return u;
}
B2_DEV int rounds_of(const MegaBank& bk, int nclusters) {
    const int per = nclusters * bk.tpc;
    return (bk.ntiles + per - 1) / per;
}

// tid 0: this unit's weight planes by TMA into the bank region
B2_DEV void issue_weights(const MegaArgs& a, int bi, const MegaBank& bk, const Unit& u, uint8_t* smem, Sh& s, Track& t) {
    if (!u.on || is_dead(a.err)) return;
    const CUtensorMap* mh = reinterpret_cast<const CUtensorMap*>(a.maps[2 * bi].bytes);
    const CUtensorMap* ml = reinterpret_cast<const CUtensorMap*>(a.maps[2 * bi + 1].bytes);
    for (int kb = 0; kb < bk.kps; kb++) {
        uint8_t* st = smem + kb * WST;
        const int kx = (u.kk * bk.kps + kb) * 128;
        mbar_expect_tx(&s.wbar[kb], WST);
        t.warm[kb]++;
        tma_load_2d(st, mh, &s.wbar[kb], kx, u.mt * 128);
        tma_load_2d(st + A_BYTES, ml, &s.wbar[kb], kx, u.mt * 128);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// one bank round (see the header). X: the bank's input [rows][nin]; xor_in: its rows' OR; out: R (PLAIN_ADD) or HID
// (GAUGED_EDGE); or_out: the next bank's OR slot (may be null); HEADS: the qkv bank's heads16 + key/value append.
// `prefetched`: the weights were issued already. All CTAs of a cluster call this the same number of times.
//
// Shared memory: weights [0, kps*32K), activation planes after them; once the MMAs are done, the partial tile P
// [64 rows][128] int64 at [0, 64K), and the receive buffers RB (one slice of rows per sub-group peer) and R12 (their
// partial S1, S2) above it. The K-split reduction is pushed, not pulled: after a cluster barrier each CTA sends every
// peer the peer's slice of rows of P (one bulk copy shared::cta -> shared::cluster each, completing on the peer's
// mbarrier), then sums its own slice locally.
// ---------------------------------------------------------------------------------------------------------------------
constexpr int RB_BASE = 64 * 1024;
B2_DEV int slice_rows(int ks) { return (BN + ks - 1) / ks; }
B2_DEV int r12_base(int ks) { return RB_BASE + ks * slice_rows(ks) * 1024; }
B2_DEV void bulk_s2c(uint32_t dst_cluster, const void* src, uint32_t bytes, uint32_t bar_cluster) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
                 "r"(saddr(src)), "r"(bytes), "r"(bar_cluster)
                 : "memory");
}
// to16 of one int64 (given as its two 32-bit halves) by the row's shift (0..49, base2.py:24-27): add half, shift
B2_DEV int32_t to16v(int lo, int hi, int sh) {
    const uint64_t x = ((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo;
    return sh ? (int32_t)((int64_t)(x + (1ull << (sh - 1))) >> sh) : (int32_t)(int64_t)x;
}
B2_DEV uint32_t hbyte(int32_t x) { return (uint32_t)(uint8_t)(int8_t)(x == 32768 ? 127 : (x >> 8)); }
B2_DEV uint32_t lbyte(int32_t x) { return (uint32_t)(uint8_t)(int8_t)((x & 255) - 128); }
B2_DEV uint32_t redux_add(uint32_t v) { return __reduce_add_sync(0xffffffffu, v); }
// named barrier `id` (1..15) over `count` threads, and its AND-reduction form
B2_DEV void group_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }
B2_DEV bool group_and(int id, int count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
B2_DEV void st_shared_u16(uint32_t addr, uint32_t v) { asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"((uint16_t)v) : "memory"); }

// the bank epilogue with the mode chosen at run time (one copy of the code for every bank keeps it in the
// instruction cache): base2.py:70-71 gauged (+ the bend, :106) or :76 plain added into the residual
B2_DEV int64_t epi_rt(int epi, int64_t pile, int64_t e_j, int64_t b_j, int64_t exr, int64_t LSr, int64_t e2r,
                      const int32_t* __restrict__ PHI) {
    const int64_t es = wadd(wadd(e_j, exr), 16);
    if (epi == EPI_PLAIN_ADD) return wadd(rshift(pile, -es), b_j);
    const int64_t F = wsub(wmul(es, 65536), LSr);
    const int64_t v = wadd(rshift(wmul(pile, e2r), 16 - (F >> 16)), b_j);
    return epi == EPI_GAUGED_EDGE ? edge(v, PHI) : v;
}

struct BankIO {
    int bi, epi;
    bool heads;                  // the qkv bank: heads16 and the key/value append instead of stores
    const int64_t* X;            // the bank's input [rows][nin]
    const uint64_t* xor_in;      // its rows' OR of magnitudes
    uint64_t* or_out;            // the next bank's OR slot (null: none)
    int64_t* out;                // R (PLAIN_ADD) or HID (GAUGED_EDGE)
    int ldo;
};

__device__ __noinline__ void bank_round(const MegaArgs& a, const BankIO& io, const Unit u, bool prefetched, int layer,
                                        uint8_t* smem, Sh& s, Track& t, int ph) {
    const MegaBank& bk = a.banks[io.bi];
    const int EPI = io.epi;
    const bool HEADS = io.heads;
    const bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    const int64_t* X = io.X;
    const uint64_t* xor_in = io.xor_in;
    uint64_t* or_out = io.or_out;
    int64_t* out = io.out;
    const int ldo = io.ldo, bi = io.bi;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tmem = s.tmem;
    uint8_t* xplanes = smem + bk.kps * WST;
    int64_t* P = (int64_t*)smem;
    const int kps = bk.kps, ks = bk.ks;
    const int SR = slice_rows(ks);
    const int n0 = u.kk * BN / ks, n1 = (u.kk + 1) * BN / ks;   // my slice of rows in the reduction
    const int g0 = u.g * ks;                                     // my sub-group's first cluster rank
    int64_t* RB = (int64_t*)(smem + RB_BASE);                    // [ks][SR][128]
    int64_t* R12 = (int64_t*)(smem + r12_base(ks));              // [ks][BN][2]
    // epilogue mapping: column m, rows n0 + ro, n0 + ro + 4, ...
    const int m = tid & 127, ro = tid >> 7;
    const int j = u.mt * 128 + m;

    if (u.on) {
        if (tid == 0 && !prefetched) issue_weights(a, bi, bk, u, smem, s, t);
        uint64_t xo = 0;
        if (tid < BN && tid < a.rows) xo = ldcgu(xor_in + tid);
        if (tid < BN) {
            s.S12[tid][0] = 0;
            s.S12[tid][1] = 0;
            s.rowc[tid] = 0;
            #pragma unroll 1
            for (int w = 0; w < MAXKPS * 4; w++) s.sat[tid][w] = 0;
        }
        if (tid == 0) s.satrows = 0;
        if (tid < BN) s.sh[tid] = to16_shift(xo);
        __syncthreads();
        stamp(a, ph, 8);
        // ---- activations: warp w takes rows w, w+16, w+32, w+48; lane l values 2l, 2l+1, 64+2l, 65+2l of each K
        //      block, a row's 1 KB loaded coalesced by the whole warp; row sums by warp reduction (redux) ----
#pragma unroll 1
        for (int kb = 0; kb < kps; kb++) {
            const int kx = (u.kk * kps + kb) * 128;
            const uint32_t bh = saddr(xplanes + kb * XST), bl = bh + B_BYTES;
            int4 ra[4], rb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int n = warp + 16 * i;
                const bool nv = n < a.rows;
                const int4* src = reinterpret_cast<const int4*>(X + (size_t)n * bk.nin + kx);
                ra[i] = nv ? __ldcg(src + lane) : make_int4(0, 0, 0, 0);
                rb[i] = nv ? __ldcg(src + 32 + lane) : make_int4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int n = warp + 16 * i;
                const int sh = s.sh[n];
                const int32_t x0 = to16v(ra[i].x, ra[i].y, sh), x1 = to16v(ra[i].z, ra[i].w, sh);
                const int32_t x2 = to16v(rb[i].x, rb[i].y, sh), x3 = to16v(rb[i].z, rb[i].w, sh);
                const uint32_t o = (uint32_t)((2 * lane) & 15);
                st_shared_u16(bh + sw128(n, lane >> 3) + o, hbyte(x0) | (hbyte(x1) << 8));
                st_shared_u16(bh + sw128(n, 4 + (lane >> 3)) + o, hbyte(x2) | (hbyte(x3) << 8));
                st_shared_u16(bl + sw128(n, lane >> 3) + o, lbyte(x0) | (lbyte(x1) << 8));
                st_shared_u16(bl + sw128(n, 4 + (lane >> 3)) + o, lbyte(x2) | (lbyte(x3) << 8));
                const int sat = (x0 == 32768) + (x1 == 32768) + (x2 == 32768) + (x3 == 32768);
                if (sat) {                                         // rare: the +32768 list
                    const int32_t xs[4] = {x0, x1, x2, x3};
#pragma unroll 1
                    for (int q = 0; q < 4; q++)
                        if (xs[q] == 32768) {
                            const int kk = q < 2 ? 2 * lane + q : 64 + 2 * lane + (q - 2);
                            atomicOr(&s.sat[n][kb * 4 + (kk >> 5)], 1u << (kk & 31));
                            atomicOr(&s.satrows, 1ull << n);
                        }
                }
                // S1 (|sum| < 2^17 per lane), S2 as 16-bit halves (each lane's sum of 4 squares <= 2^32), +32768 count
                const uint64_t sq = (uint64_t)((int64_t)x0 * x0) + (uint64_t)((int64_t)x1 * x1) +
                                    (uint64_t)((int64_t)x2 * x2) + (uint64_t)((int64_t)x3 * x3);
                const int32_t t1 = (int32_t)redux_add((uint32_t)(x0 + x1 + x2 + x3));
                const uint32_t t2l = redux_add((uint32_t)(sq & 0xFFFF)), t2h = redux_add((uint32_t)(sq >> 16));
                const uint32_t tc = redux_add((uint32_t)sat);
                if (lane == 0) {                                    // one warp per row: no atomics
                    const int64_t a1 = t1, a2 = (int64_t)t2h * 65536 + (int64_t)t2l;
                    s.S12[n][0] += a1;
                    s.S12[n][1] += a2;
                    s.rowc[n] += 128 * (a1 - 256 * (int64_t)tc);
                }
            }
            if (kb == 0) stamp(a, ph, 10);
        }
        stamp(a, ph, 11);
        fence_proxy_async();
        __syncthreads();
        stamp(a, ph, 1);
        // ---- MMAs ----
        if (warp == 1 && lane == 0) {
            bool ok = true;
            #pragma unroll 1
            for (int kb = 0; kb < kps; kb++) {
                const uint32_t par = (t.wwait >> kb) & 1;
                t.wwait ^= 1u << kb;
                if (ok && !mbar_wait(&s.wbar[kb], par, a.err)) ok = false;
            }
            tc_fence_after();
            if (ok)
                #pragma unroll 1
                for (int kb = 0; kb < kps; kb++)
                    mma_kblock2(saddr(smem + kb * WST), saddr(xplanes + kb * XST), tmem, kb == 0);
            mma_commit(&s.accbar);                   // arrives once the issued MMAs (if any) are done
        }
        __syncwarp();
        if (tid == 0 && ks > 1) {                    // my incoming slices: (ks - 1) peers x (rows x 1 KB + rows x 16 B)
            mbar_expect_tx(&s.rbar, (uint32_t)((ks - 1) * (n1 - n0) * (1024 + 16)));
        }
        int64_t colc = 0;
        {
            const int jc = u.mt * 128 + (warp & 3) * 32 + lane;
#pragma unroll 1
            for (int kb = 0; kb < kps; kb++) colc += __ldg(bk.colcorr_kb + (size_t)(u.kk * kps + kb) * bk.nout_pad + jc);
        }
        // one decision for the whole CTA: the TMEM loads below are warp-aligned
        const bool ok = __syncthreads_and(mbar_wait(&s.accbar, t.acc & 1, a.err));
        t.acc++;
        tc_fence_after();
        stamp(a, ph, 2);
        // ---- corrected partial piles -> P: warp w reads TMEM lane quadrant w % 4 (columns), rows 16 (w / 4) .. +16 ----
        {
            const int mm = (warp & 3) * 32 + lane, r0 = (warp >> 2) * 16;
            int64_t p[16];
            if (ok) {
                tmem_piles16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + r0, p);
#pragma unroll
                for (int q = 0; q < 16; q++) p[q] += colc + s.rowc[r0 + q];
            } else {
#pragma unroll
                for (int q = 0; q < 16; q++) p[q] = 0;
            }
            tc_fence_before();
            __syncthreads();                         // every read of the planes and of TMEM is done
#pragma unroll
            for (int q = 0; q < 16; q++) P[(r0 + q) * 128 + mm] = p[q];
            // rare: a row with +32768 entries in this K range gets 256 * w[k][j] for each (the bank's int16 weights)
            const unsigned long long satrows = ok ? s.satrows : 0ull;
            const int jj = u.mt * 128 + mm;
            if (((satrows >> r0) & 0xffffull) && jj < bk.nout)
#pragma unroll 1
                for (int q = 0; q < 16; q++) {
                    const int n = r0 + q;
                    if (!((satrows >> n) & 1)) continue;
                    int64_t add = 0;
#pragma unroll 1
                    for (int kb = 0; kb < kps; kb++)
#pragma unroll 1
                        for (int w = 0; w < 4; w++) {
                            uint32_t bits = s.sat[n][kb * 4 + w];
                            while (bits) {
                                const int kk = w * 32 + __ffs(bits) - 1;
                                bits &= bits - 1;
                                const int i = (u.kk * kps + kb) * 128 + kk;
                                add += 256 * (int64_t)__ldg(bk.w16 + (size_t)i * bk.nout + jj);
                            }
                        }
                    P[n * 128 + mm] += add;
                }
        }
        fence_proxy_async();                         // P and S12 are read by the bulk copies below
    }
    cluster_sync();                                  // every P written; every CTA's weights and planes are dead
    stamp(a, ph, 3);
    if (u.on && ks > 1) {
        if (tid == 0) {
            const uint32_t rb_local = saddr(RB), r12_local = saddr(R12), bar_local = saddr(&s.rbar);
            #pragma unroll 1
            for (int p = 0; p < ks; p++) {
                if (p == u.kk) continue;
                const int p0 = p * BN / ks, p1 = (p + 1) * BN / ks;
                const uint32_t rk = (uint32_t)(g0 + p);
                const uint32_t dst = mapa(rb_local + (uint32_t)(u.kk * SR * 1024), rk);
                const uint32_t d12 = mapa(r12_local + (uint32_t)((u.kk * BN + p0) * 16), rk);
                const uint32_t bar = mapa(bar_local, rk);
                bulk_s2c(dst, P + (size_t)p0 * 128, (uint32_t)((p1 - p0) * 1024), bar);
                bulk_s2c(d12, &s.S12[p0][0], (uint32_t)((p1 - p0) * 16), bar);
            }
        }
        const bool got = mbar_wait(&s.rbar, t.rpar & 1, a.err);
        (void)got;
    }
    if (u.on && ks > 1) t.rpar++;
    cluster_sync();                                  // every slice arrived: every CTA's outgoing copies are done
    stamp(a, ph, 12);
    if (u.on) {
        // ---- my slice of rows: the gauge's row terms, then sum the partial piles and finish ----
        if (tid < n1 - n0) {
            const int n = n0 + tid;
            int64_t LS = 0, e2 = 0;
            if (GAUGED && n < a.rows) {
                int64_t S1 = s.S12[n][0], S2 = s.S12[n][1];
                #pragma unroll 1
                for (int p = 0; p < ks; p++)
                    if (p != u.kk) { S1 += R12[(p * BN + n) * 2]; S2 += R12[(p * BN + n) * 2 + 1]; }
                LS = gauge_LS(S1, S2, -16 + s.sh[n], a.LOG2, a.log768, a.eps40);
                e2 = __ldg(a.EXP2 + (wsub(0, LS) & 0xFFFF));
            }
            s.LS[n] = LS;
            s.e2[n] = e2;
        }
        __syncthreads();
        stamp(a, ph, 13);
        const bool jv = j < bk.nout;
        const int64_t e_j = jv ? (int64_t)__ldg(bk.e + j) : 0, b_j = jv ? __ldg(bk.b + j) : 0;
        const int nit = (n1 - n0 + 3) >> 2;          // rows per thread (n0 + ro + 4 it)
        const int H = a.kv.H, dm = H * 64;
#pragma unroll 1
        for (int it = 0; it < nit; it++) {
            const int n = n0 + 4 * it + ro;
            const bool valid = jv && n < n1 && n < a.rows;
            int64_t val = 0;
            if (valid) {
                val = P[(size_t)n * 128 + m];
#pragma unroll 1
                for (int p = 0; p < ks; p++)
                    if (p != u.kk) val = wadd(val, RB[((size_t)p * SR + (n - n0)) * 128 + m]);
                val = epi_rt(EPI, val, e_j, b_j, -16 + s.sh[n], s.LS[n], s.e2[n], a.PHI);
            }
            if (it == 0) stamp(a, ph, 14);
            if (HEADS) {
                // heads16: each 64-column half of the tile is one head part (q, k or v of one head); a row's OR over
                // the part is the OR over its two warps (w, w ^ 1)
                const uint64_t w = warp_or64(valid ? mag(val) : 0);
                if (lane == 0) s.hor[warp][it & 1] = w;
                __syncthreads();
                const uint64_t por = s.hor[warp][it & 1] | s.hor[warp ^ 1][it & 1];
                const int part = 2 * u.mt + (m >> 6), kind = part / H, hh = part % H, dd = m & 63;
                const int sh = to16_shift(por);
                const int32_t x = (int32_t)rshift(val, sh);
                if (kind == 0) {
                    if (valid) {
                        a.q16[(size_t)n * dm + hh * 64 + dd] = x;
                        if (dd == 0) a.qexp[n * H + hh] = -16 + sh;
                    }
                } else {
                    const int pos = valid ? s.pos[n] : 0;
                    const bool pv = valid && pos >= 0 && pos < a.kv.lim;
                    if (valid && !pv && dd == 0) set_err(a.err, DERR_POS);
                    const size_t idx = pv ? kv_index(s.slot[n], layer, hh, pos, a.kv.L, H, a.kv.ctx) : 0;
                    if (kind == 1) {
                        const uint32_t sat = __ballot_sync(0xffffffffu, pv && x == 32768);
                        if (pv) {
                            a.kv.k[idx * 64 + dd] = (int16_t)(uint16_t)(uint32_t)x;
                            if (lane == 0) reinterpret_cast<uint32_t*>(&a.kv.kmask[idx])[dd >> 5] = sat;
                            if (dd == 0) a.kv.kexp[idx] = -16 + sh;
                        }
                    } else if (pv) {
                        if (val != (int64_t)(int32_t)val) set_err(a.err, DERR_VOVF);
                        a.kv.v[idx * 64 + dd] = (int32_t)val;
                    }
                }
            } else {
                int64_t o = val;
                if (valid) {
                    if (EPI == EPI_PLAIN_ADD) o = wadd(ldcg(out + (size_t)n * ldo + j), o);
                    out[(size_t)n * ldo + j] = o;
                }
                const uint64_t wor = warp_or64(valid ? mag(o) : 0);
                if (lane == 0 && or_out && valid) atomicOr((unsigned long long*)&or_out[n], (unsigned long long)wor);
            }
        }
        if (HEADS) fence_async_global();             // the key/value append is read by bulk copies next phase
    }
    stamp(a, ph, 4);
    __syncthreads();
    stamp(a, ph, 5);
}

// ---------------------------------------------------------------------------------------------------------------------
// the arrival phase (base2.py:85-100; as k_attend_bulk, 8 warps per unit): unit = (row, head), units spread over the
// CTAs, each unit's stream run copied into one of `nslots` shared-memory slots up to nslots units ahead
// ---------------------------------------------------------------------------------------------------------------------
B2_DEV void att_issue(const MegaArgs& a, int layer, int unit, int slot, uint8_t* smem, Sh& s, Track& t) {
    const int r = unit / a.H, h = unit % a.H;
    const int p = s.pos[r];
    if (p < 0 || p >= a.kv.lim || is_dead(a.err)) return;
    const int nkr = (p + 1 + 3) & ~3;
    uint8_t* base_s = smem + ATT_BASE + (size_t)slot * s.slot_bytes;
    const size_t base = kv_index(s.slot[r], layer, h, 0, a.kv.L, a.kv.H, a.kv.ctx);
    fence_async_global();
    mbar_expect_tx(&s.abar[slot], (uint32_t)nkr * (128 + 256 + 8 + 4));
    t.aarm[slot]++;
    bulk_g2s(base_s, a.kv.k + base * 64, (uint32_t)nkr * 128, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 128, a.kv.v + base * 64, (uint32_t)nkr * 256, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 384, a.kv.kmask + base, (uint32_t)nkr * 8, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 392, a.kv.kexp + base, (uint32_t)nkr * 4, &s.abar[slot]);
}

__device__ __noinline__ void att_phase(const MegaArgs& a, int layer, uint64_t* or_out, uint8_t* smem, Sh& s, Track& t, int ph) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int grp = wid >> 3, gt = tid & 255, gw = wid & 7;    // two groups of 8 warps work on different units
    const int G = gridDim.x, cid = blockIdx.x;
    const int nunits = a.rows * a.H;
    const int my = cid < nunits ? (nunits - cid + G - 1) / G : 0;
    if (!my) return;
    // slots sized for the longest run among my units; each group gets half of them
    if (tid == 0) {
        int nk = 1;
#pragma unroll 1
        for (int i = 0; i < my; i++) nk = max(nk, min(s.pos[(cid + i * G) / a.H] + 1, a.kv.lim));
        const int bytes = (((nk + 3) & ~3) * KEY_BYTES + 127) & ~127;
        s.slot_bytes = bytes;
        s.nslots = max(1, min((DYN - ATT_BASE) / bytes, MAX_SLOTS));
    }
    __syncthreads();
    const int NS = s.nslots;
    const bool two = NS >= 2 && my >= 2;            // both groups at work
    const int nsg = two ? NS / 2 : NS;              // slots per group
    const int myg = two ? (my - grp + 1) / 2 : (grp == 0 ? my : 0);   // my group's units: i = grp + 2k (or all)
    const int step = two ? 2 : 1;
    if (!myg) return;                               // (group 1 when one slot is all that fits)
    const int bar_id = 1 + grp;
    if (gt == 0) {
#pragma unroll 1
        for (int k2 = 0; k2 < min(nsg, myg); k2++)
            att_issue(a, layer, cid + (grp + step * k2) * G, grp + (two ? 2 * k2 : k2), smem, s, t);
    }
    const int d = a.H * 64;
    int64_t (*red)[66] = s.red[grp];
#pragma unroll 1
    for (int k2 = 0; k2 < myg; k2++) {
        const int unit = cid + (grp + step * k2) * G;
        const int slot = grp + (two ? 2 * (k2 % nsg) : (k2 % nsg));
        const int r = unit / a.H, h = unit % a.H;
        const int p = s.pos[r];
        const bool pv = p >= 0 && p < a.kv.lim;
        const int nk = p + 1, nkr = (nk + 3) & ~3;
        uint8_t* sb = smem + ATT_BASE + (size_t)slot * s.slot_bytes;
        int16_t* Ks = reinterpret_cast<int16_t*>(sb);
        int32_t* Vs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 128);
        uint64_t* KMs = reinterpret_cast<uint64_t*>(sb + (size_t)nkr * 384);
        int32_t* KEs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 392);
        int64_t* SCs = reinterpret_cast<int64_t*>(sb + (size_t)nkr * 396);
        int32_t* AVs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 404);
        if (gt < 64) s.qs[slot][gt] = pv ? __ldcg(a.q16 + (size_t)r * d + h * 64 + gt) : 0;
        const int64_t eq = pv ? __ldcg(a.qexp + r * a.H + h) : 0;
        bool ok = pv;
        if (pv) {
            const uint32_t par = (t.await_ >> slot) & 1;
            t.await_ ^= 1u << slot;
            ok = mbar_wait(&s.abar[slot], par, a.err);
        }
        ok = group_and(bar_id, 256, ok);            // one decision for the group: the block below synchronises
        if (k2 == 0 && grp == 0) stamp(a, ph, 1);
        if (ok) {
            // pass 1: scores, 8 lanes per key
            int qr[8];
#pragma unroll
            for (int q = 0; q < 8; q++) qr[q] = s.qs[slot][(lane & 7) * 8 + q];
            int64_t lmax = INT64_MIN;
#pragma unroll 1
            for (int c = gw; c * 4 < nk; c += 8) {
                const int key = c * 4 + (lane >> 3);
                int64_t part = 0;
                if (key < nk) {
                    const int4 raw = reinterpret_cast<const int4*>(Ks + (size_t)key * 64)[lane & 7];
                    const int16_t* kk = reinterpret_cast<const int16_t*>(&raw);
#pragma unroll
                    for (int q = 0; q < 8; q++) part += (long long)qr[q] * (long long)kk[q];
                }
                part += __shfl_xor_sync(0xffffffffu, part, 1);
                part += __shfl_xor_sync(0xffffffffu, part, 2);
                part += __shfl_xor_sync(0xffffffffu, part, 4);
                if ((lane & 7) == 0 && key < nk) {
                    uint64_t mk = KMs[key];
                    while (mk) { const int q = __ffsll((long long)mk) - 1; mk &= mk - 1; part += 65536LL * s.qs[slot][q]; }
                    const int64_t sc = rshift(part, -(eq + (int64_t)KEs[key] - 3 + 10));
                    SCs[key] = sc;
                    lmax = sc > lmax ? sc : lmax;
                }
            }
            lmax = warp_max64(lmax);
            if (lane == 0) red[gw][65] = lmax;
            group_sync(bar_id, 256);
            int64_t start = red[0][65];
#pragma unroll
            for (int q = 1; q < 8; q++) start = red[q][65] > start ? red[q][65] : start;
            // pass 1b: arrival weights and their total
            int64_t z = 0;
#pragma unroll 1
            for (int q = gt; q < nk; q += 256) {
                const int64_t av = arrival(wsub(start, SCs[q]), a.ARR, a.alen, a.err);
                AVs[q] = (int32_t)av;
                z = wadd(z, av);
            }
            z = warp_sum64(z);
            group_sync(bar_id, 256);
            if (lane == 0) red[gw][64] = z;
            // pass 2: 2 dims per lane, warps split the keys
            int64_t n0 = 0, n1 = 0;
#pragma unroll 1
            for (int q = gw; q < nk; q += 8) {
                const int64_t av = AVs[q];
                if (!av) continue;
                const int2 vv = reinterpret_cast<const int2*>(Vs + (size_t)q * 64)[lane];
                n0 = wadd(n0, wmul(av, vv.x));
                n1 = wadd(n1, wmul(av, vv.y));
            }
            red[gw][2 * lane] = n0;
            red[gw][2 * lane + 1] = n1;
            group_sync(bar_id, 256);
            if (gw == 0) {
                int64_t t0 = 0, t1 = 0, zz = 0;
#pragma unroll
                for (int q = 0; q < 8; q++) { t0 = wadd(t0, red[q][2 * lane]); t1 = wadd(t1, red[q][2 * lane + 1]); zz = wadd(zz, red[q][64]); }
                const int64_t F = -log2fix(zz, a.LOG2);
                const int64_t v0 = power(t0, F, a.EXP2), v1 = power(t1, F, a.EXP2);
                int64_t* o = a.ATT + (size_t)r * d + h * 64;
                o[2 * lane] = v0;
                o[2 * lane + 1] = v1;
                const uint64_t w = warp_or64(mag(v0) | mag(v1));
                if (lane == 0) atomicOr((unsigned long long*)&or_out[r], (unsigned long long)w);
            }
        }
        group_sync(bar_id, 256);                     // the slot and red are free again
        if (k2 == 0 && grp == 0) stamp(a, ph, 2);
        if (gt == 0 && k2 + nsg < myg) att_issue(a, layer, cid + (grp + step * (k2 + nsg)) * G, slot, smem, s, t);
    }
}

// the embed phase: rows' position and word, R = wte + wpe, OR slot 0; the other OR slots cleared
__device__ __noinline__ void embed_phase(const MegaArgs& a) {
    const int tid = threadIdx.x, G = gridDim.x, cid = blockIdx.x;
    const int d = a.d;
    __shared__ uint64_t s_or[NT / 32];
    for (int i = cid * NT + tid; i < 4 * a.L * BN; i += G * NT)
        if (i >= BN) a.OR[i] = 0;
    for (int r = cid; r < a.rows; r += G) {
        int tok = a.slot_tok[r], pos = a.slot_len[r];
        if (tok < 0 || tok >= a.vocab) { if (tid == 0) set_err(a.err, DERR_TOKEN); tok = 0; }
        if (pos < 0 || pos >= a.nctx || pos >= a.kv.lim) { if (tid == 0) set_err(a.err, DERR_POS); }
        const int pe = (pos < 0 || pos >= a.nctx) ? 0 : pos;
        if (tid == 0) { a.row_slot[r] = r; a.row_pos[r] = pos; a.row_tok[r] = tok; }
        uint64_t o = 0;
        for (int i = tid; i < d; i += NT) {
            const int64_t v = wadd(__ldg(a.wte + (size_t)tok * d + i), __ldg(a.wpe + (size_t)pe * d + i));
            a.R[(size_t)r * d + i] = v;
            o |= mag(v);
        }
        o = warp_or64(o);
        if ((tid & 31) == 0) s_or[tid >> 5] = o;
        __syncthreads();
        if (tid == 0) {
            uint64_t all = 0;
            for (int k = 0; k < NT / 32; k++) all |= s_or[k];
            a.OR[r] = all;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(NT, 1) k_decode_mega(const MegaArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ Sh s;
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int crank = (int)cluster_rank(), cluster = blockIdx.x / MEGA_CS, ncl = gridDim.x / MEGA_CS;
    Track t{};
    if (tid == 0) {
        for (int k = 0; k < MAXKPS; k++) mbar_init(&s.wbar[k], 1);
        mbar_init(&s.accbar, 1);
        for (int k = 0; k < MAX_SLOTS; k++) mbar_init(&s.abar[k], 1);
        mbar_init(&s.rbar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&s.tmem, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const int L = a.L;
    uint32_t nbar = 0;
    const uint32_t G = gridDim.x;
    int ph = 0;
    stamp(a, 0, 0);
#define SYNC()                                  \
    do {                                        \
        stamp(a, ph, 6);                        \
        grid_sync(a.bar, ++nbar * G, a.err);    \
        ph++;                                   \
        stamp(a, ph, 0);                        \
    } while (0)
    // layer 0's qkv weights while the rows are embedded
    {
        const MegaBank& b0 = a.banks[0];
        if (tid == 0) issue_weights(a, 0, b0, unit_of(b0, cluster, crank, 0, ncl), smem, s, t);
    }
    embed_phase(a);
    SYNC();
    if (tid < BN) {
        s.pos[tid] = tid < a.rows ? ldcg_i32(a.row_pos + tid) : 0;
        s.slot[tid] = tid < a.rows ? ldcg_i32(a.row_slot + tid) : 0;
    }
    __syncthreads();
    for (int l = 0; l < L; l++) {
        const int bq = 4 * l, bp = bq + 1, bf = bq + 2, bm = bq + 3;
        uint64_t* OR = a.OR;
        // ---- qkv ----
        {
            const MegaBank& bk = a.banks[bq];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round(a, BankIO{bq, EPI_GAUGED, true, a.R, OR + (size_t)bq * BN, nullptr, nullptr, 0},
                           unit_of(bk, cluster, crank, rd, ncl), rd == 0, l, smem, s, t, ph);
            // proj's weights (a 1-block bank, below the arrival's buffers) fly during the arrival
            const MegaBank& nb = a.banks[bp];
            if (tid == 0) issue_weights(a, bp, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        SYNC();
        // ---- the arrival ----
        att_phase(a, l, OR + (size_t)bp * BN, smem, s, t, ph);
        SYNC();
        // ---- proj ----
        {
            const MegaBank& bk = a.banks[bp];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round(a, BankIO{bp, EPI_PLAIN_ADD, false, a.ATT, OR + (size_t)bp * BN, OR + (size_t)bf * BN, a.R, a.d},
                           unit_of(bk, cluster, crank, rd, ncl), rd == 0, l, smem, s, t, ph);
            const MegaBank& nb = a.banks[bf];
            if (tid == 0) issue_weights(a, bf, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        SYNC();
        // ---- fc + bend ----
        {
            const MegaBank& bk = a.banks[bf];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round(a, BankIO{bf, EPI_GAUGED_EDGE, false, a.R, OR + (size_t)bf * BN, OR + (size_t)bm * BN, a.HID, a.F},
                           unit_of(bk, cluster, crank, rd, ncl), rd == 0, l, smem, s, t, ph);
            const MegaBank& nb = a.banks[bm];
            if (tid == 0) issue_weights(a, bm, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        SYNC();
        // ---- mproj ----
        {
            const MegaBank& bk = a.banks[bm];
            const int nr = rounds_of(bk, ncl);
            uint64_t* nxt = l + 1 < L ? OR + (size_t)(bm + 1) * BN : nullptr;
            for (int rd = 0; rd < nr; rd++)
                bank_round(a, BankIO{bm, EPI_PLAIN_ADD, false, a.HID, OR + (size_t)bm * BN, nxt, a.R, a.d},
                           unit_of(bk, cluster, crank, rd, ncl), rd == 0, l, smem, s, t, ph);
            if (l + 1 < L) {
                const MegaBank& nb = a.banks[bm + 1];
                if (tid == 0) issue_weights(a, bm + 1, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
                SYNC();
            }
        }
    }
#undef SYNC
    stamp(a, ph, 6);
    // drain anything still in flight (only after a timeout can there be any), then free TMEM
    if (tid == 0)
        for (int k = 0; k < MAXKPS; k++)
            if (t.warm[k]) mbar_drain(&s.wbar[k], (t.warm[k] - 1) & 1);
    if (tid == 0 || tid == 256)                      // each warp group's leader armed its own arrival slots
        for (int k = 0; k < MAX_SLOTS; k++)
            if (t.aarm[k]) mbar_drain(&s.abar[k], (t.aarm[k] - 1) & 1);
    if (tid == 32 && t.acc) mbar_drain(&s.accbar, (t.acc - 1) & 1);
    if (tid == 64 && t.rpar) mbar_drain(&s.rbar, (t.rpar - 1) & 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(s.tmem, 256);
    cluster_sync();
}

}  // namespace

int mega_att_slot_bytes(int max_ctx) {
    const int bytes = (((max_ctx + 3) & ~3) * KEY_BYTES + 127) & ~127;
    return bytes <= DYN - ATT_BASE ? bytes : 0;
}

int mega_plan(MegaPlan& p, const TcBank* tc, const int32_t* const* e, const int64_t* const* b, int L) {
    mega_free(p);
    cudaError_t err;
    if ((err = cudaFuncSetAttribute(k_decode_mega, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN + 1024)) != cudaSuccess)
        return (int)err;
    if ((err = cudaFuncSetAttribute(k_decode_mega, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess)
        return (int)err;
    // how many MEGA_CS-CTA clusters are resident at once (all of them must be: they wait on one another)
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(MEGA_CS * 64);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = DYN + 1024;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = MEGA_CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int ncl = 0;
    if ((err = cudaOccupancyMaxActiveClusters(&ncl, k_decode_mega, &cfg)) != cudaSuccess) return (int)err;
    if (ncl < 1) return (int)cudaErrorInvalidConfiguration;
    std::vector<MegaBank> host(4 * L);
    std::vector<TcMap> maps(8 * L);
    for (int i = 0; i < 4 * L; i++) {
        const TcBank& t = tc[i];
        if (!t.ready) return (int)cudaErrorInvalidValue;
        MegaBank& m = host[i];
        m.e = e[i];
        m.b = b[i];
        m.colcorr_kb = t.colcorr_kb;
        m.w16 = t.w16;
        m.nin = t.nin;
        m.nout = t.nout;
        m.nout_pad = t.nout_pad;
        m.ntiles = t.nout_pad / 128;
        const int kb = t.nin / 128;
        // the split with the fewest rounds over the resident clusters; among equals the deepest K split
        int best = -1, best_rounds = 1 << 30;
        for (int tpc = 1; tpc <= MEGA_CS; tpc++) {
            if (MEGA_CS % tpc) continue;
            const int ks = MEGA_CS / tpc;
            if (kb % ks || kb / ks > MAXKPS) continue;
            const int per = ncl * tpc, r = (m.ntiles + per - 1) / per;
            if (r < best_rounds) { best_rounds = r; best = tpc; }
        }
        if (best < 0) return (int)cudaErrorInvalidValue;
        m.tpc = best;
        m.ks = MEGA_CS / best;
        m.kps = kb / m.ks;
        maps[2 * i] = t.map_wh;
        maps[2 * i + 1] = t.map_wl;
    }
    if ((err = cudaMalloc(&p.banks, sizeof(MegaBank) * host.size())) != cudaSuccess) return (int)err;
    if ((err = cudaMalloc(&p.maps, sizeof(TcMap) * maps.size())) != cudaSuccess) return (int)err;
    if ((err = cudaMalloc(&p.bar, sizeof(uint32_t))) != cudaSuccess) return (int)err;
    cudaMemcpy(p.banks, host.data(), sizeof(MegaBank) * host.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(p.maps, maps.data(), sizeof(TcMap) * maps.size(), cudaMemcpyHostToDevice);
    p.nclusters = ncl;
    p.smem = DYN + 1024;
    p.ready = 1;
    return (int)cudaGetLastError();
}

void mega_free(MegaPlan& p) {
    if (p.banks) cudaFree(p.banks);
    if (p.maps) cudaFree(p.maps);
    if (p.bar) cudaFree(p.bar);
    p = MegaPlan{};
}

int mega_launch(const MegaPlan& p, MegaArgs a, cudaStream_t st) {
    if (!p.ready || a.rows < 1 || a.rows > BN) return (int)cudaErrorInvalidValue;
    a.maps = p.maps;
    a.banks = p.banks;
    a.bar = p.bar;
    cudaError_t err = cudaMemsetAsync(p.bar, 0, sizeof(uint32_t), st);
    if (err != cudaSuccess) return (int)err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(MEGA_CS * p.nclusters);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = MEGA_CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, k_decode_mega, a);
}

}  // namespace b2
