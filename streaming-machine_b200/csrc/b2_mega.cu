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

constexpr int NT = 256;                              // threads per CTA (8 warps)
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
            const uint64_t t0 = gtime();
            while (ld_acquire(bar) < target) {
                if (gtime() - t0 > WAIT_NS) { atomicOr(err, DERR_TIMEOUT); break; }
                if (is_dead(err)) break;
            }
        }
        __threadfence();
    }
    __syncthreads();
}

struct Sh {
    uint64_t wbar[MAXKPS], accbar, abar[MAX_SLOTS];
    uint32_t tmem;
    int sh[BN];
    int64_t S1[BN], S2[BN], rowc[BN], LS[BN], e2[BN];
    uint32_t sat[BN][MAXKPS * 4];
    unsigned long long satrows;
    uint64_t hor[8][4];
    int32_t qs[MAX_SLOTS][64];
    int64_t red[8][66];
    int nslots, slot_bytes;
};

// per-thread bookkeeping of the asynchronous work this CTA has in flight (meaningful in the thread that owns it)
struct Track {
    uint32_t warm[MAXKPS];     // tid 0: times wbar[kb] was armed
    uint32_t wwait;            // MMA thread: parity bits of the next wbar waits
    uint32_t acc;              // all threads: completed accbar phases
    uint32_t aarm[MAX_SLOTS];  // tid 0: times abar[s] was armed
    uint32_t await_;           // all threads: parity bits of the next abar waits
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
// ---------------------------------------------------------------------------------------------------------------------
template <int EPI, bool HEADS>
B2_DEV void bank_round(const MegaArgs& a, int bi, const MegaBank& bk, const Unit u, bool prefetched, const int64_t* X,
                       const uint64_t* xor_in, uint64_t* or_out, int64_t* out, int ldo, int layer, uint8_t* smem, Sh& s,
                       Track& t) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tmem = s.tmem;
    uint8_t* xplanes = smem + bk.kps * WST;
    int64_t* P = (int64_t*)smem;                     // [BN][128] partial tile, over the planes once read
    const int kps = bk.kps, ks = bk.ks;

    if (u.on) {
        if (tid == 0 && !prefetched) issue_weights(a, bi, bk, u, smem, s, t);
        if (tid < BN) {
            s.S1[tid] = 0;
            s.S2[tid] = 0;
            s.rowc[tid] = 0;
            for (int w = 0; w < MAXKPS * 4; w++) s.sat[tid][w] = 0;
        }
        if (tid == 0) s.satrows = 0;
        __syncthreads();
        // ---- activations: to16 with the row's shift, the two byte planes, partial S1 / S2 / row correction ----
        {
            const int n = tid >> 2, cg = tid & 3;
            const bool nv = n < a.rows;
            const int sh = nv ? to16_shift(ldcgu(xor_in + n)) : 0;
            if (cg == 0) s.sh[n] = sh;
            int64_t S1 = 0, S2 = 0, rc = 0;
            for (int kb = 0; kb < kps; kb++) {
                const int k0 = (u.kk * kps + kb) * 128 + cg * 32;
                uint32_t hw[8], lw[8];
                uint32_t satw = 0;
                int64_t s1 = 0;
                int4 raw[16];
                const int4* src = reinterpret_cast<const int4*>(X + (size_t)n * bk.nin + k0);
#pragma unroll
                for (int v = 0; v < 16; v++) raw[v] = nv ? __ldcg(src + v) : make_int4(0, 0, 0, 0);
#pragma unroll
                for (int v4 = 0; v4 < 8; v4++) {
                    const int4 r0 = raw[2 * v4], r1 = raw[2 * v4 + 1];
                    const int64_t xv[4] = {(int64_t)(((uint64_t)(uint32_t)r0.y << 32) | (uint32_t)r0.x),
                                           (int64_t)(((uint64_t)(uint32_t)r0.w << 32) | (uint32_t)r0.z),
                                           (int64_t)(((uint64_t)(uint32_t)r1.y << 32) | (uint32_t)r1.x),
                                           (int64_t)(((uint64_t)(uint32_t)r1.w << 32) | (uint32_t)r1.z)};
                    uint32_t h = 0, l = 0;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int32_t x = (int32_t)rshift(xv[q], sh);
                        const bool sat = x == 32768;
                        h |= (uint32_t)(uint8_t)(int8_t)(sat ? 127 : (x >> 8)) << (8 * q);
                        l |= (uint32_t)(uint8_t)(int8_t)((x & 255) - 128) << (8 * q);
                        s1 += x;
                        S2 += (int64_t)x * x;
                        satw |= (uint32_t)sat << (v4 * 4 + q);
                    }
                    hw[v4] = h;
                    lw[v4] = l;
                }
                S1 += s1;
                rc += 128 * (s1 - 256 * (int64_t)__popc(satw));
                s.sat[n][kb * 4 + cg] = satw;
                if (satw) atomicOr(&s.satrows, 1ull << n);
                const uint32_t bh = saddr(xplanes + kb * XST), bl = bh + B_BYTES;
                st_shared_v4(bh + sw128(n, 2 * cg), hw[0], hw[1], hw[2], hw[3]);
                st_shared_v4(bh + sw128(n, 2 * cg + 1), hw[4], hw[5], hw[6], hw[7]);
                st_shared_v4(bl + sw128(n, 2 * cg), lw[0], lw[1], lw[2], lw[3]);
                st_shared_v4(bl + sw128(n, 2 * cg + 1), lw[4], lw[5], lw[6], lw[7]);
            }
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {        // the row's four threads are adjacent lanes
                S1 += __shfl_xor_sync(0xffffffffu, S1, o);
                S2 += __shfl_xor_sync(0xffffffffu, S2, o);
                rc += __shfl_xor_sync(0xffffffffu, rc, o);
            }
            if (cg == 0) { s.S1[n] = S1; s.S2[n] = S2; s.rowc[n] = rc; }
        }
        fence_proxy_async();
        __syncthreads();
        // ---- MMAs ----
        if (warp == 1 && lane == 0) {
            bool ok = true;
            for (int kb = 0; kb < kps; kb++) {
                const uint32_t par = (t.wwait >> kb) & 1;
                t.wwait ^= 1u << kb;
                if (ok && !mbar_wait(&s.wbar[kb], par, a.err)) ok = false;
            }
            tc_fence_after();
            if (ok)
                for (int kb = 0; kb < kps; kb++)
                    mma_kblock2(saddr(smem + kb * WST), saddr(xplanes + kb * XST), tmem, kb == 0);
            mma_commit(&s.accbar);                   // arrives once the issued MMAs (if any) are done
        }
        __syncwarp();
        int64_t colc = 0;
        {
            const int j = u.mt * 128 + (warp & 3) * 32 + lane;
            for (int kb = 0; kb < kps; kb++) colc += __ldg(bk.colcorr_kb + (size_t)(u.kk * kps + kb) * bk.nout_pad + j);
        }
        // one decision for the whole CTA: the TMEM loads below are warp-aligned
        const bool ok = __syncthreads_and(mbar_wait(&s.accbar, t.acc & 1, a.err));
        t.acc++;
        tc_fence_after();
        // ---- corrected partial piles -> P ----
        {
            const int m = (warp & 3) * 32 + lane, r0 = (warp >> 2) * 32;
            int64_t p[32];
            if (ok) {
                const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16) + r0;
                int64_t t16[16];
                tmem_piles16(trow, t16);
#pragma unroll
                for (int q = 0; q < 16; q++) p[q] = t16[q];
                tmem_piles16(trow + 16, t16);
#pragma unroll
                for (int q = 0; q < 16; q++) p[16 + q] = t16[q];
                const unsigned long long satrows = s.satrows;
#pragma unroll
                for (int q = 0; q < 32; q++) p[q] += colc + s.rowc[r0 + q];
                if ((satrows >> r0) & 0xffffffffull)      // rare: rows of this warp with +32768 entries
                    for (int q = 0; q < 32; q++) {
                        const int n = r0 + q;
                        if (!((satrows >> n) & 1)) continue;
                        int64_t add = 0;
                        for (int kb = 0; kb < kps; kb++)
                            for (int w = 0; w < 4; w++) {
                                uint32_t bits = s.sat[n][kb * 4 + w];
                                while (bits) {
                                    const int k = w * 32 + __ffs(bits) - 1;
                                    bits &= bits - 1;
                                    const uint8_t* A = smem + kb * WST;
                                    const int off = (int)sw128(m, k >> 4) + (k & 15);
                                    const int64_t wv = 256 * (int64_t)(int8_t)A[off] + (int64_t)(int8_t)A[A_BYTES + off] + 128;
                                    add += 256 * wv;
                                }
                            }
#pragma unroll
                        for (int v = 0; v < 32; v++)
                            if (v == q) p[v] += add;
                    }
            } else {
#pragma unroll
                for (int q = 0; q < 32; q++) p[q] = 0;
            }
            tc_fence_before();
            __syncthreads();                         // every read of the planes and of TMEM is done
#pragma unroll
            for (int q = 0; q < 32; q++) P[(r0 + q) * 128 + m] = p[q];
        }
    }
    cluster_sync();                                  // the cluster's partial tiles and row sums are written
    if (u.on) {
        // ---- my slice of rows: sum over my sub-group's CTAs, finish ----
        const int n0 = u.kk * BN / ks, n1 = (u.kk + 1) * BN / ks;
        const int g0 = u.g * ks;
        uint32_t peer[MEGA_CS];
        {
            const uint32_t pbase = saddr(P);
#pragma unroll
            for (int p = 0; p < MEGA_CS; p++) peer[p] = p < ks ? mapa(pbase, g0 + p) : 0;
        }
        if (tid < n1 - n0) {
            const int n = n0 + tid;
            int64_t LS = 0, e2 = 0;
            if (GAUGED && n < a.rows) {
                const uint32_t o1 = saddr(&s.S1[n]), o2 = saddr(&s.S2[n]);
                int64_t S1 = 0, S2 = 0;
                for (int p = 0; p < ks; p++) {
                    S1 += ld_dsmem(mapa(o1, g0 + p));
                    S2 += ld_dsmem(mapa(o2, g0 + p));
                }
                LS = gauge_LS(S1, S2, -16 + s.sh[n], a.LOG2, a.log768, a.eps40);
                e2 = __ldg(a.EXP2 + (wsub(0, LS) & 0xFFFF));
            }
            s.LS[n] = LS;
            s.e2[n] = e2;
        }
        __syncthreads();
        const int m = tid & 127, ro = tid >> 7;
        const int j = u.mt * 128 + m;
        const bool jv = j < bk.nout;
        const int64_t e_j = jv ? (int64_t)__ldg(bk.e + j) : 0, b_j = jv ? __ldg(bk.b + j) : 0;
        const int nit = (n1 - n0 + 1) >> 1;
        const int H = a.kv.H, dm = H * 64;
        for (int it0 = 0; it0 < nit; it0 += 4) {
            int64_t sums[4];
            {
                int64_t tt[4][MEGA_CS];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int n = n0 + 2 * (it0 + q) + ro;
                    const bool ld = jv && it0 + q < nit && n < n1 && n < a.rows;
                    const uint32_t off = (uint32_t)(n * 128 + m) * 8;
#pragma unroll
                    for (int p = 0; p < MEGA_CS; p++) tt[q][p] = (ld && p < ks) ? ld_dsmem(peer[p] + off) : 0;
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    int64_t v = 0;
#pragma unroll
                    for (int p = 0; p < MEGA_CS; p++) v = wadd(v, tt[q][p]);
                    sums[q] = v;
                }
            }
            int64_t vals[4];
            bool valids[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int n = n0 + 2 * (it0 + q) + ro;
                valids[q] = jv && it0 + q < nit && n < n1 && n < a.rows;
                vals[q] = valids[q] ? epi_value<EPI>(sums[q], e_j, b_j, -16 + s.sh[n], s.LS[n], s.e2[n], a.PHI) : 0;
            }
            if (HEADS) {
                // heads16: each 64-column half of the tile is one head part (q, k or v of one head); a row's OR over
                // the part is the OR over its two warps
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const uint64_t w = warp_or64(valids[q] ? mag(vals[q]) : 0);
                    if (lane == 0) s.hor[warp][q] = w;
                }
                __syncthreads();
                uint64_t por[4];
#pragma unroll
                for (int q = 0; q < 4; q++) por[q] = s.hor[warp][q] | s.hor[warp ^ 1][q];
                __syncthreads();
                const int part = 2 * u.mt + (m >> 6), kind = part / H, hh = part % H, dd = m & 63;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int n = n0 + 2 * (it0 + q) + ro;
                    const bool valid = valids[q];
                    const int64_t val = vals[q];
                    const int sh = to16_shift(por[q]);
                    const int32_t x = (int32_t)rshift(val, sh);
                    if (kind == 0) {
                        if (valid) {
                            a.q16[(size_t)n * dm + hh * 64 + dd] = x;
                            if (dd == 0) a.qexp[n * H + hh] = -16 + sh;
                        }
                    } else {
                        const int pos = valid ? ldcg_i32(a.row_pos + n) : 0;
                        const bool pv = valid && pos >= 0 && pos < a.kv.lim;
                        if (valid && !pv && dd == 0) set_err(a.err, DERR_POS);
                        const size_t idx = pv ? kv_index(ldcg_i32(a.row_slot + n), layer, hh, pos, a.kv.L, H, a.kv.ctx) : 0;
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
                }
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int n = n0 + 2 * (it0 + q) + ro;
                    const bool valid = valids[q];
                    int64_t o = vals[q];
                    if (valid) {
                        int64_t* dst = out + (size_t)n * ldo + j;
                        if (EPI == EPI_PLAIN_ADD) o = wadd(ldcg(dst), o);
                        *dst = o;
                    }
                    const uint64_t wor = warp_or64(valid ? mag(o) : 0);
                    if (lane == 0 && or_out && valid) atomicOr((unsigned long long*)&or_out[n], (unsigned long long)wor);
                }
            }
        }
        if (HEADS) fence_async_global();             // the key/value append is read by bulk copies next phase
    }
    cluster_sync();                                  // no CTA reuses its shared memory while a peer may read it
}

// ---------------------------------------------------------------------------------------------------------------------
// the arrival phase (base2.py:85-100; as k_attend_bulk, 8 warps per unit): unit = (row, head), units spread over the
// CTAs, each unit's stream run copied into one of `nslots` shared-memory slots up to nslots units ahead
// ---------------------------------------------------------------------------------------------------------------------
B2_DEV void att_issue(const MegaArgs& a, int layer, int unit, int slot, uint8_t* smem, Sh& s, Track& t) {
    const int r = unit / a.H, h = unit % a.H;
    const int p = ldcg_i32(a.row_pos + r);
    if (p < 0 || p >= a.kv.lim || is_dead(a.err)) return;
    const int nkr = (p + 1 + 3) & ~3;
    uint8_t* base_s = smem + ATT_BASE + (size_t)slot * s.slot_bytes;
    const size_t base = kv_index(ldcg_i32(a.row_slot + r), layer, h, 0, a.kv.L, a.kv.H, a.kv.ctx);
    fence_async_global();
    mbar_expect_tx(&s.abar[slot], (uint32_t)nkr * (128 + 256 + 8 + 4));
    t.aarm[slot]++;
    bulk_g2s(base_s, a.kv.k + base * 64, (uint32_t)nkr * 128, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 128, a.kv.v + base * 64, (uint32_t)nkr * 256, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 384, a.kv.kmask + base, (uint32_t)nkr * 8, &s.abar[slot]);
    bulk_g2s(base_s + (size_t)nkr * 392, a.kv.kexp + base, (uint32_t)nkr * 4, &s.abar[slot]);
}

B2_DEV void att_phase(const MegaArgs& a, int layer, uint64_t* or_out, uint8_t* smem, Sh& s, Track& t) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int G = gridDim.x, cid = blockIdx.x;
    const int nunits = a.rows * a.H;
    const int my = cid < nunits ? (nunits - cid + G - 1) / G : 0;
    if (!my) return;
    // slots sized for the longest run among my units
    if (tid == 0) {
        int nk = 1;
        for (int i = 0; i < my; i++) {
            const int p = ldcg_i32(a.row_pos + (cid + i * G) / a.H);
            nk = max(nk, min(max(p + 1, 1), a.kv.lim));
        }
        const int bytes = (((nk + 3) & ~3) * KEY_BYTES + 127) & ~127;
        int ns = (DYN - ATT_BASE) / bytes;
        ns = min(ns, min(MAX_SLOTS, my));
        s.slot_bytes = bytes;
        s.nslots = max(ns, 1);
        for (int i = 0; i < s.nslots; i++) att_issue(a, layer, cid + i * G, i, smem, s, t);
    }
    __syncthreads();
    const int NS = s.nslots;
    const int d = a.H * 64;
    for (int i = 0; i < my; i++) {
        const int unit = cid + i * G, slot = i % NS;
        const int r = unit / a.H, h = unit % a.H;
        const int p = ldcg_i32(a.row_pos + r);
        const bool pv = p >= 0 && p < a.kv.lim;
        const int nk = p + 1, nkr = (nk + 3) & ~3;
        uint8_t* sb = smem + ATT_BASE + (size_t)slot * s.slot_bytes;
        int16_t* Ks = reinterpret_cast<int16_t*>(sb);
        int32_t* Vs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 128);
        uint64_t* KMs = reinterpret_cast<uint64_t*>(sb + (size_t)nkr * 384);
        int32_t* KEs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 392);
        int64_t* SCs = reinterpret_cast<int64_t*>(sb + (size_t)nkr * 396);
        int32_t* AVs = reinterpret_cast<int32_t*>(sb + (size_t)nkr * 404);
        if (tid < 64) s.qs[slot][tid] = pv ? __ldcg(a.q16 + (size_t)r * d + h * 64 + tid) : 0;
        const int64_t eq = pv ? __ldcg(a.qexp + r * a.H + h) : 0;
        bool ok = pv;
        if (pv) {
            const uint32_t par = (t.await_ >> slot) & 1;
            t.await_ ^= 1u << slot;
            ok = mbar_wait(&s.abar[slot], par, a.err);
        }
        ok = __syncthreads_and(ok);                  // one decision for the CTA: the block below synchronises
        if (ok) {
            // pass 1: scores, 8 lanes per key
            int qr[8];
#pragma unroll
            for (int q = 0; q < 8; q++) qr[q] = s.qs[slot][(lane & 7) * 8 + q];
            int64_t lmax = INT64_MIN;
            for (int c = wid; c * 4 < nk; c += 8) {
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
            if (lane == 0) s.red[wid][65] = lmax;
            __syncthreads();
            int64_t start = s.red[0][65];
#pragma unroll
            for (int k = 1; k < 8; k++) start = s.red[k][65] > start ? s.red[k][65] : start;
            // pass 1b: arrival weights and their total
            int64_t z = 0;
            for (int q = tid; q < nk; q += NT) {
                const int64_t av = arrival(wsub(start, SCs[q]), a.ARR, a.alen, a.err);
                AVs[q] = (int32_t)av;
                z = wadd(z, av);
            }
            z = warp_sum64(z);
            __syncthreads();
            if (lane == 0) s.red[wid][64] = z;
            // pass 2: 2 dims per lane, warps split the keys
            int64_t n0 = 0, n1 = 0;
            for (int q = wid; q < nk; q += 8) {
                const int64_t av = AVs[q];
                if (!av) continue;
                const int2 vv = reinterpret_cast<const int2*>(Vs + (size_t)q * 64)[lane];
                n0 = wadd(n0, wmul(av, vv.x));
                n1 = wadd(n1, wmul(av, vv.y));
            }
            s.red[wid][2 * lane] = n0;
            s.red[wid][2 * lane + 1] = n1;
            __syncthreads();
            if (wid == 0) {
                int64_t t0 = 0, t1 = 0, zz = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) { t0 = wadd(t0, s.red[k][2 * lane]); t1 = wadd(t1, s.red[k][2 * lane + 1]); zz = wadd(zz, s.red[k][64]); }
                const int64_t F = -log2fix(zz, a.LOG2);
                const int64_t v0 = power(t0, F, a.EXP2), v1 = power(t1, F, a.EXP2);
                int64_t* o = a.ATT + (size_t)r * d + h * 64;
                o[2 * lane] = v0;
                o[2 * lane + 1] = v1;
                const uint64_t w = warp_or64(mag(v0) | mag(v1));
                if (lane == 0) atomicOr((unsigned long long*)&or_out[r], (unsigned long long)w);
            }
        }
        __syncthreads();                             // the slot and s.red are free again
        if (tid == 0 && i + NS < my) att_issue(a, layer, cid + (i + NS) * G, slot, smem, s, t);
    }
}

// the embed phase: rows' position and word, R = wte + wpe, OR slot 0; the other OR slots cleared
B2_DEV void embed_phase(const MegaArgs& a) {
    const int tid = threadIdx.x, G = gridDim.x, cid = blockIdx.x;
    const int d = a.d;
    __shared__ uint64_t s_or[8];
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
            for (int k = 0; k < 8; k++) all |= s_or[k];
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
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&s.tmem, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const int L = a.L;
    uint32_t nbar = 0;
    const uint32_t G = gridDim.x;
    // layer 0's qkv weights while the rows are embedded
    {
        const MegaBank& b0 = a.banks[0];
        if (tid == 0) issue_weights(a, 0, b0, unit_of(b0, cluster, crank, 0, ncl), smem, s, t);
    }
    embed_phase(a);
    grid_sync(a.bar, ++nbar * G, a.err);
    for (int l = 0; l < L; l++) {
        const int bq = 4 * l, bp = bq + 1, bf = bq + 2, bm = bq + 3;
        uint64_t* OR = a.OR;
        // ---- qkv ----
        {
            const MegaBank& bk = a.banks[bq];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round<EPI_GAUGED, true>(a, bq, bk, unit_of(bk, cluster, crank, rd, ncl), rd == 0, a.R,
                                             OR + (size_t)bq * BN, nullptr, nullptr, 0, l, smem, s, t);
            // proj's weights (a 1-block bank, below the arrival's buffers) fly during the arrival
            const MegaBank& nb = a.banks[bp];
            if (tid == 0) issue_weights(a, bp, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        grid_sync(a.bar, ++nbar * G, a.err);
        // ---- the arrival ----
        att_phase(a, l, OR + (size_t)bp * BN, smem, s, t);
        grid_sync(a.bar, ++nbar * G, a.err);
        // ---- proj ----
        {
            const MegaBank& bk = a.banks[bp];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round<EPI_PLAIN_ADD, false>(a, bp, bk, unit_of(bk, cluster, crank, rd, ncl), rd == 0, a.ATT,
                                                 OR + (size_t)bp * BN, OR + (size_t)bf * BN, a.R, a.d, l, smem, s, t);
            const MegaBank& nb = a.banks[bf];
            if (tid == 0) issue_weights(a, bf, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        grid_sync(a.bar, ++nbar * G, a.err);
        // ---- fc + bend ----
        {
            const MegaBank& bk = a.banks[bf];
            const int nr = rounds_of(bk, ncl);
            for (int rd = 0; rd < nr; rd++)
                bank_round<EPI_GAUGED_EDGE, false>(a, bf, bk, unit_of(bk, cluster, crank, rd, ncl), rd == 0, a.R,
                                                   OR + (size_t)bf * BN, OR + (size_t)bm * BN, a.HID, a.F, l, smem, s, t);
            const MegaBank& nb = a.banks[bm];
            if (tid == 0) issue_weights(a, bm, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
        }
        grid_sync(a.bar, ++nbar * G, a.err);
        // ---- mproj ----
        {
            const MegaBank& bk = a.banks[bm];
            const int nr = rounds_of(bk, ncl);
            uint64_t* nxt = l + 1 < L ? OR + (size_t)(bm + 1) * BN : nullptr;
            for (int rd = 0; rd < nr; rd++)
                bank_round<EPI_PLAIN_ADD, false>(a, bm, bk, unit_of(bk, cluster, crank, rd, ncl), rd == 0, a.HID,
                                                 OR + (size_t)bm * BN, nxt, a.R, a.d, l, smem, s, t);
            if (l + 1 < L) {
                const MegaBank& nb = a.banks[bm + 1];
                if (tid == 0) issue_weights(a, bm + 1, nb, unit_of(nb, cluster, crank, 0, ncl), smem, s, t);
                grid_sync(a.bar, ++nbar * G, a.err);
            }
        }
    }
    // drain anything still in flight (only after a timeout can there be any), then free TMEM
    if (tid == 0) {
        for (int k = 0; k < MAXKPS; k++)
            if (t.warm[k]) mbar_drain(&s.wbar[k], (t.warm[k] - 1) & 1);
        for (int k = 0; k < MAX_SLOTS; k++)
            if (t.aarm[k]) mbar_drain(&s.abar[k], (t.aarm[k] - 1) & 1);
    }
    if (tid == 32 && t.acc) mbar_drain(&s.accbar, (t.acc - 1) & 1);
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
