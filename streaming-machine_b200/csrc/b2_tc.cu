// b2_tc.cu -- the bank product on tcgen05 tensor cores (kind::i8), exact (see b2_tc.cuh for the identity).
//
// A tile = 128 output columns (the MMA's M, TMEM lanes) x 64 rows (the MMA's N, TMEM columns). One thread streams
// the four planes of each 128-byte K block into shared memory with TMA (SWIZZLE_128B, K-major), one thread issues
// 16 MMAs per K block (4 K steps x {wh.xh, wh.xl, wl.xh, wl.xl}) into three int32 accumulators in TMEM, and
// epilogue warps read them back (tcgen05.ld). Two kernels: k_bank_split (decode: few output tiles, the K range split
// over a thread-block cluster and reduced over DSMEM) and k_bank_tiles (many tiles: persistent, TMEM double-buffered).
// Every mbarrier wait is bounded; on a timeout the kernel sets DERR_TIMEOUT, stops issuing work, frees its TMEM and
// returns (the call then reports an error).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "b2_epi.cuh"
#include "b2_ptx.cuh"
#include "b2_tc.cuh"
#include "b2_tcgen05.cuh"

namespace b2 {

namespace {

struct TcArgs {
    int nin, nout, rows;
    int kps;          // K blocks (of 128) per CTA (split) / per tile (tiles)
    int ksplit;       // CTAs along K per tile (= cluster size)
    int stages;
    int mtiles, ntiles;
    const int64_t* colcorr;
    const int64_t* rowcorr;
    const int32_t* nsat;
    const int16_t* sat;
    int sat_ld;
    const int16_t* w16;
    uint32_t* err;
    EpiArgs epi;
    int heads;        // EPI_GAUGED on the split path: heads16 in the epilogue (hd), no q/k/v stores
    TcHeads hd;
    uint64_t* trace;  // optional (profiling aid): %globaltimer stamps [CTA][8] of this launch
    TcQuant q;        // k_bank_wide: quantise the rows in the kernel (q.X set) instead of reading a quant kernel's
    uint64_t* or_out; // optional: OR of |stored value| over each output row (atomicOr), for the next bank's q.xor_in
    TcRace race;      // k_bank_tiles: each 32-column group's race winner per row (race.v set); out may then be null
    uint64_t* stamp;  // b2_profile mode 2
};

B2_DEV void ld_dsmem2(uint32_t addr, uint64_t& a0, uint64_t& a1) {
    asm volatile("ld.shared::cluster.v2.u64 {%0, %1}, [%2];" : "=l"(a0), "=l"(a1) : "r"(addr));
}
B2_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
B2_DEV unsigned long long atom_add_release_u64(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.release.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}
B2_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// to16 of one int64 given as its two 32-bit halves, by the row's shift (0..49, base2.py:24-27): add half, shift
B2_DEV int32_t to16_halves(int lo, int hi, int sh) {
    const uint64_t x = ((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo;
    return sh ? (int32_t)((int64_t)(x + (1ull << (sh - 1))) >> sh) : (int32_t)(int64_t)x;
}
B2_DEV uint32_t hibyte16(int32_t x) { return (uint32_t)(uint8_t)(int8_t)(x == 32768 ? 127 : (x >> 8)); }
B2_DEV uint32_t lobyte16(int32_t x) { return (uint32_t)(uint8_t)(int8_t)((x & 255) - 128); }
// bit i of e -> bit 2i, bit i of o -> bit 2i + 1
B2_DEV uint64_t interleave32(uint32_t e, uint32_t o) {
    uint64_t x = e, y = o;
    x = (x | (x << 16)) & 0x0000FFFF0000FFFFull;
    y = (y | (y << 16)) & 0x0000FFFF0000FFFFull;
    x = (x | (x << 8)) & 0x00FF00FF00FF00FFull;
    y = (y | (y << 8)) & 0x00FF00FF00FF00FFull;
    x = (x | (x << 4)) & 0x0F0F0F0F0F0F0F0Full;
    y = (y | (y << 4)) & 0x0F0F0F0F0F0F0F0Full;
    x = (x | (x << 2)) & 0x3333333333333333ull;
    y = (y | (y << 2)) & 0x3333333333333333ull;
    x = (x | (x << 1)) & 0x5555555555555555ull;
    y = (y | (y << 1)) & 0x5555555555555555ull;
    return x | (y << 1);
}

// profiling aid: thread 0 of the CTA stamps step k
B2_DEV void tstamp(const TcArgs& a, int k) {
    if (a.trace && threadIdx.x == 0)
        a.trace[(((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 + k] = gtime();
}

// the 16 MMAs of one K block: 4 K steps x {wh.xh -> A1, wh.xl + wl.xh -> A2, wl.xl -> A3}
B2_DEV void mma_kblock(uint32_t base, uint32_t tacc, bool first) {
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        uint64_t ah = sdesc(base + kk * 32), al = sdesc(base + A_BYTES + kk * 32);
        uint64_t bh = sdesc(base + 2 * A_BYTES + kk * 32), bl = sdesc(base + 2 * A_BYTES + B_BYTES + kk * 32);
        uint32_t acc = (!first || kk) ? 1u : 0u;
        mma_i8(tacc + 0 * BN, ah, bh, IDESC, acc);
        mma_i8(tacc + 1 * BN, ah, bl, IDESC, acc);
        mma_i8(tacc + 1 * BN, al, bh, IDESC, 1);
        mma_i8(tacc + 2 * BN, al, bl, IDESC, acc);
    }
}

// everything a finished pile of row n needs besides its column
struct RowData {
    int64_t ex, LS, e2, rowc;
    int32_t nsat, orow;
};
template <bool GAUGED>
B2_DEV RowData load_row(const TcArgs& a, int n) {
    RowData d{0, 0, 0, 0, 0, n};
    if (n < a.rows) {
        d.ex = a.epi.ex[n];
        if (GAUGED) {
            d.LS = a.epi.LS[n];
            d.e2 = __ldg(a.epi.EXP2 + (wsub(0, d.LS) & 0xFFFF));
        }
        d.rowc = a.rowcorr[n];
        d.nsat = a.nsat[n];
        if (a.epi.out_map) d.orow = a.epi.out_map[n];
    }
    return d;
}

// the finished value of (row n, column j): corrections, then the bank's epilogue
template <int EPI>
B2_DEV int64_t finish_value(const TcArgs& a, const RowData& r, int n, int j, int64_t pile, int64_t colc, int64_t e_j,
                            int64_t b_j) {
    pile += colc + r.rowc;
    for (int u = 0; u < r.nsat; u++) pile += 256 * (int64_t)a.w16[(size_t)a.sat[(size_t)n * a.sat_ld + u] * a.nout + j];
    return epi_value<EPI>(pile, e_j, b_j, r.ex, r.LS, r.e2, a.epi.PHI);
}

// the finished pile of (row n, column j): corrections, then the bank's epilogue, stored
template <int EPI>
B2_DEV void finish(const TcArgs& a, const RowData& r, int n, int j, int64_t pile, int64_t colc, int64_t e_j, int64_t b_j) {
    pile += colc + r.rowc;
    for (int u = 0; u < r.nsat; u++) pile += 256 * (int64_t)a.w16[(size_t)a.sat[(size_t)n * a.sat_ld + u] * a.nout + j];
    int64_t v = epi_value<EPI>(pile, e_j, b_j, r.ex, r.LS, r.e2, a.epi.PHI);
    int64_t* o = a.epi.out + (size_t)r.orow * a.epi.ldo + j;
    *o = EPI == EPI_PLAIN_ADD ? wadd(*o, v) : v;
}

// the qkv bank's epilogue when its 64-column tile is one head part (heads16: base2_stream.swift:112-119, base2.py:93;
// Pythia's turn first: pythia_base2.py:116-134, the arithmetic of k_heads_pythia): one row held by one warp, lane l
// with columns 2l, 2l + 1 (values v0, v1). GPT-2's parts are q of every head, then k, then v (part = kind H + head);
// Pythia's are q, k, v per head (part = 3 head + kind). Pythia's q and k are turned (dims t and t + 8 of the first 16
// pair up: lanes l and l ^ 4 for l < 8; an input past 2^31 is where the reference asserts); then q and k are to16'd
// over the part (the row's OR is this warp's): q to q16, k to the key store with its +32768 bits and exponent; v goes
// to the value store as it is (int32, or DERR_VOVF).
B2_DEV void heads_row(const TcArgs& a, int mt, int n, int slot, int pos, bool rv, int64_t v0, int64_t v1) {
    const int lane = threadIdx.x & 31, H = a.hd.kv.H, dm = H * 64, dd = 2 * lane;
    const bool py = a.hd.pythia != 0;
    const int kind = py ? mt % 3 : mt / H, hh = py ? mt / 3 : mt % H;
    const bool pv = rv && pos >= 0 && pos < a.hd.kv.lim;
    if (rv && !pv && lane == 0 && (py || kind > 0)) set_err(a.err, DERR_POS);
    if (py && kind < 2) {
        const bool big = pv && lane < 8 && (mag(v0) >= (1ull << 31) || mag(v1) >= (1ull << 31));
        if (__any_sync(0xffffffffu, big) && lane == 0) set_err(a.err, DERR_RANGE);
        const int64_t p0 = __shfl_xor_sync(0xffffffffu, v0, 4), p1 = __shfl_xor_sync(0xffffffffu, v1, 4);
        if (pv && lane < 8) {
            const int t0 = (2 * lane) & 7;              // dims 2l, 2l + 1 modulo the pair distance 8
            const size_t cb = (size_t)pos * 8 + t0;
            const int64_t c0 = a.hd.COS[cb], s0 = a.hd.SIN[cb], c1 = a.hd.COS[cb + 1], s1 = a.hd.SIN[cb + 1];
            if (lane < 4) {                             // a (this lane), b (the partner): a c - b s
                v0 = rshift(wsub(wmul(v0, c0), wmul(p0, s0)), 30);
                v1 = rshift(wsub(wmul(v1, c1), wmul(p1, s1)), 30);
            } else {                                    // b (this lane), a (the partner): b c + a s
                v0 = rshift(wadd(wmul(v0, c0), wmul(p0, s0)), 30);
                v1 = rshift(wadd(wmul(v1, c1), wmul(p1, s1)), 30);
            }
        }
    }
    const uint64_t por = warp_or64(rv ? (mag(v0) | mag(v1)) : 0);
    const int sh = to16_shift(por);
    const int32_t x0 = (int32_t)rshift(v0, sh), x1 = (int32_t)rshift(v1, sh);
    if (kind == 0) {
        if (rv && (!py || pv)) {
            *reinterpret_cast<int2*>(a.hd.q16 + (size_t)n * dm + hh * 64 + dd) = make_int2(x0, x1);
            if (lane == 0) a.hd.qexp[n * H + hh] = -16 + sh;
        }
        return;
    }
    const size_t idx = pv ? kv_index(slot, a.hd.layer, hh, pos, a.hd.kv.L, H, a.hd.kv.ctx) : 0;
    if (kind == 1) {
        // +32768 is not an int16: a bit per entry, lane l's two columns are bits 2l, 2l + 1
        const uint32_t be = __ballot_sync(0xffffffffu, pv && x0 == 32768);
        const uint32_t bo = __ballot_sync(0xffffffffu, pv && x1 == 32768);
        if (pv) {
            *reinterpret_cast<uint32_t*>(a.hd.kv.k + idx * 64 + dd) = ((uint32_t)x0 & 0xFFFFu) | ((uint32_t)x1 << 16);
            if (lane == 0) {
                a.hd.kv.kmask[idx] = interleave32(be, bo);
                a.hd.kv.kexp[idx] = -16 + sh;
            }
        }
    } else if (pv) {
        if (v0 != (int64_t)(int32_t)v0 || v1 != (int64_t)(int32_t)v1) set_err(a.err, DERR_VOVF);
        *reinterpret_cast<int2*>(a.hd.kv.v + idx * 64 + dd) = make_int2((int32_t)v0, (int32_t)v1);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// Decode banks (rows <= 64, few output tiles): split-K over a thread-block cluster (1, ksplit, 1). Each CTA holds one
// or two K blocks (all loaded at once; the weights before the dependency wait), keeps its partial int64 tile in its
// own shared memory, and after a cluster barrier reduces a 1/ksplit slice of the rows over DSMEM and finishes it.
// 256 threads: warp 0 lane 0 = TMA, warp 1 lane 0 = MMA, warps 2-7 stage the rows, all 8 warps in the epilogue.
// ---------------------------------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256, 1)
    k_bank_split(const __grid_constant__ CUtensorMap mwh, const __grid_constant__ CUtensorMap mwl,
                 const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl, const TcArgs a) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full_bar[MAX_KPS], acc_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_dead, s_abort;
    __shared__ RowData s_row[BN];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    int64_t* P = (int64_t*)smem;   // partial tile [BN][128], over the stage memory once the MMAs are done
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, ks = blockIdx.y;
    const uint32_t crank = cluster_rank();
    tstamp(a, 0);

    if (tid == 0) {
        for (int kb = 0; kb < a.kps; kb++) mbar_init(&full_bar[kb], 1);
        mbar_init(&acc_bar, 1);
        s_abort = 0;
        s_dead = (*(volatile uint32_t*)a.err & DERR_TIMEOUT) != 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const bool dead = s_dead != 0;
    tstamp(a, 1);
    if (tid == 0 && !dead) {          // weights: independent of earlier kernels
        for (int kb = 0; kb < a.kps; kb++) {
            uint8_t* st = smem + kb * STAGE;
            int kx = (ks * a.kps + kb) * 128;
            mbar_expect_tx(&full_bar[kb], STAGE);
            const uint64_t pol = l2_evict_first();   // a decode step reads each weight once
            tma_load_2d_hint(st, &mwh, &full_bar[kb], kx, mt * 128, pol);
            tma_load_2d_hint(st + A_BYTES, &mwl, &full_bar[kb], kx, mt * 128, pol);
        }
    }
    // this thread's two columns' constants (the bank's own data: read before the dependency wait)
    const int cp = tid & 63, rg = tid >> 6;
    const int j0 = mt * 128 + 2 * cp, j1 = j0 + 1;
    const bool cv0 = j0 < a.nout, cv1 = j1 < a.nout;
    const int64_t colc0 = cv0 ? a.colcorr[j0] : 0, colc1 = cv1 ? a.colcorr[j1] : 0;
    const int64_t e0 = cv0 ? (int64_t)a.epi.e[j0] : 0, b0 = cv0 ? a.epi.b[j0] : 0;
    const int64_t e1 = cv1 ? (int64_t)a.epi.e[j1] : 0, b1 = cv1 ? a.epi.b[j1] : 0;
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    tstamp(a, 2);
    if (tid == 0 && !dead) {
        for (int kb = 0; kb < a.kps; kb++) {
            uint8_t* st = smem + kb * STAGE;
            int kx = (ks * a.kps + kb) * 128;
            tma_load_2d(st + 2 * A_BYTES, &mxh, &full_bar[kb], kx, 0);
            tma_load_2d(st + 2 * A_BYTES + B_BYTES, &mxl, &full_bar[kb], kx, 0);
        }
    } else if (warp == 1 && lane == 0 && !dead) {
        for (int kb = 0; kb < a.kps; kb++) {
            if (!mbar_wait(&full_bar[kb], 0, a.err)) { s_abort = 1; break; }
            tc_fence_after();
            mma_kblock(saddr(smem + kb * STAGE), tmem, kb == 0);
        }
        mma_commit(&acc_bar);
    } else if (warp >= 2) {
        for (int q = tid - 64; q < BN; q += 192) s_row[q] = load_row<GAUGED>(a, q);
    }
    __syncwarp();
    __syncthreads();
    const bool ok = !dead && mbar_wait(&acc_bar, 0, a.err);
    tc_fence_after();
    __syncthreads();
    tstamp(a, 3);
    const bool go = ok && !s_abort;
    if (go) {
        // this warp's quadrant (TMEM lanes = output columns) and row half
        const int m = (warp & 3) * 32 + lane, r0 = (warp >> 2) * 32;
        const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < 2; c++) {
            int64_t p[16];
            tmem_piles16(trow + r0 + 16 * c, p);
#pragma unroll
            for (int q = 0; q < 16; q++) P[(r0 + 16 * c + q) * 128 + m] = p[q];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);   // TMEM is no longer needed
    tstamp(a, 4);
    cluster_sync();                   // every CTA's partial tile is written
    tstamp(a, 5);
    {
        // my slice of rows, summed over the cluster. Thread (column pair cp, row group rg) takes columns 2 cp, 2 cp + 1
        // and rows n0 + rg, n0 + rg + 4, ..: one 16-byte DSMEM load per peer and row (the rate of DSMEM operations,
        // not its bandwidth, bounds this step). For the qkv bank with heads16 a head part's 64 columns are one warp.
        const int ksz = a.ksplit;
        const int n0 = (int)crank * BN / ksz, n1 = ((int)crank + 1) * BN / ksz;
        const bool jv0 = cv0 && go, jv1 = cv1 && go;
        uint32_t peer[MAX_SPLIT];
        const uint32_t pbase = saddr(P);
#pragma unroll
        for (int p = 0; p < MAX_SPLIT; p++) peer[p] = p < ksz ? mapa(pbase, p) : 0;
        const bool heads = EPI == EPI_GAUGED && a.heads;
        const int H = heads ? a.hd.kv.H : 1, dm = H * 64;
        const int part = 2 * mt + (cp >> 5), kind = part / H, hh = part % H, dd = (2 * cp) & 63;
        for (int nb = n0; nb < n1; nb += 4) {
            const int n = nb + rg;                   // the same for the whole warp
            const bool rv = n < n1 && n < a.rows;
            int64_t v0 = 0, v1 = 0;
            if (rv && (jv0 || jv1)) {
                const uint32_t off = (uint32_t)(n * 128 + 2 * cp) * 8;
                uint64_t t0[MAX_SPLIT], t1[MAX_SPLIT];
#pragma unroll
                for (int p = 0; p < MAX_SPLIT; p++) {
                    t0[p] = 0;
                    t1[p] = 0;
                    if (p < ksz) ld_dsmem2(peer[p] + off, t0[p], t1[p]);
                }
                uint64_t s0 = 0, s1 = 0;
#pragma unroll
                for (int p = 0; p < MAX_SPLIT; p++) { s0 += t0[p]; s1 += t1[p]; }
                if (jv0) v0 = finish_value<EPI>(a, s_row[n], n, j0, (int64_t)s0, colc0, e0, b0);
                if (jv1) v1 = finish_value<EPI>(a, s_row[n], n, j1, (int64_t)s1, colc1, e1, b1);
            }
            if (!heads) {
                int64_t w0 = v0, w1 = v1;
                if (rv) {
                    int64_t* o = a.epi.out + (size_t)s_row[n].orow * a.epi.ldo + j0;
                    if (EPI == EPI_PLAIN_ADD) {
                        if (jv0) w0 = wadd(o[0], v0);
                        if (jv1) w1 = wadd(o[1], v1);
                    }
                    if (jv0) o[0] = w0;
                    if (jv1) o[1] = w1;
                }
                if (a.or_out) {                      // the next bank's row OR over this warp's 64 columns
                    const uint64_t wor = warp_or64(rv ? ((jv0 ? mag(w0) : 0) | (jv1 ? mag(w1) : 0)) : 0);
                    if (lane == 0 && rv) atomicOr((unsigned long long*)&a.or_out[n], (unsigned long long)wor);
                }
                continue;
            }
            // heads16 (the Metal engine's heads16, base2_stream.swift:112-119; base2.py:93): the row's OR over the part
            const uint64_t por = warp_or64(rv ? (mag(v0) | mag(v1)) : 0);
            const int sh = to16_shift(por);
            const int32_t x0 = (int32_t)rshift(v0, sh), x1 = (int32_t)rshift(v1, sh);
            if (kind == 0) {
                if (rv) {
                    *reinterpret_cast<int2*>(a.hd.q16 + (size_t)n * dm + hh * 64 + dd) = make_int2(x0, x1);
                    if (dd == 0) a.hd.qexp[n * H + hh] = -16 + sh;
                }
            } else {
                const int pos = rv ? a.hd.row_pos[n] : 0;
                const bool pv = rv && pos >= 0 && pos < a.hd.kv.lim;
                if (rv && !pv && dd == 0) set_err(a.err, DERR_POS);
                const size_t idx = pv ? kv_index(a.hd.row_slot[n], a.hd.layer, hh, pos, a.hd.kv.L, H, a.hd.kv.ctx) : 0;
                if (kind == 1) {
                    // +32768 is not an int16: a bit per entry, lane l's two columns are bits 2l, 2l + 1
                    const uint32_t be = __ballot_sync(0xffffffffu, pv && x0 == 32768);
                    const uint32_t bo = __ballot_sync(0xffffffffu, pv && x1 == 32768);
                    if (pv) {
                        *reinterpret_cast<uint32_t*>(a.hd.kv.k + idx * 64 + dd) =
                            ((uint32_t)x0 & 0xFFFFu) | ((uint32_t)x1 << 16);
                        if (lane == 0) a.hd.kv.kmask[idx] = interleave32(be, bo);
                        if (dd == 0) a.hd.kv.kexp[idx] = -16 + sh;
                    }
                } else if (pv) {
                    if (v0 != (int64_t)(int32_t)v0 || v1 != (int64_t)(int32_t)v1) set_err(a.err, DERR_VOVF);
                    *reinterpret_cast<int2*>(a.hd.kv.v + idx * 64 + dd) = make_int2((int32_t)v0, (int32_t)v1);
                }
            }
        }
    }
    __syncthreads();
    tstamp(a, 6);
    cluster_sync();                   // no CTA leaves while a peer may still read its partial tile
    tstamp(a, 7);
}

// ---------------------------------------------------------------------------------------------------------------------
// Decode banks with at most 6 K blocks (nin <= 768) and rows <= 64: no K split, no cluster. CTA (mt, rh) owns 64
// output columns and 32 rows (32 rh ..) over the whole K range, every K block resident (<= 6 x 24 KB; the weights
// loaded before the dependency wait). Per K block the A operand is the two weight planes of its 64 columns stacked
// (wh in rows 0-63, wl in rows 64-127: M = 128) and the B operand the two row planes of its 32 rows stacked (xh in
// rows 0-31, xl in rows 32-63: N = 64), so ONE MMA (M128 N64 K32) per K step makes all four byte products in one
// 128 x 64 int32 accumulator:
//     D[o][r] = wh.xh (A1)   D[o][32 + r] = wh.xl   D[64 + o][r] = wl.xh   D[64 + o][32 + r] = wl.xl (A3)
// 512 threads: warp 0 lane 0 = TMA, warp 1 lane 0 = MMA, warps 2-15 load the row data. Epilogue: warp w < 8 reads
// TMEM lane quadrant w % 4, columns 16 (w / 4) .. + 16 of both halves, and parks H = 65536 A1 + 256 wh.xl (quadrants
// 0, 1) or L = 256 wl.xh + A3 (quadrants 2, 3) in shared memory, [row][column]; then warp w finishes rows w, w + 16
// (lane l: columns 2l, 2l + 1; for the qkv bank the tile is one head part, so heads16's OR is one warp's).
// ---------------------------------------------------------------------------------------------------------------------
constexpr int WIDE_THREADS = 512;
constexpr int WIDE_MAX_KB = 6;
constexpr int WIDE_ROWS = 32;
constexpr int WIDE_A = 2 * 64 * 128;                    // [wh; wl] of one K block
constexpr int WIDE_B = 2 * WIDE_ROWS * 128;             // [xh; xl]
constexpr int WIDE_KBLOCK = WIDE_A + WIDE_B;
__host__ __device__ inline int wide_smem_bytes(int nkb) {
    return (nkb * WIDE_KBLOCK > 2 * WIDE_ROWS * 64 * 8 ? nkb * WIDE_KBLOCK : 2 * WIDE_ROWS * 64 * 8) + 1024;
}

template <int EPI, bool QUANT>
__global__ void __launch_bounds__(WIDE_THREADS, 1)
    k_bank_wide(const __grid_constant__ CUtensorMap mwh, const __grid_constant__ CUtensorMap mwl,
                const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl, const TcArgs a) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full_bar[WIDE_MAX_KB], acc_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_dead, s_abort;
    __shared__ RowData s_row[WIDE_ROWS];
    __shared__ int32_t s_pos[WIDE_ROWS], s_slot[WIDE_ROWS];   // heads16: where each row's key / value goes
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    int64_t* HB = (int64_t*)smem;     // [32 rows][64 columns] H, over the K blocks once the MMAs are done
    int64_t* LB = HB + WIDE_ROWS * 64;   // [32 rows][64 columns] L
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x;        // output columns 64 mt .. + 64
    const int kz = blockIdx.y, nz = gridDim.y;   // K range: blocks kz * kps .. + kps (cluster (1, nz, 1))
    const int r0 = blockIdx.z * WIDE_ROWS;   // rows r0 .. + 32
    const int nkb = a.kps, kb0 = kz * nkb;
    tstamp(a, 0);

    if (tid == 0) {
        for (int kb = 0; kb < nkb; kb++) mbar_init(&full_bar[kb], 1);
        mbar_init(&acc_bar, 1);
        s_abort = 0;
        s_dead = (*(volatile uint32_t*)a.err & DERR_TIMEOUT) != 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tmem_slot, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const bool dead = s_dead != 0;
    tstamp(a, 1);
    if (tid == 0 && !dead) {          // weights: independent of earlier kernels
        for (int kb = 0; kb < nkb; kb++) {
            uint8_t* st = smem + kb * WIDE_KBLOCK;
            mbar_expect_tx(&full_bar[kb], WIDE_KBLOCK);
            const uint64_t pol = l2_evict_first();   // a decode step reads each weight once
            tma_load_2d_hint(st, &mwh, &full_bar[kb], (kb0 + kb) * 128, mt * 64, pol);
            tma_load_2d_hint(st + 64 * 128, &mwl, &full_bar[kb], (kb0 + kb) * 128, mt * 64, pol);
        }
    }
    // this lane's two columns' constants (the bank's own data: read before the dependency wait)
    const int j0 = mt * 64 + 2 * lane, j1 = j0 + 1;
    const bool cv0 = j0 < a.nout, cv1 = j1 < a.nout;
    const int64_t colc0 = cv0 ? a.colcorr[j0] : 0, colc1 = cv1 ? a.colcorr[j1] : 0;
    const int64_t e0 = cv0 ? (int64_t)a.epi.e[j0] : 0, b0 = cv0 ? a.epi.b[j0] : 0;
    const int64_t e1 = cv1 ? (int64_t)a.epi.e[j1] : 0, b1 = cv1 ? a.epi.b[j1] : 0;
    const bool heads = (EPI == EPI_GAUGED || EPI == EPI_PLAIN_OUT) && a.heads;
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    tstamp(a, 2);
    // the residual this thread adds to, final now that the wait has returned (in-kernel quantisation: no out_map)
    constexpr int RPW = WIDE_ROWS / (WIDE_THREADS / 32);   // rows per warp in the finish
    // the finish's rows: warp w takes rows w, w + 16 of the 32 (no split) or row 16 kz + w (2-CTA split, each CTA
    // finishing half of the rows); 4- and 8-CTA splits finish 8-row slices with one column per thread (plain banks)
    const int nrpw = nz == 1 ? RPW : 1;
    int64_t pre0[RPW], pre1[RPW], pres = 0;
    if (QUANT && EPI == EPI_PLAIN_ADD) {
        if (nz <= 2) {
#pragma unroll
            for (int it = 0; it < RPW; it++) {
                pre0[it] = 0;
                pre1[it] = 0;
                if (it >= nrpw) break;
                const int n = r0 + (nz == 1 ? warp + 16 * it : 16 * kz + warp);
                const int64_t* o = a.epi.out + (size_t)(n < a.rows ? n : 0) * a.epi.ldo + j0;
                pre0[it] = n < a.rows && cv0 ? o[0] : 0;
                pre1[it] = n < a.rows && cv1 ? o[1] : 0;
            }
        } else {
            const int n = r0 + kz * (WIDE_ROWS / nz) + (warp & 7), j = mt * 64 + 32 * (warp >> 3) + lane;
            if ((warp & 7) < WIDE_ROWS / nz && n < a.rows && j < a.nout) pres = a.epi.out[(size_t)n * a.epi.ldo + j];
        }
    }
    if (QUANT) {
        // the rows' to16 and byte planes, shared out over the CTAs of this row half: item (K block kb, rows
        // r0 + 8g ..) goes to CTA mt, mt + ntx, ..; thread t takes row 8g + t / 64, values 2 (t % 64), + 1 of the K
        // block. The row sums go to the per-row accumulators (atomics), +32768 entries to the row's list.
        const int ntx = gridDim.x * nz, nitems = nkb * nz * 4, cid = mt + gridDim.x * kz;
        const int c = 2 * (tid & 63);
        for (int it0 = cid; it0 < nitems && !dead; it0 += 2 * ntx) {
            // up to two items per pass, both rows' loads in flight together
            int4 v[2];
            int n[2], kbv[2], sh[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int it = it0 + u * ntx;
                kbv[u] = it >> 2;
                n[u] = it < nitems ? r0 + 8 * (it & 3) + (tid >> 6) : a.rows;
                v[u] = make_int4(0, 0, 0, 0);
                sh[u] = 0;
                if (n[u] < a.rows) {
                    sh[u] = to16_shift(a.q.xor_in[n[u]]);
                    v[u] = *reinterpret_cast<const int4*>(a.q.X + (size_t)n[u] * a.q.ldx + kbv[u] * 128 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (it0 + u * ntx >= nitems) break;        // the same for the whole CTA
                const int nn = n[u], kb = kbv[u];
                int32_t x0 = 0, x1 = 0;
                if (nn < a.rows) {
                    x0 = to16_halves(v[u].x, v[u].y, sh[u]);
                    x1 = to16_halves(v[u].z, v[u].w, sh[u]);
                    const size_t o = (size_t)nn * a.q.kmax + kb * 128 + c;
                    *reinterpret_cast<uint16_t*>(a.q.xh + o) = (uint16_t)(hibyte16(x0) | (hibyte16(x1) << 8));
                    *reinterpret_cast<uint16_t*>(a.q.xl + o) = (uint16_t)(lobyte16(x0) | (lobyte16(x1) << 8));
                    if (x0 == 32768) a.q.sat[(size_t)nn * a.q.kmax + atomicAdd(a.q.nsat + nn, 1)] = (int16_t)(kb * 128 + c);
                    if (x1 == 32768) a.q.sat[(size_t)nn * a.q.kmax + atomicAdd(a.q.nsat + nn, 1)] = (int16_t)(kb * 128 + c + 1);
                }
                // a row's 64 threads are two whole warps: warp sums, one atomic per warp and sum
                const uint32_t sq = (uint32_t)(x0 * x0) + (uint32_t)(x1 * x1);   // <= 2^31
                const int32_t t1 = (int32_t)__reduce_add_sync(0xffffffffu, (uint32_t)(x0 + x1));
                const uint32_t t2l = __reduce_add_sync(0xffffffffu, sq & 0xFFFFu);
                const uint32_t t2h = __reduce_add_sync(0xffffffffu, sq >> 16);
                if (lane == 0 && nn < a.rows) {
                    atomicAdd((unsigned long long*)(a.q.S1 + nn), (unsigned long long)(int64_t)t1);
                    atomicAdd((unsigned long long*)(a.q.S2 + nn), (unsigned long long)t2h * 65536ull + t2l);
                }
            }
        }
        // arrival on this row half's counter, then wait for all ntx CTAs of it (their planes and sums are complete)
        __syncthreads();
        if (tid == 0) {   // the release add covers the whole CTA's writes above (they happen before it: bar.sync)
            unsigned long long* ctr = a.q.ctr + blockIdx.z;
            const unsigned long long arrival = atom_add_release_u64(ctr, 1);
            const unsigned long long target = (arrival / ntx + 1) * ntx;
            if (!dead) {
                const uint64_t t0 = gtime(), lim = wait_limit(a.err);
                while (ld_acquire_u64(ctr) < target) {
                    if (gtime() - t0 > lim || (*(volatile uint32_t*)a.err & DERR_TIMEOUT)) {
                        atomicOr(a.err, DERR_TIMEOUT);
                        s_abort = 1;
                        break;
                    }
                }
            }
            fence_proxy_async_global();   // the planes were written through the generic proxy; TMA reads them next
        }
        __syncthreads();
    }
    tstamp(a, 6);
    if (tid == 0 && !dead && !s_abort) {
        for (int kb = 0; kb < nkb; kb++) {
            uint8_t* st = smem + kb * WIDE_KBLOCK + WIDE_A;
            tma_load_2d(st, &mxh, &full_bar[kb], (kb0 + kb) * 128, r0);
            tma_load_2d(st + WIDE_ROWS * 128, &mxl, &full_bar[kb], (kb0 + kb) * 128, r0);
        }
    } else if (warp == 1 && lane == 0 && !dead && !s_abort) {
        for (int kb = 0; kb < nkb; kb++) {
            if (!mbar_wait(&full_bar[kb], 0, a.err)) { s_abort = 1; break; }
            tc_fence_after();
            const uint32_t base = saddr(smem + kb * WIDE_KBLOCK);
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                mma_i8(tmem, sdesc(base + kk * 32), sdesc(base + WIDE_A + kk * 32), IDESC, (kb || kk) ? 1u : 0u);
        }
        mma_commit(&acc_bar);
    } else if (warp >= 2) {
        for (int q = tid - 64; q < WIDE_ROWS; q += WIDE_THREADS - 64) {
            if (QUANT) {
                RowData d{0, 0, 0, 0, 0, r0 + q};
                const int n = r0 + q;
                if (n < a.rows) {
                    const int64_t ex = -16 + to16_shift(a.q.xor_in[n]);
                    const int64_t S1 = a.q.S1[n], S2 = a.q.S2[n];
                    const int32_t ns = a.q.nsat[n];
                    d.ex = ex;
                    if (GAUGED) {
                        d.LS = gauge_LS(S1, S2, (int)ex, a.q.LOG2, a.q.log768, a.q.eps40);
                        d.e2 = __ldg(a.epi.EXP2 + (wsub(0, d.LS) & 0xFFFF));
                    }
                    d.rowc = 128 * (S1 - 256 * (int64_t)ns);
                    d.nsat = ns;
                }
                s_row[q] = d;
            } else {
                s_row[q] = load_row<GAUGED>(a, r0 + q);
            }
            if (heads) {
                s_pos[q] = r0 + q < a.rows ? a.hd.row_pos[r0 + q] : 0;
                s_slot[q] = r0 + q < a.rows ? a.hd.row_slot[r0 + q] : 0;
            }
        }
    }
    __syncwarp();
    __syncthreads();
    const bool ok = !dead && mbar_wait(&acc_bar, 0, a.err);
    tc_fence_after();
    __syncthreads();
    tstamp(a, 3);
    const bool go = ok && !s_abort;
    if (go && warp < 8) {
        const int q = warp & 3, g = warp >> 2;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        uint32_t xh_part[16], xl_part[16];
        tmem_ld16(taddr + 16 * g, xh_part);                  // columns r = 16 g .. + 16: the products with xh
        tmem_ld16(taddr + WIDE_ROWS + 16 * g, xl_part);      // the same rows' products with xl
        tmem_wait_ld();
        const int o = (q & 1) * 32 + lane;
        int64_t* dst = q < 2 ? HB : LB;
        const int64_t sh = q < 2 ? 65536 : 256, sl = q < 2 ? 256 : 1;
#pragma unroll
        for (int i = 0; i < 16; i++)
            dst[(16 * g + i) * 64 + o] = sh * (int64_t)(int32_t)xh_part[i] + sl * (int64_t)(int32_t)xl_part[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
    tstamp(a, 4);
    if (nz > 2) {
        // split K: P = H + L in place, then CTA kz of the cluster sums rows kz * 32 / nz .. of every CTA's P over DSMEM
        // and finishes them (warp w: row w % 8 of the slice, columns 32 (w / 8) + lane). Plain banks only.
        for (int i = tid; i < WIDE_ROWS * 64; i += WIDE_THREADS) HB[i] = (int64_t)((uint64_t)HB[i] + (uint64_t)LB[i]);
        cluster_sync();
        const int rs = WIDE_ROWS / nz, nl = kz * rs + (warp & 7), col = 32 * (warp >> 3) + lane;
        const int j = mt * 64 + col, n = r0 + nl;
        const bool live = (warp & 7) < rs && (warp >> 3) < 2 && n < a.rows && j < a.nout && go;
        int64_t w = 0;
        if (live) {
            const uint32_t off = saddr(HB + nl * 64 + col);
            uint64_t t[8];
#pragma unroll
            for (int p = 0; p < 8; p++) t[p] = p < nz ? (uint64_t)ld_dsmem(mapa(off, (uint32_t)p)) : 0;
            uint64_t sum = 0;
#pragma unroll
            for (int p = 0; p < 8; p++) sum += t[p];
            const int64_t colc = a.colcorr[j];
            const int64_t v = finish_value<EPI>(a, s_row[nl], n, j, (int64_t)sum, colc, (int64_t)a.epi.e[j], a.epi.b[j]);
            int64_t* o = a.epi.out + (size_t)s_row[nl].orow * a.epi.ldo + j;
            w = EPI == EPI_PLAIN_ADD ? wadd(QUANT ? pres : *o, v) : v;
            *o = w;
        }
        if (a.or_out && (warp & 7) < rs && (warp >> 3) < 2) {   // the next bank's row OR over these 32 columns
            const uint64_t wor = warp_or64(live ? mag(w) : 0);
            if (lane == 0 && n < a.rows && go) atomicOr((unsigned long long*)&a.or_out[n], (unsigned long long)wor);
        }
        tstamp(a, 5);
        cluster_sync();               // no CTA leaves while a peer may still read its P
        return;
    }

    if (nz == 2) {                    // P = H + L in place; the pair's tiles are complete after the barrier
        for (int i = tid; i < WIDE_ROWS * 64; i += WIDE_THREADS) HB[i] = (int64_t)((uint64_t)HB[i] + (uint64_t)LB[i]);
        cluster_sync();
    }

    // ---- finish: lane l columns 2l, 2l + 1 of the tile ----
    const bool jv0 = cv0 && go, jv1 = cv1 && go;
    int64_t v0[RPW], v1[RPW];
#pragma unroll
    for (int it = 0; it < RPW; it++) {
        v0[it] = 0;
        v1[it] = 0;
        if (it >= nrpw) break;
        const int nl = nz == 1 ? warp + 16 * it : 16 * kz + warp, n = r0 + nl;
        if (n < a.rows && (jv0 || jv1)) {
            uint64_t p0, p1;
            if (nz == 1) {
                const longlong2 h = *reinterpret_cast<const longlong2*>(HB + nl * 64 + 2 * lane);
                const longlong2 l = *reinterpret_cast<const longlong2*>(LB + nl * 64 + 2 * lane);
                p0 = (uint64_t)h.x + (uint64_t)l.x;
                p1 = (uint64_t)h.y + (uint64_t)l.y;
            } else {                      // this row's two partial tiles, over DSMEM
                const uint32_t off = saddr(HB + nl * 64 + 2 * lane);
                uint64_t a0, a1, c0, c1;
                ld_dsmem2(mapa(off, 0), a0, a1);
                ld_dsmem2(mapa(off, 1), c0, c1);
                p0 = a0 + c0;
                p1 = a1 + c1;
            }
            if (jv0) v0[it] = finish_value<EPI>(a, s_row[nl], n, j0, (int64_t)p0, colc0, e0, b0);
            if (jv1) v1[it] = finish_value<EPI>(a, s_row[nl], n, j1, (int64_t)p1, colc1, e1, b1);
        }
    }
    tstamp(a, 7);
    if (!heads) {
        int64_t old0[RPW], old1[RPW];
        if (EPI == EPI_PLAIN_ADD) {                  // the residual, read for every row before any store
#pragma unroll
            for (int it = 0; it < RPW; it++) {
                const int nl = nz == 1 ? warp + 16 * it : 16 * kz + warp, n = r0 + nl;
                if (QUANT) {
                    old0[it] = pre0[it];
                    old1[it] = pre1[it];
                    continue;
                }
                const int64_t* o = a.epi.out + (size_t)(n < a.rows ? s_row[nl].orow : 0) * a.epi.ldo + j0;
                old0[it] = n < a.rows && jv0 ? o[0] : 0;
                old1[it] = n < a.rows && jv1 ? o[1] : 0;
            }
        }
#pragma unroll
        for (int it = 0; it < RPW; it++) {
            if (it >= nrpw) break;
            const int nl = nz == 1 ? warp + 16 * it : 16 * kz + warp, n = r0 + nl;
            const bool rv = n < a.rows;
            const int64_t w0 = EPI == EPI_PLAIN_ADD ? wadd(old0[it], v0[it]) : v0[it];
            const int64_t w1 = EPI == EPI_PLAIN_ADD ? wadd(old1[it], v1[it]) : v1[it];
            if (rv) {
                int64_t* o = a.epi.out + (size_t)s_row[nl].orow * a.epi.ldo + j0;
                if (jv0) o[0] = w0;
                if (jv1) o[1] = w1;
            }
            if (a.or_out) {                          // the next bank's row OR over this tile's 64 columns
                const uint64_t wor = warp_or64(rv ? ((jv0 ? mag(w0) : 0) | (jv1 ? mag(w1) : 0)) : 0);
                if (lane == 0 && rv) atomicOr((unsigned long long*)&a.or_out[n], (unsigned long long)wor);
            }
        }
    } else {
#pragma unroll
        for (int it = 0; it < RPW; it++) {
            if (it >= nrpw) break;
            const int nl = nz == 1 ? warp + 16 * it : 16 * kz + warp, n = r0 + nl;
            const bool rv = n < a.rows && go;
            heads_row(a, mt, n, rv ? s_slot[nl] : 0, rv ? s_pos[nl] : 0, rv, v0[it], v1[it]);
        }
    }
    tstamp(a, 5);
    if (nz == 2) cluster_sync();     // no CTA leaves while its pair may still read its P
}

// ---------------------------------------------------------------------------------------------------------------------
// Many tiles (the head; prompt passes): a persistent loop over 128-column x 64-row tiles. TMEM holds two accumulator
// sets (columns 0 and 256) so the epilogue of one tile overlaps the loads and MMAs of the next; a ring of `stages`
// K blocks feeds the MMAs. 640 threads: warp 0 lane 0 = TMA, warp 1 lane 0 = MMA, warps 4-19 = epilogue (the int64
// epilogue is the bound, so it gets 16 warps: warp w reads TMEM lane quadrant w % 4, rows 16 * ((w - 4) / 4) .. + 16).
// ---------------------------------------------------------------------------------------------------------------------
constexpr int TILE_THREADS = 640;
template <int EPI>
__global__ void __launch_bounds__(TILE_THREADS, 1)
    k_bank_tiles(const __grid_constant__ CUtensorMap mwh, const __grid_constant__ CUtensorMap mwl,
                 const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl, const TcArgs a) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    constexpr int NEPI = 16;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full_bar[MAX_STAGES], empty_bar[MAX_STAGES], tfull[2], tempty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_dead;
    __shared__ RowData s_row[NEPI][16];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = a.stages, KB = a.kps;
    // one row tile (a decode step's head): each weight is read once, so it goes first from L2; prompt passes reuse
    // each weight tile across row tiles
    const uint64_t wpol = a.ntiles == 1 ? l2_evict_first() : l2_evict_normal();
    const int total = a.mtiles * a.ntiles;
    const int G = gridDim.x;
    tstamp(a, 0);
    const int my_tiles = blockIdx.x < total ? (total - blockIdx.x + G - 1) / G : 0;
    const int nkb = my_tiles * KB;
    const int npre = nkb < S ? nkb : S;

    if (tid == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], NEPI); }
        s_dead = (*(volatile uint32_t*)a.err & DERR_TIMEOUT) != 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const bool dead = s_dead != 0;
    if (tid == 0 && !dead) {          // the first weights: independent of earlier kernels
        for (int g = 0; g < npre; g++) {
            const int t = blockIdx.x + (g / KB) * G, kx = (g % KB) * 128;
            uint8_t* st = smem + g * STAGE;
            mbar_expect_tx(&full_bar[g], STAGE);
            tma_load_2d_hint(st, &mwh, &full_bar[g], kx, (t % a.mtiles) * 128, wpol);
            tma_load_2d_hint(st + A_BYTES, &mwl, &full_bar[g], kx, (t % a.mtiles) * 128, wpol);
        }
    }
    tstamp(a, 1);
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    tstamp(a, 2);
    if (dead) {
        // nothing was issued; fall through to the teardown
    } else if (warp == 0) {
        if (lane == 0) {
            for (int g = 0; g < nkb; g++) {
                const int s = g % S, t = blockIdx.x + (g / KB) * G, kx = (g % KB) * 128;
                const int mt = t % a.mtiles, nt = t / a.mtiles;
                uint8_t* st = smem + s * STAGE;
                if (g >= npre) {
                    if (!mbar_wait(&empty_bar[s], ((g / S) - 1) & 1, a.err)) break;
                    mbar_expect_tx(&full_bar[s], STAGE);
                    tma_load_2d_hint(st, &mwh, &full_bar[s], kx, mt * 128, wpol);
                    tma_load_2d_hint(st + A_BYTES, &mwl, &full_bar[s], kx, mt * 128, wpol);
                }
                tma_load_2d(st + 2 * A_BYTES, &mxh, &full_bar[s], kx, nt * BN);
                tma_load_2d(st + 2 * A_BYTES + B_BYTES, &mxl, &full_bar[s], kx, nt * BN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; i++) {
                const int b = i & 1;
                if (i >= 2 && !mbar_wait(&tempty[b], ((i >> 1) - 1) & 1, a.err)) break;
                tc_fence_after();
                for (int kk = 0; kk < KB; kk++) {
                    const int g = i * KB + kk, s = g % S;
                    if (!mbar_wait(&full_bar[s], (g / S) & 1, a.err)) { ok = false; break; }
                    tc_fence_after();
                    mma_kblock(saddr(smem + s * STAGE), tmem + b * 256, kk == 0);
                    mma_commit(&empty_bar[s]);
                }
                mma_commit(&tfull[b]);
            }
        }
    } else if (warp >= 4) {
        const int e = warp - 4, quad = warp & 3, r0 = (e >> 2) * 16;
        const uint32_t tq = (uint32_t)(quad * 32) << 16;
        for (int i = 0; i < my_tiles; i++) {
            const int b = i & 1, t = blockIdx.x + i * G;
            const int mt = t % a.mtiles, nt = t / a.mtiles;
            // this warp's 16 rows of the tile, staged per warp while the accumulators fill
            if (lane < 16) s_row[e][lane] = load_row<GAUGED>(a, nt * BN + r0 + lane);
            const int j = mt * 128 + quad * 32 + lane;
            const bool jv = j < a.nout;
            const int64_t colc = jv ? a.colcorr[j] : 0;
            const int64_t e_j = jv ? (int64_t)a.epi.e[j] : 0, b_j = jv ? a.epi.b[j] : 0;
            __syncwarp();
            if (!mbar_wait(&tfull[b], (i >> 1) & 1, a.err)) break;
            tc_fence_after();
            // four rows at a time (a rolled loop keeps the epilogue's code small: it runs once per tile per warp)
            const uint32_t tb = tmem + b * 256 + tq + r0;
#pragma unroll 1
            for (int q0 = 0; q0 < 16; q0 += 4) {
                int64_t p[4];
                int ix[4];
                tmem_piles4(tb + q0, p);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int q = q0 + u, n = nt * BN + r0 + q;
                    const bool ok = n < a.rows && jv;
                    if (a.race.v) {
                        // the race inside the epilogue (greedy decoding): the row's largest value over this warp's 32
                        // columns, ties to the lowest column (base2.py:114 argmax)
                        p[u] = ok ? finish_value<EPI>(a, s_row[e][q], n, j, p[u], colc, e_j, b_j) : INT64_MIN;
                        ix[u] = ok ? j : 0x7fffffff;
                        if (ok && a.epi.out) a.epi.out[(size_t)s_row[e][q].orow * a.epi.ldo + j] = p[u];
                    } else if (ok) {
                        finish<EPI>(a, s_row[e][q], n, j, p[u], colc, e_j, b_j);
                    }
                }
                if (a.race.v) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const int64_t ov = __shfl_xor_sync(0xffffffffu, p[u], o);
                            const int oi = __shfl_xor_sync(0xffffffffu, ix[u], o);
                            race_merge(p[u], ix[u], ov, oi);
                        }
                    }
                    if (lane < 4) {
                        const int64_t v = lane == 0 ? p[0] : lane == 1 ? p[1] : lane == 2 ? p[2] : p[3];
                        const int iv = lane == 0 ? ix[0] : lane == 1 ? ix[1] : lane == 2 ? ix[2] : ix[3];
                        const int n = nt * BN + r0 + q0 + lane;
                        if (n < a.rows) {
                            const size_t o = (size_t)n * a.race.ld + mt * 4 + quad;
                            a.race.v[o] = v;
                            a.race.i[o] = iv;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
    tstamp(a, 7);
}

// ---------------------------------------------------------------------------------------------------------------------
// Decode banks at <= 2 rows (batch-1 streams): a coalesced int16 GEMV on the CUDA cores over the reference-layout
// weights [nin][nout], the rows quantised in every CTA (a row of 768 inputs is 6 KB: converting it in each CTA costs
// less than any hand-off between CTAs, and nothing waits on another CTA). CTA (mt, kz) owns output columns
// 64 mt .. + 64 and inputs 768 kz .. + 768; a bank with more inputs is split over a (1, nin / 768, 1) cluster whose
// partial piles are summed over DSMEM by rank 0. 512 threads: thread t takes columns 8 (t % 8) .. + 8 and inputs
// 12 (t / 8) .. + 12 of the range; its 12 x 8 weights (one 16-byte load per input, eight threads reading one
// 128-byte row segment) are read BEFORE the dependency wait and held in registers. After the wait: the rows' x16 into
// shared memory (to16 by the OR the producer published; x16 = +32768 is an ordinary int32 here, no correction), S1 and
// S2 (gauged banks, whose 768 inputs are one CTA's), the exact products summed in int64 (|x16 w| <= 2^30), a shuffle
// and shared-memory reduction over the 64 input slices, then the bank's epilogue with warp r on row r, lane l on
// columns 2l, 2l + 1 (the qkv bank's 64 columns are one head part: heads16's OR is one warp's).
// ---------------------------------------------------------------------------------------------------------------------
constexpr int GEMV_THREADS = 512;
constexpr int GEMV_KR = 768;          // inputs per CTA
constexpr int GEMV_MAX_ROWS = 2;

template <int EPI, int R>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_bank_gemv(const TcArgs a) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    __shared__ int32_t xs[R][GEMV_KR];                // the rows' x16 over this CTA's inputs
    __shared__ int64_t red[GEMV_THREADS / 32][64][R]; // per-warp partial piles
    __shared__ int64_t s_pile[R][64];                 // this CTA's piles (read by rank 0 of a K split over DSMEM)
    __shared__ int64_t s_1[GEMV_THREADS / 32][R], s_2[GEMV_THREADS / 32][R];
    __shared__ int32_t s_sh[R];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, kz = blockIdx.y, nz = gridDim.y;
    const int cg = tid & 7, ks = tid >> 3;
    const int k0 = kz * GEMV_KR + ks * 12;            // this thread's first input
    const int c0 = mt * 64 + cg * 8;                  // its first column
    const bool cvalid = c0 < a.nout;                  // nout % 8 == 0: a column group is all in or all out
    // the weights, independent of earlier kernels
    int4 w[12];
#pragma unroll
    for (int u = 0; u < 12; u++)
        w[u] = cvalid ? __ldg(reinterpret_cast<const int4*>(a.w16 + (size_t)(k0 + u) * a.nout + c0)) : make_int4(0, 0, 0, 0);
    const int j0 = mt * 64 + 2 * lane, j1 = j0 + 1;  // the epilogue's columns (warp r < R: row r)
    const bool cv0 = j0 < a.nout, cv1 = j1 < a.nout;
    const int64_t e0 = cv0 ? (int64_t)a.epi.e[j0] : 0, b0 = cv0 ? a.epi.b[j0] : 0;
    const int64_t e1 = cv1 ? (int64_t)a.epi.e[j1] : 0, b1 = cv1 ? a.epi.b[j1] : 0;
    const bool heads = (EPI == EPI_GAUGED || EPI == EPI_PLAIN_OUT) && a.heads;
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();

    // ---- the rows' x16 over this CTA's inputs; S1, S2 over the row (gauged banks: the CTA holds the whole row) ----
    if (tid < R) s_sh[tid] = tid < a.rows ? to16_shift(a.q.xor_in[tid]) : 0;
    __syncthreads();
    int64_t p1[R], p2[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        p1[r] = 0;
        p2[r] = 0;
        const int sh = s_sh[r];
        for (int i = tid; i < GEMV_KR; i += GEMV_THREADS) {
            int32_t x = 0;
            if (r < a.rows) {
                const int64_t v = a.q.X[(size_t)r * a.q.ldx + kz * GEMV_KR + i];
                x = (int32_t)(sh ? (int64_t)((uint64_t)v + (1ull << (sh - 1))) >> sh : v);
            }
            xs[r][i] = x;
            p1[r] += x;
            p2[r] += (int64_t)x * x;
        }
        if (GAUGED) {
            p1[r] = warp_sum64(p1[r]);
            p2[r] = warp_sum64(p2[r]);
            if (lane == 0) {
                s_1[warp][r] = p1[r];
                s_2[warp][r] = p2[r];
            }
        }
    }
    __syncthreads();

    // ---- the products: 12 inputs x 8 columns x R rows per thread ----
    int64_t acc[R][8];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int c = 0; c < 8; c++) acc[r][c] = 0;
#pragma unroll
    for (int u = 0; u < 12; u++) {
        const int32_t wv[8] = {(int16_t)(w[u].x & 0xFFFF), (int16_t)((uint32_t)w[u].x >> 16),
                               (int16_t)(w[u].y & 0xFFFF), (int16_t)((uint32_t)w[u].y >> 16),
                               (int16_t)(w[u].z & 0xFFFF), (int16_t)((uint32_t)w[u].z >> 16),
                               (int16_t)(w[u].w & 0xFFFF), (int16_t)((uint32_t)w[u].w >> 16)};
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int32_t x = xs[r][ks * 12 + u];
#pragma unroll
            for (int c = 0; c < 8; c++) acc[r][c] += (int64_t)x * wv[c];
        }
    }
    // over the warp's four input slices (lanes cg, cg + 8, cg + 16, cg + 24), then over the 16 warps
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int c = 0; c < 8; c++) {
            acc[r][c] += __shfl_xor_sync(0xffffffffu, acc[r][c], 8);
            acc[r][c] += __shfl_xor_sync(0xffffffffu, acc[r][c], 16);
        }
    if (lane < 8) {
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int c = 0; c < 8; c++) red[warp][lane * 8 + c][r] = acc[r][c];
    }
    __syncthreads();
    if (tid < 64 * R) {
        const int col = tid & 63, r = tid >> 6;
        int64_t s = 0;
#pragma unroll
        for (int q = 0; q < GEMV_THREADS / 32; q++) s += red[q][col][r];
        s_pile[r][col] = s;
    }
    __syncthreads();
    if (nz > 1) cluster_sync();       // every CTA's piles are in place
    if (kz == 0 && warp < R && warp < a.rows) {
        const int r = warp;
        int64_t P0 = s_pile[r][2 * lane], P1 = s_pile[r][2 * lane + 1];
        for (int p = 1; p < nz; p++) {
            P0 += ld_dsmem(mapa(saddr(&s_pile[r][2 * lane]), (uint32_t)p));
            P1 += ld_dsmem(mapa(saddr(&s_pile[r][2 * lane + 1]), (uint32_t)p));
        }
        const int64_t ex = -16 + s_sh[r];
        int64_t LS = 0, e2 = 0;
        if (GAUGED) {
            int64_t S1 = 0, S2 = 0;
#pragma unroll
            for (int q = 0; q < GEMV_THREADS / 32; q++) {
                S1 = wadd(S1, s_1[q][r]);
                S2 = wadd(S2, s_2[q][r]);
            }
            LS = gauge_LS(S1, S2, (int)ex, a.q.LOG2, a.q.log768, a.q.eps40);
            e2 = __ldg(a.epi.EXP2 + (wsub(0, LS) & 0xFFFF));
        }
        const int64_t v0 = cv0 ? epi_value<EPI>(P0, e0, b0, ex, LS, e2, a.epi.PHI) : 0;
        const int64_t v1 = cv1 ? epi_value<EPI>(P1, e1, b1, ex, LS, e2, a.epi.PHI) : 0;
        if (!heads) {
            int64_t* o = a.epi.out + (size_t)r * a.epi.ldo + j0;
            const int64_t w0 = EPI == EPI_PLAIN_ADD && cv0 ? wadd(o[0], v0) : v0;
            const int64_t w1 = EPI == EPI_PLAIN_ADD && cv1 ? wadd(o[1], v1) : v1;
            if (cv0) o[0] = w0;
            if (cv1) o[1] = w1;
            if (a.or_out) {                          // the next bank's row OR over these 64 columns
                const uint64_t wor = warp_or64((cv0 ? mag(w0) : 0) | (cv1 ? mag(w1) : 0));
                if (lane == 0) atomicOr((unsigned long long*)&a.or_out[r], (unsigned long long)wor);
            }
        } else {
            heads_row(a, mt, r, a.hd.row_slot[r], a.hd.row_pos[r], true, v0, v1);
        }
    }
    if (nz > 1) cluster_sync();       // no CTA leaves while rank 0 may still read its piles
}

// ---------------------------------------------------------------------------------------------------------------------
// Layer 0's qkv bank of a decode step from stored rows (the reference's stored layer-0 entry: base2_entry.py,
// base2_layer0.py; Metal carry0 / entry_gate1 / entry_add1, base2_stream_fr2.swift:407-428). A decode row is
// x = wte[word] + wpe[position]; when every embedded value is below 2^15 in magnitude (checked when the tables are
// built) to16 keeps x as it is (shift 0), so the pile is exactly Tw[word] + Tp[position], Tw = wte . W and Tp = wpe . W
// computed once (the product is linear; the reference's carry, the rounding of a sum against the sum of roundings, is
// zero at shift 0). The row's S1 and S2 for the gauge come from x itself. One CTA of 16 warps per row: the block sums,
// then warp w takes head parts w, w + 16, w + 32 (64 columns each, lane l columns 2l, 2l + 1) through the gauged
// epilogue and heads_row.
// ---------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) k_entry_qkv(const TcArgs a, const int64_t* __restrict__ Tw,
                                                    const int64_t* __restrict__ Tp, const int32_t* __restrict__ row_tok,
                                                    const int64_t* __restrict__ wte, const int64_t* __restrict__ wpe,
                                                    int vocab, int nctx) {
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    __shared__ int64_t s_1[16], s_2[16];
    const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tok = row_tok[r], pos = a.hd.row_pos[r], slot = a.hd.row_slot[r];
    const bool ok = tok >= 0 && tok < vocab && pos >= 0 && pos < nctx;   // otherwise flagged by the embedding kernel
    const int d = a.nin, nout = a.nout;
    int64_t p1 = 0, p2 = 0;
    if (ok)
        for (int i = tid; i < d; i += 512) {
            const int64_t x = wte[(size_t)tok * d + i] + wpe[(size_t)pos * d + i];
            p1 += x;
            p2 += x * x;
        }
    p1 = warp_sum64(p1);
    p2 = warp_sum64(p2);
    if (lane == 0) {
        s_1[warp] = p1;
        s_2[warp] = p2;
    }
    __syncthreads();
    int64_t S1 = 0, S2 = 0;
#pragma unroll
    for (int q = 0; q < 16; q++) {
        S1 = wadd(S1, s_1[q]);
        S2 = wadd(S2, s_2[q]);
    }
    const int64_t ex = -16;                           // shift 0
    const int64_t LS = gauge_LS(S1, S2, (int)ex, a.q.LOG2, a.q.log768, a.q.eps40);
    const int64_t e2 = __ldg(a.epi.EXP2 + (wsub(0, LS) & 0xFFFF));
    for (int part = warp; part * 64 < nout; part += 16) {
        const int j0 = part * 64 + 2 * lane;
        const bool c0 = j0 < nout, c1 = j0 + 1 < nout;
        int64_t v0 = 0, v1 = 0;
        if (ok && c0) {
            const int64_t P0 = Tw[(size_t)tok * nout + j0] + Tp[(size_t)pos * nout + j0];
            v0 = epi_value<EPI_GAUGED>(P0, (int64_t)a.epi.e[j0], a.epi.b[j0], ex, LS, e2, a.epi.PHI);
        }
        if (ok && c1) {
            const int64_t P1 = Tw[(size_t)tok * nout + j0 + 1] + Tp[(size_t)pos * nout + j0 + 1];
            v1 = epi_value<EPI_GAUGED>(P1, (int64_t)a.epi.e[j0 + 1], a.epi.b[j0 + 1], ex, LS, e2, a.epi.PHI);
        }
        heads_row(a, part, r, slot, pos, ok, v0, v1);
    }
}

// the largest |x| over n int64 values (atomicMax into *out, which starts at 0)
__global__ void k_absmax(const int64_t* __restrict__ x, size_t n, unsigned long long* out) {
    uint64_t m = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = max(m, mag(x[i]));
    m = warp_max_u64(m);
    if ((threadIdx.x & 31) == 0) atomicMax(out, (unsigned long long)m);
}

// ---------------------------------------------------------------------------------------------------------------------
// The head of a decode step of <= 2 rows as a CUDA-core GEMV over the weights stored as 64-column tiles
// ([tile][768][64] int16, each tile one contiguous 96 KB block, so the reads stream through DRAM in order):
// persistent CTAs (one an SM) walk the tiles, each brought into shared memory by three TMA boxes (64 columns x 256
// rows) through a two-stage ring, the first two, and the columns' exponents and biases, before the dependency wait.
// The CTA reads its rows
// whole (768 values) and quantises them itself (OR, to16, S1 and S2 for the gauge); per tile thread t multiplies
// columns 8 (t % 8) .. + 8 over inputs 12 (t / 8) .. + 12 (exact int64 piles), the 64 input slices are summed by
// shuffles and shared memory, and warp r forms row r's values and races each 32-column group (ties to the lowest
// column, base2.py:114) into the race buffer k_race_parts reads. Every wait on the ring is bounded and agreed on by
// the whole CTA (a timeout ends the CTA's loop, flagged, after the copies in flight have landed or a bound passed).
// ---------------------------------------------------------------------------------------------------------------------
constexpr int HG_BOX_ROWS = 256;
constexpr int HG_TILE = GEMV_KR * 64;             // int16 of one tile
constexpr int HG_TILE_BYTES = HG_TILE * 2;        // 98,304
constexpr size_t HG_SMEM = 2 * (size_t)HG_TILE_BYTES + 128;
constexpr int HG_PRE = 8;                         // tiles per CTA whose exponents and biases are staged in shared memory

template <int EPI, int R>
__global__ void __launch_bounds__(GEMV_THREADS, 1)
    k_head_gemv(const __grid_constant__ CUtensorMap mw, const TcArgs a, const TcRace race) {
    constexpr bool GAUGED = EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE;
    extern __shared__ uint8_t smem_raw[];
    int16_t* W = reinterpret_cast<int16_t*>(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);   // [2][768][64]
    __shared__ uint64_t full[2];
    __shared__ int32_t xs[R][GEMV_KR];
    __shared__ int64_t red[GEMV_THREADS / 32][64][R];
    __shared__ int64_t s_pile[R][64];
    __shared__ uint64_t s_or[GEMV_THREADS / 32][R];
    __shared__ int64_t s_1[GEMV_THREADS / 32][R], s_2[GEMV_THREADS / 32][R];
    __shared__ int32_t s_e[HG_PRE][64];
    __shared__ int64_t s_b[HG_PRE][64];
    __shared__ int s_dead;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cg = tid & 7, ks = tid >> 3;
    const int ntiles = (a.nout + 63) / 64, G = gridDim.x;
    const int my = (int)blockIdx.x < ntiles ? (ntiles - (int)blockIdx.x + G - 1) / G : 0;
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        s_dead = (*(volatile uint32_t*)a.err & DERR_TIMEOUT) != 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int nissue = s_dead ? 0 : my;
    if (tid == 0) {                   // the first two tiles' weights: independent of earlier kernels
        const uint64_t pol = l2_evict_first();
        for (int s = 0; s < 2 && s < nissue; s++) {
            const int tile = blockIdx.x + s * G;
            mbar_expect_tx(&full[s], HG_TILE_BYTES);
            for (int bx = 0; bx < GEMV_KR / HG_BOX_ROWS; bx++)
                tma_load_2d_hint(W + (size_t)s * HG_TILE + bx * HG_BOX_ROWS * 64, &mw, &full[s], 0,
                                 tile * GEMV_KR + bx * HG_BOX_ROWS, pol);
        }
    }
    for (int q = tid; q < HG_PRE * 64; q += GEMV_THREADS) {     // the columns' exponents and biases (read-only inputs)
        const int t = q >> 6, j = (blockIdx.x + t * G) * 64 + (q & 63);
        const bool v = t < my && j < a.nout;
        s_e[t][q & 63] = v ? __ldg(a.epi.e + j) : 0;
        s_b[t][q & 63] = v ? __ldg(a.epi.b + j) : 0;
    }
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();

    // ---- the rows: OR, to16 shift, x16, S1, S2 ----
#pragma unroll
    for (int r = 0; r < R; r++) {
        uint64_t o = 0;
        if (r < a.rows)
            for (int i = tid; i < GEMV_KR; i += GEMV_THREADS) o |= mag(a.q.X[(size_t)r * a.q.ldx + i]);
        o = warp_or64(o);
        if (lane == 0) s_or[warp][r] = o;
    }
    __syncthreads();
    int sh[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        uint64_t all = 0;
#pragma unroll
        for (int q = 0; q < GEMV_THREADS / 32; q++) all |= s_or[q][r];
        sh[r] = to16_shift(all);
        int64_t p1 = 0, p2 = 0;
        for (int i = tid; i < GEMV_KR; i += GEMV_THREADS) {
            int32_t x = 0;
            if (r < a.rows) x = (int32_t)rshift(a.q.X[(size_t)r * a.q.ldx + i], sh[r]);
            xs[r][i] = x;
            p1 += x;
            p2 += (int64_t)x * x;
        }
        if (GAUGED) {
            p1 = warp_sum64(p1);
            p2 = warp_sum64(p2);
            if (lane == 0) {
                s_1[warp][r] = p1;
                s_2[warp][r] = p2;
            }
        }
    }
    __syncthreads();
    // the epilogue's row constants (warp r < R forms row r)
    const int er = warp < R ? warp : 0;
    const int64_t ex = -16 + sh[er];
    int64_t LS = 0, e2 = 0;
    if (GAUGED && warp < R && warp < a.rows) {
        int64_t S1 = 0, S2 = 0;
#pragma unroll
        for (int q = 0; q < GEMV_THREADS / 32; q++) {
            S1 = wadd(S1, s_1[q][er]);
            S2 = wadd(S2, s_2[q][er]);
        }
        LS = gauge_LS(S1, S2, (int)ex, a.q.LOG2, a.q.log768, a.q.eps40);
        e2 = __ldg(a.epi.EXP2 + (wsub(0, LS) & 0xFFFF));
    }

    int it = 0;
    for (; it < nissue; it++) {
        const int s = it & 1, tile = blockIdx.x + it * G;
        const bool got = mbar_wait(&full[s], (it >> 1) & 1, a.err);
        if (__syncthreads_or(!got)) break;       // a wait that gave up ends every thread's loop (flagged)
        const int16_t* Ws = W + (size_t)s * HG_TILE;
        int64_t acc[R][8];
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int c = 0; c < 8; c++) acc[r][c] = 0;
#pragma unroll
        for (int u = 0; u < 12; u++) {
            const int4 w = *reinterpret_cast<const int4*>(Ws + (ks * 12 + u) * 64 + cg * 8);
            const int32_t wv[8] = {(int16_t)(w.x & 0xFFFF), (int16_t)((uint32_t)w.x >> 16),
                                   (int16_t)(w.y & 0xFFFF), (int16_t)((uint32_t)w.y >> 16),
                                   (int16_t)(w.z & 0xFFFF), (int16_t)((uint32_t)w.z >> 16),
                                   (int16_t)(w.w & 0xFFFF), (int16_t)((uint32_t)w.w >> 16)};
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int32_t x = xs[r][ks * 12 + u];
#pragma unroll
                for (int c = 0; c < 8; c++) acc[r][c] += (int64_t)x * wv[c];
            }
        }
        // over the warp's four input slices (lanes cg, cg + 8, cg + 16, cg + 24), then over the 16 warps
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int c = 0; c < 8; c++) {
                acc[r][c] += __shfl_xor_sync(0xffffffffu, acc[r][c], 8);
                acc[r][c] += __shfl_xor_sync(0xffffffffu, acc[r][c], 16);
            }
        if (lane < 8) {
#pragma unroll
            for (int r = 0; r < R; r++)
#pragma unroll
                for (int c = 0; c < 8; c++) red[warp][lane * 8 + c][r] = acc[r][c];
        }
        __syncthreads();                         // the partial piles are in; every thread is done with stage s
        if (tid == 0 && it + 2 < nissue) {       // refill stage s with the tile after next
            const int nt = blockIdx.x + (it + 2) * G;
            mbar_expect_tx(&full[s], HG_TILE_BYTES);
            for (int bx = 0; bx < GEMV_KR / HG_BOX_ROWS; bx++)
                tma_load_2d_hint(W + (size_t)s * HG_TILE + bx * HG_BOX_ROWS * 64, &mw, &full[s], 0,
                                 nt * GEMV_KR + bx * HG_BOX_ROWS, l2_evict_first());
        }
        if (tid < 64 * R) {
            const int col = tid & 63, r = tid >> 6;
            int64_t v = 0;
#pragma unroll
            for (int q = 0; q < GEMV_THREADS / 32; q++) v += red[q][col][r];
            s_pile[r][col] = v;
        }
        __syncthreads();
        if (warp < R && warp < a.rows) {
            const int r = warp, j0 = tile * 64 + 2 * lane, j1 = j0 + 1;
            const bool cv0 = j0 < a.nout, cv1 = j1 < a.nout;
            const bool pre = it < HG_PRE;
            const int64_t e0 = !cv0 ? 0 : pre ? (int64_t)s_e[it][2 * lane] : (int64_t)a.epi.e[j0];
            const int64_t e1 = !cv1 ? 0 : pre ? (int64_t)s_e[it][2 * lane + 1] : (int64_t)a.epi.e[j1];
            const int64_t b0 = !cv0 ? 0 : pre ? s_b[it][2 * lane] : a.epi.b[j0];
            const int64_t b1 = !cv1 ? 0 : pre ? s_b[it][2 * lane + 1] : a.epi.b[j1];
            const int64_t v0 = cv0 ? epi_value<EPI>(s_pile[r][2 * lane], e0, b0, ex, LS, e2, a.epi.PHI) : 0;
            const int64_t v1 = cv1 ? epi_value<EPI>(s_pile[r][2 * lane + 1], e1, b1, ex, LS, e2, a.epi.PHI) : 0;
            if (a.epi.out) {
                int64_t* op = a.epi.out + (size_t)r * a.epi.ldo + j0;
                if (cv0) op[0] = v0;
                if (cv1) op[1] = v1;
            }
            int64_t bv = cv0 ? v0 : INT64_MIN;
            int bi = cv0 ? j0 : 0x7fffffff;
            if (cv1) race_merge(bv, bi, v1, j1);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) {
                const int64_t ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                race_merge(bv, bi, ov, oi);
            }
            if ((lane & 15) == 0) {              // lanes 0-15: the tile's columns 0-31, lanes 16-31: 32-63
                const size_t q = (size_t)r * race.ld + tile * 2 + (lane >> 4);
                race.v[q] = bv;
                race.i[q] = bi;
            }
        }
    }
    if (it < nissue && tid == 0) {     // gave up: let the copies still in flight land (bounded) before the CTA leaves
        const uint64_t t0 = gtime(), lim = wait_limit(a.err);
        for (int j = it; j < nissue && j < it + 2; j++)
            while (!mbar_try_wait(&full[j & 1], (j >> 1) & 1) && gtime() - t0 <= lim) {
            }
    }
}

// ---- weight planes: [nin][nout] int16 -> [nout_pad][nin] wh, wl (transposed through shared memory) ----
__global__ void k_weight_planes(const int16_t* __restrict__ w, int nin, int nout, int8_t* __restrict__ wh,
                                int8_t* __restrict__ wl) {
    __shared__ int16_t t[32][33];
    const int j0 = blockIdx.x * 32, i0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    for (int r = ty; r < 32; r += 8) {
        int i = i0 + r, j = j0 + tx;
        t[r][tx] = (i < nin && j < nout) ? w[(size_t)i * nout + j] : (int16_t)0;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        int j = j0 + r, i = i0 + tx;
        if (i < nin) {
            int v = t[tx][r];
            wh[(size_t)j * nin + i] = (int8_t)(v >> 8);
            wl[(size_t)j * nin + i] = (int8_t)((v & 255) - 128);
        }
    }
}

__global__ void k_colcorr(const int16_t* __restrict__ w, int nin, int nout, int nout_pad, int64_t* __restrict__ cc) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= nout_pad) return;
    int64_t s = 0;
    if (j < nout)
        for (int i = 0; i < nin; i++) s += w[(size_t)i * nout + j];
    cc[j] = j < nout ? 128 * s - 16384 * (int64_t)nin : 0;
}

// per 128-input block: 128 * sum_{i in block} w[i][j] - 16384 * 128 (a CTA over part of the K range adds its blocks' share)
__global__ void k_colcorr_kb(const int16_t* __restrict__ w, int nin, int nout, int nout_pad, int64_t* __restrict__ cc) {
    int j = blockIdx.x * blockDim.x + threadIdx.x, kb = blockIdx.y;
    if (j >= nout_pad) return;
    int64_t s = 0;
    if (j < nout)
        for (int i = kb * 128; i < kb * 128 + 128; i++) s += w[(size_t)i * nout + j];
    cc[(size_t)kb * nout_pad + j] = j < nout ? 128 * s - 16384 * 128 : 0;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 2-D byte tensor [outer][inner] (row stride ld bytes), box = 128 bytes x box_outer rows, SWIZZLE_128B
int make_map(TcMap& m, void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) return (int)cudaErrorNotSupported;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {128, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(reinterpret_cast<CUtensorMap*>(m.bytes), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// 2-D int16 tensor [outer][inner] (row stride ld elements, a multiple of 8; mapped as uint16, a copy of the bits), box
// 64 x 256, no swizzle (k_head_gemv's tiles: inner 64, outer tiles x 768)
int make_map16(TcMap& m, void* base, uint64_t inner, uint64_t outer, uint64_t ld) {
    auto fn = encode_fn();
    if (!fn) return (int)cudaErrorNotSupported;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)HG_BOX_ROWS};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(reinterpret_cast<CUtensorMap*>(m.bytes), CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

template <class K>
cudaError_t launch_k(K kernel, dim3 grid, dim3 block, size_t smem, int cluster_y, cudaStream_t st, bool pdl,
                     const TcBank& t, const TcMap& xh, const TcMap& xl, const TcArgs& a, bool w64 = false) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (cluster_y > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = cluster_y;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, *reinterpret_cast<const CUtensorMap*>((w64 ? t.map_wh64 : t.map_wh).bytes),
                              *reinterpret_cast<const CUtensorMap*>((w64 ? t.map_wl64 : t.map_wl).bytes),
                              *reinterpret_cast<const CUtensorMap*>(xh.bytes), *reinterpret_cast<const CUtensorMap*>(xl.bytes), a);
}

// a kernel that takes only TcArgs (k_bank_gemv), as a cluster (1, cluster_y, 1) when cluster_y > 1
template <class K>
cudaError_t launch_args(K kernel, dim3 grid, dim3 block, int cluster_y, cudaStream_t st, bool pdl, const TcArgs& a) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (cluster_y > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = cluster_y;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

#define B2_EPI_SWITCH(EPIV, CALL)                                      \
    switch (EPIV) {                                                    \
        case EPI_GAUGED: { constexpr int E = EPI_GAUGED; CALL; }           \
        case EPI_GAUGED_EDGE: { constexpr int E = EPI_GAUGED_EDGE; CALL; } \
        case EPI_PLAIN_ADD: { constexpr int E = EPI_PLAIN_ADD; CALL; }     \
        case EPI_PLAIN_EDGE: { constexpr int E = EPI_PLAIN_EDGE; CALL; }   \
        default: { constexpr int E = EPI_PLAIN_OUT; CALL; }                \
    }

}  // namespace

int tc_min_rows_default() { return 1; }

// decode banks with nin <= 768: k_bank_wide (1, default) or the split-K cluster kernel (B2_WIDE=0)
static int tc_wide = 1;
// k_bank_wide's CTAs of a row half wait for one another (arrival counter), so a launch must fit on the GPU at once.
// Per device (filled by tc_init with that device current): how many k_bank_wide CTAs can be resident at once when
// launched as clusters of 1, 2 or 4 (cudaOccupancyMaxActiveClusters at the kernel's largest shared memory, so GPC
// partitioning is accounted for, not just the SM count).
constexpr int TC_MAX_DEVICES = 64;
struct WideCaps {
    int ready = 0;
    int ctas[MAX_SPLIT + 1] = {0};
};
static WideCaps tc_caps[TC_MAX_DEVICES];
static std::mutex tc_caps_mu;
static const WideCaps& wide_caps() {
    static const WideCaps none{};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= TC_MAX_DEVICES) return none;
    return tc_caps[dev];
}
// the in-kernel-quantising decode banks split a 768-input bank over this many CTAs when the launch still fits
// (2: half the K blocks, MMAs, quantisation and finish per CTA, one DSMEM pair sum; 1: B2_WIDE_KZ=1)
static int tc_wide_kz = 2;
// decode banks at <= 2 rows run the CUDA-core GEMV (k_bank_gemv) instead of k_bank_wide (B2_GEMV=0: k_bank_wide)
static int tc_gemv = 1;

// shared-memory and cluster opt-ins for every instantiation, once, before any launch (never inside a capture)
int tc_init() {
    if (const char* v = getenv("B2_WIDE")) tc_wide = atoi(v);
    if (const char* v = getenv("B2_WIDE_KZ")) tc_wide_kz = atoi(v);
    if (const char* v = getenv("B2_GEMV")) tc_gemv = atoi(v);
    void* split[] = {(void*)k_bank_split<EPI_GAUGED>, (void*)k_bank_split<EPI_GAUGED_EDGE>,
                     (void*)k_bank_split<EPI_PLAIN_ADD>, (void*)k_bank_split<EPI_PLAIN_OUT>,
                     (void*)k_bank_split<EPI_PLAIN_EDGE>};
    void* tiles[] = {(void*)k_bank_tiles<EPI_GAUGED>, (void*)k_bank_tiles<EPI_GAUGED_EDGE>,
                     (void*)k_bank_tiles<EPI_PLAIN_ADD>, (void*)k_bank_tiles<EPI_PLAIN_OUT>,
                     (void*)k_bank_tiles<EPI_PLAIN_EDGE>};
    for (void* f : split) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_KPS * STAGE + 1024);
        if (e != cudaSuccess) return (int)e;
    }
    for (void* f : tiles) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_STAGES * STAGE + 1024);
        if (e != cudaSuccess) return (int)e;
    }
    void* wide[] = {(void*)k_bank_wide<EPI_GAUGED, false>,     (void*)k_bank_wide<EPI_GAUGED_EDGE, false>,
                    (void*)k_bank_wide<EPI_PLAIN_ADD, false>,  (void*)k_bank_wide<EPI_PLAIN_OUT, false>,
                    (void*)k_bank_wide<EPI_PLAIN_EDGE, false>, (void*)k_bank_wide<EPI_GAUGED, true>,
                    (void*)k_bank_wide<EPI_GAUGED_EDGE, true>, (void*)k_bank_wide<EPI_PLAIN_ADD, true>,
                    (void*)k_bank_wide<EPI_PLAIN_OUT, true>,   (void*)k_bank_wide<EPI_PLAIN_EDGE, true>};
    for (void* f : wide) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, wide_smem_bytes(WIDE_MAX_KB));
        if (e != cudaSuccess) return (int)e;
    }
    void* heads[] = {(void*)k_head_gemv<EPI_GAUGED, 1>, (void*)k_head_gemv<EPI_GAUGED, 2>,
                     (void*)k_head_gemv<EPI_PLAIN_OUT, 1>, (void*)k_head_gemv<EPI_PLAIN_OUT, 2>};
    for (void* f : heads) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)HG_SMEM);
        if (e != cudaSuccess) return (int)e;
    }
    // this device's co-residency for k_bank_wide launches (cluster sizes 1, 2, 4)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= TC_MAX_DEVICES) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(tc_caps_mu);
    if (!tc_caps[dev].ready) {
        WideCaps c{};
        for (int cz = 1; cz <= 4; cz *= 2) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(1, cz, 1);
            cfg.blockDim = dim3(WIDE_THREADS);
            cfg.dynamicSmemBytes = wide_smem_bytes(WIDE_MAX_KB);
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 1;
            at[0].val.clusterDim.y = cz;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int nc = 0;
            e = cudaOccupancyMaxActiveClusters(&nc, (void*)k_bank_wide<EPI_PLAIN_ADD, true>, &cfg);
            if (e != cudaSuccess) return (int)e;
            c.ctas[cz] = nc * cz;
        }
        c.ready = 1;
        tc_caps[dev] = c;
    }
    return 0;
}

static int tc_bank_alloc(TcBank& t, int nin, int nout) {
    tc_bank_free(t);
    if (nin % 128) return (int)cudaErrorInvalidValue;
    t.nin = nin;
    t.nout = nout;
    t.nout_pad = (nout + 127) / 128 * 128;
    cudaError_t e;
    if ((e = cudaMalloc(&t.wh, (size_t)t.nout_pad * nin)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&t.wl, (size_t)t.nout_pad * nin)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&t.colcorr, sizeof(int64_t) * t.nout_pad)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&t.colcorr_kb, sizeof(int64_t) * t.nout_pad * (nin / 128))) != cudaSuccess) return (int)e;
    return 0;
}

int tc_bank_upload(TcBank& t, int nin, int nout, const int8_t* wh, const int8_t* wl, const int64_t* cc, const int64_t* cckb) {
    int rc = tc_bank_alloc(t, nin, nout);
    if (rc) return rc;
    const size_t np = (size_t)t.nout_pad;
    cudaError_t e;
    if ((e = cudaMemcpy(t.wh, wh, np * nin, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(t.wl, wl, np * nin, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(t.colcorr, cc, sizeof(int64_t) * np, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(t.colcorr_kb, cckb, sizeof(int64_t) * np * (nin / 128), cudaMemcpyHostToDevice)) != cudaSuccess)
        return (int)e;
    t.prebuilt = 1;
    return 0;
}

int tc_bank_download(const TcBank& t, int8_t* wh, int8_t* wl, int64_t* cc, int64_t* cckb) {
    if (!t.ready) return (int)cudaErrorInvalidValue;
    const size_t np = (size_t)t.nout_pad;
    cudaError_t e;
    if ((e = cudaMemcpy(wh, t.wh, np * t.nin, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(wl, t.wl, np * t.nin, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(cc, t.colcorr, sizeof(int64_t) * np, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(cckb, t.colcorr_kb, sizeof(int64_t) * np * (t.nin / 128), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return (int)e;
    return 0;
}

int tc_bank_build(TcBank& t, const int16_t* w, int nin, int nout) {
    cudaError_t e;
    if (!(t.prebuilt && t.nin == nin && t.nout == nout)) {   // no uploaded layout: build it from w on the device
        int rc = tc_bank_alloc(t, nin, nout);
        if (rc) return rc;
        k_weight_planes<<<dim3(t.nout_pad / 32, (nin + 31) / 32), dim3(32, 8)>>>(w, nin, nout, t.wh, t.wl);
        k_colcorr<<<(t.nout_pad + 255) / 256, 256>>>(w, nin, nout, t.nout_pad, t.colcorr);
        k_colcorr_kb<<<dim3((t.nout_pad + 255) / 256, nin / 128), 256>>>(w, nin, nout, t.nout_pad, t.colcorr_kb);
        if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;
    }
    t.w16 = w;
    if (t.wt) cudaFree(t.wt);
    t.wt = nullptr;
    t.map_w16_ok = 0;
    if (nout > 4096 && nin == GEMV_KR) {      // a head: the GEMV head's copy, 64-column tiles each one contiguous block
        const int nt = (nout + 63) / 64;
        const size_t tile = (size_t)nin * 64;
        if ((e = cudaMalloc(&t.wt, sizeof(int16_t) * tile * nt)) != cudaSuccess) return (int)e;
        if ((e = cudaMemset(t.wt, 0, sizeof(int16_t) * tile * nt)) != cudaSuccess) return (int)e;
        for (int q = 0; q < nt; q++) {
            const int wc = nout - q * 64 < 64 ? nout - q * 64 : 64;
            if ((e = cudaMemcpy2D(t.wt + q * tile, sizeof(int16_t) * 64, w + (size_t)q * 64, sizeof(int16_t) * nout,
                                  sizeof(int16_t) * wc, nin, cudaMemcpyDeviceToDevice)) != cudaSuccess)
                return (int)e;
        }
        if (make_map16(t.map_w16, t.wt, 64, (uint64_t)nt * nin, 64) == 0) t.map_w16_ok = 1;
    }
    int rc = make_map(t.map_wh, t.wh, nin, t.nout_pad, nin, 128);
    if (!rc) rc = make_map(t.map_wl, t.wl, nin, t.nout_pad, nin, 128);
    if (!rc) rc = make_map(t.map_wh64, t.wh, nin, t.nout_pad, nin, 64);
    if (!rc) rc = make_map(t.map_wl64, t.wl, nin, t.nout_pad, nin, 64);
    if (rc) return rc;
    t.ready = 1;
    return 0;
}

void tc_bank_free(TcBank& t) {
    if (t.wh) cudaFree(t.wh);
    if (t.wl) cudaFree(t.wl);
    if (t.colcorr) cudaFree(t.colcorr);
    if (t.colcorr_kb) cudaFree(t.colcorr_kb);
    if (t.wt) cudaFree(t.wt);
    t.wt = nullptr;
    t.map_w16_ok = 0;
    t.wh = t.wl = nullptr;
    t.colcorr = t.colcorr_kb = nullptr;
    t.ready = 0;
    t.prebuilt = 0;
}

int tc_rows_alloc(TcRows& r, int rows_cap, int kmax, uint32_t* err) {
    tc_rows_free(r);
    r.rows_cap = (rows_cap + 127) / 128 * 128;
    r.kmax = kmax;
    r.err = err;
    cudaError_t e;
    size_t n = (size_t)r.rows_cap * kmax;
    if ((e = cudaMalloc(&r.xh, n)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&r.xl, n)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&r.sat, n * sizeof(int16_t))) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&r.rowcorr, sizeof(int64_t) * r.rows_cap)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&r.nsat, sizeof(int32_t) * r.rows_cap)) != cudaSuccess) return (int)e;
    cudaMemset(r.xh, 0, n);
    cudaMemset(r.xl, 0, n);
    cudaMemset(r.nsat, 0, sizeof(int32_t) * r.rows_cap);
    r.nmaps = 0;
    return (int)cudaGetLastError();
}

void tc_rows_free(TcRows& r) {
    void* ps[] = {r.xh, r.xl, r.sat, r.rowcorr, r.nsat};
    for (void* p : ps)
        if (p) cudaFree(p);
    r.xh = r.xl = nullptr;
    r.sat = nullptr;
    r.rowcorr = nullptr;
    r.nsat = nullptr;
    r.nmaps = 0;
}

// k_bank_wide takes this bank for `rows` rows (<= 64): the K split over wz CTAs of a cluster when one CTA cannot hold
// all K blocks, 64-column tiles, and every CTA on the GPU at once
bool wide_fits(const TcBank& t, int rows, int* wz_out) {
    const int kb = t.nin / 128;
    int wz = 1;
    while (wz <= MAX_SPLIT && (kb % wz || kb / wz > WIDE_MAX_KB)) wz++;
    if (wz_out) *wz_out = wz;
    const int wrh = (rows + WIDE_ROWS - 1) / WIDE_ROWS;
    const WideCaps& c = wide_caps();
    return t.ready && c.ready && rows >= 1 && rows <= BN && wz <= 4 && WIDE_ROWS % wz == 0 && t.nout % 64 == 0 &&
           (t.nout / 64) * wz * wrh <= c.ctas[wz];
}

// the K split of the in-kernel-quantising k_bank_wide for this bank: a function of the bank alone, never of the
// step's row count, because the per-(bank, row half) arrival counter assumes every launch at a site adds the same
// number of arrivals (the CTAs along x and K). A 768-input bank goes to a CTA pair when a 64-row launch of pairs
// still fits the device at once (qkv, proj); otherwise (fc) it stays unsplit.
static int wide_quant_split(const TcBank& t) {
    int wz = 1;
    wide_fits(t, BN, &wz);
    const int kb = t.nin / 128;
    const WideCaps& c = wide_caps();
    if (wz == 1 && tc_wide_kz == 2 && kb % 2 == 0 && (t.nout / 64) * 2 * (BN / WIDE_ROWS) <= c.ctas[2]) wz = 2;
    return wz;
}

// the qkv bank's epilogue does the q/k/v split (heads_row) for GPT-2's gauged qkv and Pythia's plain one
static bool heads_fit(const TcHeads& h, int epi) {
    return h.pythia ? (epi == EPI_PLAIN_OUT && h.COS && h.SIN) : epi == EPI_GAUGED;
}

// k_bank_gemv takes this quantised decode bank at `rows` rows: whole 768-input ranges (a cluster of at most 4 along K),
// 16-byte weight rows (nout % 8 == 0), and a gauged bank's row in one CTA
static bool gemv_fits(const TcBank& t, int epi, int rows) {
    const int nz = t.nin / GEMV_KR;
    const bool gauged = epi == EPI_GAUGED || epi == EPI_GAUGED_EDGE;
    return tc_gemv && t.w16 && rows >= 1 && rows <= GEMV_MAX_ROWS && t.nin % GEMV_KR == 0 && (nz == 1 || nz == 2 || nz == 4) &&
           t.nout % 8 == 0 && !(gauged && nz != 1) && wide_caps().ctas[nz] >= nz;
}

int tc_bank(const TcBank& t, TcRows& r, int epi, int rows, const int32_t* ex, const int64_t* LS, const int32_t* e,
            const int64_t* b, int64_t* out, int ldo, const int32_t* out_map, const int32_t* EXP2, const int32_t* PHI,
            cudaStream_t st, bool pdl, const TcHeads* heads, bool* heads_done, uint64_t* trace, const TcQuant* quant,
            uint64_t* or_out, const TcRace* race, uint64_t* stamp) {
    if (heads_done) *heads_done = false;
    if (!t.ready || rows < 1 || rows > r.rows_cap || t.nin > r.kmax) return (int)cudaErrorInvalidValue;
    // the row planes' tensor maps for K = nin (box: 128 bytes x 64 rows), made once
    int mi = -1;
    for (int i = 0; i < r.nmaps; i++)
        if (r.maps[i].k == t.nin) mi = i;
    if (mi < 0) {
        if (r.nmaps == 4) return (int)cudaErrorInvalidValue;
        mi = r.nmaps;
        int rc = make_map(r.maps[mi].h, r.xh, t.nin, r.rows_cap, r.kmax, BN);
        if (!rc) rc = make_map(r.maps[mi].l, r.xl, t.nin, r.rows_cap, r.kmax, BN);
        if (!rc) rc = make_map(r.maps[mi].h32, r.xh, t.nin, r.rows_cap, r.kmax, WIDE_ROWS);
        if (!rc) rc = make_map(r.maps[mi].l32, r.xl, t.nin, r.rows_cap, r.kmax, WIDE_ROWS);
        if (rc) return rc;
        r.maps[mi].k = t.nin;
        r.maps[mi].bn = BN;
        r.nmaps++;
    }
    const int mtiles = t.nout_pad / 128, ntiles = (rows + BN - 1) / BN, kb = t.nin / 128;
    TcArgs a{};
    a.nin = t.nin;
    a.nout = t.nout;
    a.rows = rows;
    a.mtiles = mtiles;
    a.ntiles = ntiles;
    a.colcorr = t.colcorr;
    a.rowcorr = r.rowcorr;
    a.nsat = r.nsat;
    a.sat = r.sat;
    a.sat_ld = r.kmax;
    a.w16 = t.w16;
    a.err = r.err;
    a.epi = EpiArgs{ex, LS, e, b, out, ldo, out_map, EXP2, PHI};
    a.or_out = or_out;
    a.stamp = stamp;
    // split-K over a cluster when there is one row tile and too few output tiles to fill the GPU
    int ksplit = 1;
    if (ntiles == 1 && mtiles < 148)
        for (int d = MAX_SPLIT; d >= 2; d--)
            if (kb % d == 0 && kb / d <= MAX_KPS && mtiles * d <= 160) { ksplit = d; break; }
    if (race && !out && !race->v) return (int)cudaErrorInvalidValue;
    cudaError_t err;
    int wz = 1;
    const bool wide_ok = wide_fits(t, rows, &wz);
    const int wrh = (rows + WIDE_ROWS - 1) / WIDE_ROWS;
    if (quant) {                      // the rows quantised in the kernel: only k_bank_wide does that
        if (!wide_ok || out_map || race ||
            ((uintptr_t)quant->X & 15) || (quant->ldx & 1))
            return (int)cudaErrorInvalidValue;
        a.q = *quant;
        if (gemv_fits(t, epi, rows)) {            // batch-1 decode: the CUDA-core GEMV, no hand-off between CTAs
            if (heads && heads_fit(*heads, epi)) {
                a.heads = 1;
                a.hd = *heads;
                if (heads_done) *heads_done = true;
            }
            const int nz = t.nin / GEMV_KR;
            dim3 grid((t.nout + 63) / 64, nz, 1);
            if (rows == 1) {
                B2_EPI_SWITCH(epi, err = launch_args(k_bank_gemv<E, 1>, grid, dim3(GEMV_THREADS), nz, st, pdl, a); break)
            } else {
                B2_EPI_SWITCH(epi, err = launch_args(k_bank_gemv<E, 2>, grid, dim3(GEMV_THREADS), nz, st, pdl, a); break)
            }
            return (int)err;
        }
        a.q.xh = r.xh;
        a.q.xl = r.xl;
        a.q.sat = r.sat;
        a.q.kmax = r.kmax;
        const int qz = quant->unsplit ? 1 : wide_quant_split(t);
        if (qz > 2 && (heads || epi != EPI_PLAIN_ADD)) return (int)cudaErrorInvalidValue;
        if ((t.nout / 64) * qz * wrh > wide_caps().ctas[qz]) return (int)cudaErrorInvalidValue;
        wz = qz;
        a.ksplit = wz;
        a.kps = kb / wz;
        a.trace = trace;
        if (heads && heads_fit(*heads, epi)) {
            a.heads = 1;
            a.hd = *heads;
            if (heads_done) *heads_done = true;
        }
        dim3 grid(t.nout / 64, wz, wrh);
        const size_t sm = wide_smem_bytes(a.kps);
        B2_EPI_SWITCH(epi, err = launch_k(k_bank_wide<E, true>, grid, dim3(WIDE_THREADS), sm, wz, st, pdl, t,
                                          r.maps[mi].h32, r.maps[mi].l32, a, true);
                      break)
    } else if (tc_wide && wide_ok && wz == 1 && !race) {   // the race runs in k_bank_tiles' epilogue only
        // one CTA per 64 output columns over the whole K range (no split, no cluster)
        a.ksplit = 1;
        a.kps = kb;
        a.trace = trace;
        if (heads && epi == EPI_GAUGED && !heads->pythia && !out_map) {
            a.heads = 1;
            a.hd = *heads;
            if (heads_done) *heads_done = true;
        }
        dim3 grid(t.nout / 64, 1, wrh);
        B2_EPI_SWITCH(epi, err = launch_k(k_bank_wide<E, false>, grid, dim3(WIDE_THREADS), wide_smem_bytes(kb), 1, st, pdl, t,
                                          r.maps[mi].h32, r.maps[mi].l32, a, true);
                      break)
    } else if (ksplit > 1 && !race) {
        a.ksplit = ksplit;
        a.kps = kb / ksplit;
        a.trace = trace;
        if (heads && epi == EPI_GAUGED && !heads->pythia && !out_map) {
            a.heads = 1;
            a.hd = *heads;
            if (heads_done) *heads_done = true;
        }
        a.stages = a.kps;
        size_t smem = (size_t)(a.kps > 2 ? a.kps : 2) * STAGE + 1024;   // >= the 64 KB partial tile
        dim3 grid(mtiles, ksplit, 1);
        B2_EPI_SWITCH(epi, err = launch_k(k_bank_split<E>, grid, dim3(256), smem, ksplit, st, pdl, t, r.maps[mi].h,
                                          r.maps[mi].l, a);
                      break)
    } else {
        a.ksplit = 1;
        a.kps = kb;
        a.stages = MAX_STAGES;
        a.trace = trace;
        if (race) {
            if ((epi != EPI_GAUGED && epi != EPI_PLAIN_OUT) || race->ld < mtiles * 4) return (int)cudaErrorInvalidValue;
            a.race = *race;
        }
        size_t smem = (size_t)MAX_STAGES * STAGE + 1024;
        int total = mtiles * ntiles;
        dim3 grid(total < 148 ? total : 148);
        B2_EPI_SWITCH(epi, err = launch_k(k_bank_tiles<E>, grid, dim3(TILE_THREADS), smem, 1, st, pdl, t, r.maps[mi].h,
                                          r.maps[mi].l, a);
                      break)
    }
    return (int)err;
}

int tc_head_gemv(const TcBank& t, int epi, const int64_t* X, int ldx, int rows, const int32_t* e, const int64_t* b,
                 const int32_t* EXP2, const int32_t* LOG2, int64_t log768, int64_t eps40, const TcRace& race,
                 int64_t* out, int ldo, uint32_t* err, int grid, cudaStream_t st, bool pdl, uint64_t* stamp) {
    if (!t.map_w16_ok || t.nin != GEMV_KR || rows < 1 || rows > GEMV_MAX_ROWS || (epi != EPI_GAUGED && epi != EPI_PLAIN_OUT) ||
        !race.v || race.ld < 2 * ((t.nout + 63) / 64) || grid < 1)
        return (int)cudaErrorInvalidValue;
    TcArgs a{};
    a.nin = t.nin;
    a.nout = t.nout;
    a.rows = rows;
    a.err = err;
    a.q.X = X;
    a.q.ldx = ldx;
    a.q.LOG2 = LOG2;
    a.q.log768 = log768;
    a.q.eps40 = eps40;
    a.epi = EpiArgs{nullptr, nullptr, e, b, out, ldo, nullptr, EXP2, nullptr};
    a.stamp = stamp;
    const int ntiles = (t.nout + 63) / 64;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid < ntiles ? grid : ntiles);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = HG_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    const CUtensorMap& m = *reinterpret_cast<const CUtensorMap*>(t.map_w16.bytes);
    cudaError_t r;
    if (epi == EPI_GAUGED)
        r = rows == 1 ? cudaLaunchKernelEx(&cfg, k_head_gemv<EPI_GAUGED, 1>, m, a, race)
                      : cudaLaunchKernelEx(&cfg, k_head_gemv<EPI_GAUGED, 2>, m, a, race);
    else
        r = rows == 1 ? cudaLaunchKernelEx(&cfg, k_head_gemv<EPI_PLAIN_OUT, 1>, m, a, race)
                      : cudaLaunchKernelEx(&cfg, k_head_gemv<EPI_PLAIN_OUT, 2>, m, a, race);
    return (int)r;
}

int tc_entry_qkv(const TcBank& t, const int64_t* Tw, const int64_t* Tp, const int32_t* row_tok, const int64_t* wte,
                 const int64_t* wpe, int vocab, int nctx, int rows, const int32_t* e, const int64_t* b, const int32_t* EXP2,
                 const TcQuant& q, const TcHeads& hd, uint32_t* err, cudaStream_t st, bool pdl, uint64_t* stamp) {
    if (rows < 1 || hd.pythia || t.nout % 64) return (int)cudaErrorInvalidValue;
    TcArgs a{};
    a.nin = t.nin;
    a.nout = t.nout;
    a.rows = rows;
    a.err = err;
    a.q = q;
    a.epi = EpiArgs{nullptr, nullptr, e, b, nullptr, 0, nullptr, EXP2, nullptr};
    a.heads = 1;
    a.hd = hd;
    a.stamp = stamp;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(512);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, k_entry_qkv, a, Tw, Tp, row_tok, wte, wpe, vocab, nctx);
}

int tc_absmax(const int64_t* x, size_t n, unsigned long long* out, cudaStream_t st) {
    k_absmax<<<296, 256, 0, st>>>(x, n, out);
    return (int)cudaGetLastError();
}

}  // namespace b2
