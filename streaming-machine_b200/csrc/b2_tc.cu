// b2_tc.cu -- the bank product on tcgen05 tensor cores (kind::i8), exact (see b2_tc.cuh for the identity).
//
// One CTA = 128 output columns (the MMA's M, TMEM lanes) x BN rows (the MMA's N, TMEM columns) x a K range.
// Warp 0 lane 0 streams the four planes of each 128-byte K block into shared memory with TMA (SWIZZLE_128B,
// K-major), warp 1 lane 0 issues 16 MMAs per K block (4 K steps x {wh.xh, wh.xl, wl.xh, wl.xl}) into three int32
// accumulators in TMEM, and all four warps read them back (tcgen05.ld) for the epilogue. When the K range is split
// over CTAs (few tiles, as in a 64-stream decode step), partial piles meet in an int64 buffer by atomic adds (exact
// in any order) and the last CTA to arrive for a tile finishes it. Every wait is bounded; on a timeout the CTA
// sets DERR_TIMEOUT, skips its stores, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "b2_epi.cuh"
#include "b2_tc.cuh"

namespace b2 {

namespace {

// ---- PTX wrappers ---------------------------------------------------------------------------------------------------
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
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
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
B2_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            saddr(dst)),
        "l"((uint64_t)map), "r"(saddr(bar)), "r"(c0), "r"(c1)
        : "memory");
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
B2_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int BN>
struct Cfg {
    static constexpr int A = 128 * 128;              // one weight plane of a K block
    static constexpr int B = BN * 128;               // one row plane of a K block
    static constexpr int STAGE = 2 * A + 2 * B;
    static constexpr uint32_t TMEM_COLS = 3 * BN <= 256 ? 256 : 512;
    // kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, N = BN, M = 128
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};
constexpr int MAX_STAGES = 4;

struct TcArgs {
    int nin, nout, rows;
    int kps;          // K blocks (of 128) per CTA
    int ksplit;       // CTAs along K per tile
    int stages;
    const int64_t* colcorr;
    const int64_t* rowcorr;
    const int32_t* nsat;
    const int16_t* sat;
    int sat_ld;
    const int16_t* w16;
    int64_t* pile;
    uint32_t* counters;
    uint32_t* err;
    EpiArgs epi;
};

template <int EPI, int BN>
__global__ void __launch_bounds__(128, 1)
    k_bank_tc(const __grid_constant__ CUtensorMap mwh, const __grid_constant__ CUtensorMap mwl,
              const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl, const TcArgs a) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full_bar[MAX_STAGES], empty_bar[MAX_STAGES], acc_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort, s_last;
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, ks = blockIdx.y, nt = blockIdx.z;
    const int S = a.stages;
    // after any timeout in this or an earlier launch, do nothing (the call is already reported as failed)
    if (*(volatile uint32_t*)a.err & DERR_TIMEOUT) return;

    if (tid == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        mbar_init(&acc_bar, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer ----
        for (int kb = 0; kb < a.kps; kb++) {
            int s = kb % S;
            if (kb >= S && !mbar_wait(&empty_bar[s], ((kb / S) - 1) & 1, a.err)) { s_abort = 1; break; }
            uint8_t* st = smem + s * C::STAGE;
            int kx = (ks * a.kps + kb) * 128;
            mbar_expect_tx(&full_bar[s], C::STAGE);
            tma_load_2d(st, &mwh, &full_bar[s], kx, mt * 128);
            tma_load_2d(st + C::A, &mwl, &full_bar[s], kx, mt * 128);
            tma_load_2d(st + 2 * C::A, &mxh, &full_bar[s], kx, nt * BN);
            tma_load_2d(st + 2 * C::A + C::B, &mxl, &full_bar[s], kx, nt * BN);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        for (int kb = 0; kb < a.kps; kb++) {
            int s = kb % S;
            if (!mbar_wait(&full_bar[s], (kb / S) & 1, a.err)) { s_abort = 1; break; }
            tc_fence_after();
            uint32_t base = saddr(smem + s * C::STAGE);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                uint64_t ah = sdesc(base + kk * 32), al = sdesc(base + C::A + kk * 32);
                uint64_t bh = sdesc(base + 2 * C::A + kk * 32), bl = sdesc(base + 2 * C::A + C::B + kk * 32);
                uint32_t acc = (kb | kk) != 0;
                mma_i8(tmem + 0 * BN, ah, bh, C::IDESC, acc);   // A1 += wh . xh
                mma_i8(tmem + 1 * BN, ah, bl, C::IDESC, acc);   // A2 += wh . xl
                mma_i8(tmem + 1 * BN, al, bh, C::IDESC, 1);     // A2 += wl . xh
                mma_i8(tmem + 2 * BN, al, bl, C::IDESC, acc);   // A3 += wl . xl
            }
            mma_commit(&empty_bar[s]);
        }
        mma_commit(&acc_bar);
    }
    __syncwarp();

    // ---- epilogue: thread = output column m of the tile; TMEM columns = rows ----
    bool ok = mbar_wait(&acc_bar, 0, a.err);
    tc_fence_after();
    __syncthreads();
    if (!ok || s_abort) goto teardown;
    {
        const int m = warp * 32 + lane;
        const int j = mt * 128 + m;
        const bool jv = j < a.nout;
        const int64_t colc = (ks == 0 && jv) ? a.colcorr[j] : 0;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int n0 = 0; n0 < BN; n0 += 16) {
            uint32_t r1[16], r2[16], r3[16];
            tmem_ld16(trow + 0 * BN + n0, r1);
            tmem_ld16(trow + 1 * BN + n0, r2);
            tmem_ld16(trow + 2 * BN + n0, r3);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 16; q++) {
                const int n = nt * BN + n0 + q;
                if (n >= a.rows || !jv) continue;
                int64_t pile = (int64_t)(int32_t)r1[q] * 65536 + (int64_t)(int32_t)r2[q] * 256 + (int64_t)(int32_t)r3[q];
                if (ks == 0) {
                    pile += colc + a.rowcorr[n];
                    const int ns = a.nsat[n];
                    for (int u = 0; u < ns; u++)
                        pile += 256 * (int64_t)a.w16[(size_t)a.sat[(size_t)n * a.sat_ld + u] * a.nout + j];
                }
                if (a.ksplit == 1)
                    epi_store<EPI>(a.epi, n, j, pile);
                else
                    atomicAdd((unsigned long long*)&a.pile[(size_t)n * PILE_COLS + j], (unsigned long long)pile);
            }
        }
        if (a.ksplit > 1) {
            __threadfence();
            __syncthreads();
            const int tile = nt * gridDim.x + mt;
            if (tid == 0) s_last = atomicAdd(&a.counters[tile], 1u) == (uint32_t)(a.ksplit - 1);
            __syncthreads();
            if (s_last) {
                __threadfence();
                if (jv) {
                    for (int q = 0; q < BN; q++) {
                        const int n = nt * BN + q;
                        if (n >= a.rows) break;
                        int64_t* p = &a.pile[(size_t)n * PILE_COLS + j];
                        int64_t v = (int64_t)__ldcg((const long long*)p);
                        *p = 0;
                        epi_store<EPI>(a.epi, n, j, v);
                    }
                }
                if (tid == 0) a.counters[tile] = 0;
            }
        }
    }
teardown:
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
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

template <int EPI, int BN>
cudaError_t launch(dim3 grid, size_t smem, cudaStream_t st, const TcBank& t, const TcMap& xh, const TcMap& xl, const TcArgs& a) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k_bank_tc<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    k_bank_tc<EPI, BN><<<grid, 128, smem, st>>>(*reinterpret_cast<const CUtensorMap*>(t.map_wh.bytes),
                                                 *reinterpret_cast<const CUtensorMap*>(t.map_wl.bytes),
                                                 *reinterpret_cast<const CUtensorMap*>(xh.bytes),
                                                 *reinterpret_cast<const CUtensorMap*>(xl.bytes), a);
    return cudaGetLastError();
}

template <int BN>
cudaError_t launch_epi(int epi, dim3 grid, size_t smem, cudaStream_t st, const TcBank& t, const TcMap& xh, const TcMap& xl,
                       const TcArgs& a) {
    switch (epi) {
        case EPI_GAUGED: return launch<EPI_GAUGED, BN>(grid, smem, st, t, xh, xl, a);
        case EPI_GAUGED_EDGE: return launch<EPI_GAUGED_EDGE, BN>(grid, smem, st, t, xh, xl, a);
        case EPI_PLAIN_ADD: return launch<EPI_PLAIN_ADD, BN>(grid, smem, st, t, xh, xl, a);
        default: return launch<EPI_PLAIN_OUT, BN>(grid, smem, st, t, xh, xl, a);
    }
}

}  // namespace

int tc_min_rows_default() { return 1; }

int tc_bank_build(TcBank& t, const int16_t* w, int nin, int nout) {
    tc_bank_free(t);
    if (nin % 128) return (int)cudaErrorInvalidValue;
    t.nin = nin;
    t.nout = nout;
    t.nout_pad = (nout + 127) / 128 * 128;
    t.w16 = w;
    cudaError_t e;
    if ((e = cudaMalloc(&t.wh, (size_t)t.nout_pad * nin)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&t.wl, (size_t)t.nout_pad * nin)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&t.colcorr, sizeof(int64_t) * t.nout_pad)) != cudaSuccess) return (int)e;
    k_weight_planes<<<dim3(t.nout_pad / 32, (nin + 31) / 32), dim3(32, 8)>>>(w, nin, nout, t.wh, t.wl);
    k_colcorr<<<(t.nout_pad + 255) / 256, 256>>>(w, nin, nout, t.nout_pad, t.colcorr);
    if ((e = cudaGetLastError()) != cudaSuccess) return (int)e;
    int rc = make_map(t.map_wh, t.wh, nin, t.nout_pad, nin, 128);
    if (!rc) rc = make_map(t.map_wl, t.wl, nin, t.nout_pad, nin, 128);
    if (rc) return rc;
    t.ready = 1;
    return 0;
}

void tc_bank_free(TcBank& t) {
    if (t.wh) cudaFree(t.wh);
    if (t.wl) cudaFree(t.wl);
    if (t.colcorr) cudaFree(t.colcorr);
    t.wh = t.wl = nullptr;
    t.colcorr = nullptr;
    t.ready = 0;
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
    if ((e = cudaMalloc(&r.pile, sizeof(int64_t) * PILE_ROWS * PILE_COLS)) != cudaSuccess) return (int)e;
    if ((e = cudaMalloc(&r.counters, sizeof(uint32_t) * MAX_COUNTERS)) != cudaSuccess) return (int)e;
    cudaMemset(r.xh, 0, n);
    cudaMemset(r.xl, 0, n);
    cudaMemset(r.pile, 0, sizeof(int64_t) * PILE_ROWS * PILE_COLS);
    cudaMemset(r.counters, 0, sizeof(uint32_t) * MAX_COUNTERS);
    cudaMemset(r.nsat, 0, sizeof(int32_t) * r.rows_cap);
    r.nmaps = 0;
    return (int)cudaGetLastError();
}

void tc_rows_free(TcRows& r) {
    void* ps[] = {r.xh, r.xl, r.sat, r.rowcorr, r.nsat, r.pile, r.counters};
    for (void* p : ps)
        if (p) cudaFree(p);
    r.xh = r.xl = nullptr;
    r.sat = nullptr;
    r.rowcorr = r.pile = nullptr;
    r.nsat = nullptr;
    r.counters = nullptr;
    r.nmaps = 0;
}

int tc_bank(const TcBank& t, TcRows& r, int epi, int rows, const int32_t* ex, const int64_t* LS, const int32_t* e,
            const int64_t* b, int64_t* out, int ldo, const int32_t* out_map, const int32_t* EXP2, const int32_t* PHI,
            cudaStream_t st) {
    if (!t.ready || rows < 1 || rows > r.rows_cap || t.nin > r.kmax) return (int)cudaErrorInvalidValue;
    const int BN = rows <= 64 ? 64 : 128;
    // the row planes' tensor maps for (K = nin, box height BN), made once
    int mi = -1;
    for (int i = 0; i < r.nmaps; i++)
        if (r.maps[i].k == t.nin && r.maps[i].bn == BN) mi = i;
    if (mi < 0) {
        if (r.nmaps == 4) return (int)cudaErrorInvalidValue;
        mi = r.nmaps;
        int rc = make_map(r.maps[mi].h, r.xh, t.nin, r.rows_cap, r.kmax, BN);
        if (!rc) rc = make_map(r.maps[mi].l, r.xl, t.nin, r.rows_cap, r.kmax, BN);
        if (rc) return rc;
        r.maps[mi].k = t.nin;
        r.maps[mi].bn = BN;
        r.nmaps++;
    }
    const int mtiles = t.nout_pad / 128, ntiles = (rows + BN - 1) / BN, kb = t.nin / 128;
    int ksplit = 1;
    if (rows <= PILE_ROWS && t.nout <= PILE_COLS && mtiles * ntiles < 148 && mtiles * ntiles <= MAX_COUNTERS) {
        int want = (2 * 148 + mtiles * ntiles - 1) / (mtiles * ntiles);
        for (int d = 1; d <= kb; d++)
            if (kb % d == 0 && d <= want) ksplit = d;
    }
    TcArgs a{};
    a.nin = t.nin;
    a.nout = t.nout;
    a.rows = rows;
    a.ksplit = ksplit;
    a.kps = kb / ksplit;
    a.stages = a.kps < (BN == 64 ? 4 : 3) ? a.kps : (BN == 64 ? 4 : 3);
    a.colcorr = t.colcorr;
    a.rowcorr = r.rowcorr;
    a.nsat = r.nsat;
    a.sat = r.sat;
    a.sat_ld = r.kmax;
    a.w16 = t.w16;
    a.pile = r.pile;
    a.counters = r.counters;
    a.err = r.err;
    a.epi = EpiArgs{ex, LS, e, b, out, ldo, out_map, EXP2, PHI};
    dim3 grid(mtiles, ksplit, ntiles);
    cudaError_t err;
    if (BN == 64)
        err = launch_epi<64>(epi, grid, (size_t)a.stages * Cfg<64>::STAGE + 1024, st, t, r.maps[mi].h, r.maps[mi].l, a);
    else
        err = launch_epi<128>(epi, grid, (size_t)a.stages * Cfg<128>::STAGE + 1024, st, t, r.maps[mi].h, r.maps[mi].l, a);
    return (int)err;
}

}  // namespace b2
