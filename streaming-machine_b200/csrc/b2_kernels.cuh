// b2_kernels.cuh -- the machine's kernels other than the tensor-core bank product: embedding, to16 + gauge,
// head split into q16/k16/v with the key/value store append, the arrival (attention), the race, the row bookkeeping,
// and the CUDA-core bank product used for small row counts and as the on-device cross-check of the tensor path.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "b2_arith.cuh"
#include "b2_epi.cuh"
#include "b2_float.cuh"
#include "b2_ptx.cuh"

namespace b2 {


// ---------------------------------------------------------------------------------------------------------------------
// embedding: R = wte[tok] + wpe[pos] (base2.py:103; the Metal engine's nextin, base2_stream.swift:143-146)
// ---------------------------------------------------------------------------------------------------------------------
__global__ void k_embed(const int32_t* __restrict__ row_tok, const int32_t* __restrict__ row_pos, int rows,
                        const int64_t* __restrict__ wte, const int64_t* __restrict__ wpe, int d, int V, int nctx,
                        int64_t* __restrict__ R, uint32_t* err) {
    griddep_wait();
    griddep_launch();
    int r = blockIdx.x;
    if (r >= rows) return;
    int tok = row_tok[r], pos = row_pos[r];
    if (tok < 0 || tok >= V) { if (threadIdx.x == 0) set_err(err, DERR_TOKEN); tok = 0; }
    if (pos < 0 || pos >= nctx) { if (threadIdx.x == 0) set_err(err, DERR_POS); pos = 0; }
    const int64_t* a = wte + (size_t)tok * d;
    const int64_t* b = wpe ? wpe + (size_t)pos * d : nullptr;   // Pythia has no position table (rotary instead)
    for (int i = threadIdx.x; i < d; i += blockDim.x) R[(size_t)r * d + i] = b ? wadd(__ldg(a + i), __ldg(b + i)) : __ldg(a + i);
}

// ---------------------------------------------------------------------------------------------------------------------
// to16 (base2.py:24-27) + the gauge (base2.py:55-60): one CTA per row. x16 fits int32 (|x16| <= 32768).
// src_rows (optional) gathers rows (the head reads only the rows it scores).
// ---------------------------------------------------------------------------------------------------------------------
// Planes (optional, the tensor-core path): each x16 split into signed bytes xh = min(x >> 8, 127),
// xl = (x & 255) - 128; the +32768 entries listed in sat/nsat; rowcorr = 128 * sum of the represented values.
struct PlaneOut {
    int8_t* xh;
    int8_t* xl;
    int ld;             // row stride of xh/xl/sat
    int64_t* rowcorr;
    int32_t* nsat;
    int16_t* sat;
    uint64_t* stamp = nullptr;   // b2_profile mode 2
};

template <int NT>
__global__ void __launch_bounds__(NT) k_quant(const int64_t* __restrict__ X, int n, const int32_t* __restrict__ src_rows,
                                              int rows, int32_t* __restrict__ x16, int32_t* __restrict__ ex,
                                              int64_t* __restrict__ LS, int gauge, const int32_t* __restrict__ LOG2,
                                              int64_t log768, int64_t eps40, PlaneOut pl) {
    griddep_wait();
    stamp_begin(pl.stamp);
    griddep_launch();
    __shared__ uint64_t s_or[NT / 32];
    __shared__ int64_t s_1[NT / 32], s_2[NT / 32];
    __shared__ int s_nsat;
    int r = blockIdx.x;
    if (r >= rows) return;
    int sr = src_rows ? src_rows[r] : r;
    const int64_t* x = X + (size_t)sr * n;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint64_t o = 0;
    for (int i = threadIdx.x; i < n; i += NT) o |= mag(x[i]);
    o = warp_or64(o);
    if (lane == 0) s_or[wid] = o;
    __syncthreads();
    uint64_t all = 0;
#pragma unroll
    for (int k = 0; k < NT / 32; k++) all |= s_or[k];
    int sh = to16_shift(all);
    if (threadIdx.x == 0) s_nsat = 0;
    __syncthreads();
    int64_t q1 = 0, q2 = 0;
    for (int i = threadIdx.x; i < n; i += NT) {
        int64_t v = rshift(x[i], sh);
        if (x16) x16[(size_t)r * n + i] = (int32_t)v;
        q1 += v;
        q2 += v * v;
        if (pl.xh) {
            bool sat = v == 32768;
            pl.xh[(size_t)r * pl.ld + i] = (int8_t)(sat ? 127 : (v >> 8));
            pl.xl[(size_t)r * pl.ld + i] = (int8_t)((v & 255) - 128);
            if (sat) pl.sat[(size_t)r * pl.ld + atomicAdd(&s_nsat, 1)] = (int16_t)i;
        }
    }
    if (!gauge && !pl.xh) {
        if (threadIdx.x == 0) ex[r] = -16 + sh;
        return;
    }
    q1 = warp_sum64(q1);
    q2 = warp_sum64(q2);
    if (lane == 0) { s_1[wid] = q1; s_2[wid] = q2; }
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t S1 = 0, S2 = 0;
        for (int k = 0; k < NT / 32; k++) { S1 = wadd(S1, s_1[k]); S2 = wadd(S2, s_2[k]); }
        ex[r] = -16 + sh;
        if (gauge) LS[r] = gauge_LS(S1, S2, -16 + sh, LOG2, log768, eps40);
        if (pl.xh) {
            pl.nsat[r] = s_nsat;
            pl.rowcorr[r] = 128 * (S1 - 256 * (int64_t)s_nsat);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// Pythia's gauge (pythia_base2.py:100-110), the layer norm kept whole: to16 of the row, S1, S2,
// V = d*S2 - S1^2 + (EPS40 >> (40 + 2 ex)), LS = log2fix(V) >> 1, and for each lane
// out = power(c * g, (ge + 16) * 65536 - LS) + b with c = d * x16 - S1 (power exactly, as the reference's big ints).
// One CTA per row; src_rows (optional) gathers rows. Output int64 [rows][d] (the plain bank after it to16s it).
// ---------------------------------------------------------------------------------------------------------------------
// a second norm of the same rows in the same launch (blockIdx.y = 1): Pythia's two norms of a layer both read R
// before either branch adds into it (pythia_base2.py:163-167)
struct GaugeTwo {
    const int64_t* g = nullptr;
    int64_t ge = 0;
    const int64_t* b = nullptr;
    int64_t* out = nullptr;
    uint64_t* or_out = nullptr;
};
template <int NT>
__global__ void __launch_bounds__(NT) k_gauge_ln(const int64_t* __restrict__ R, int d, const int32_t* __restrict__ src_rows,
                                                 int rows, const int64_t* __restrict__ g, int64_t ge,
                                                 const int64_t* __restrict__ b, int64_t* __restrict__ out,
                                                 const int32_t* __restrict__ LOG2, const int32_t* __restrict__ EXP2,
                                                 int64_t eps40, uint32_t* err, uint64_t* stamp, uint64_t* or_out,
                                                 GaugeTwo two) {
    griddep_wait();
    stamp_begin(stamp);
    griddep_launch();
    if (blockIdx.y == 1) { g = two.g; ge = two.ge; b = two.b; out = two.out; or_out = two.or_out; }
    __shared__ uint64_t s_or[NT / 32];
    __shared__ int64_t s_1[NT / 32], s_2[NT / 32];
    __shared__ int64_t s_F, s_S1;
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int sr = src_rows ? src_rows[r] : r;
    const int64_t* x = R + (size_t)sr * d;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint64_t o = 0;
    for (int i = threadIdx.x; i < d; i += NT) o |= mag(x[i]);
    o = warp_or64(o);
    if (lane == 0) s_or[wid] = o;
    __syncthreads();
    uint64_t all = 0;
#pragma unroll
    for (int k = 0; k < NT / 32; k++) all |= s_or[k];
    const int sh = to16_shift(all);
    int64_t q1 = 0, q2 = 0;
    for (int i = threadIdx.x; i < d; i += NT) {
        const int64_t v = rshift(x[i], sh);
        q1 += v;
        q2 += v * v;
    }
    q1 = warp_sum64(q1);
    q2 = warp_sum64(q2);
    if (lane == 0) { s_1[wid] = q1; s_2[wid] = q2; }
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t S1 = 0, S2 = 0;
        for (int k = 0; k < NT / 32; k++) { S1 = wadd(S1, s_1[k]); S2 = wadd(S2, s_2[k]); }
        const int64_t ex = -16 + sh;
        const int64_t V = wadd(wsub(wmul(d, S2), wmul(S1, S1)), np_rsh(eps40, 40 + 2 * ex));
        const int64_t LS = log2fix(V, LOG2) >> 1;
        s_F = wsub(wmul(wadd(ge, 16), 65536), LS);
        s_S1 = S1;
    }
    __syncthreads();
    const int64_t F = s_F, S1 = s_S1;
    bool bad = false;
    uint64_t oo = 0;
    for (int i = threadIdx.x; i < d; i += NT) {
        const int64_t c = wsub(wmul(d, rshift(x[i], sh)), S1);
        const int64_t v = wadd(power_exact(wmul(c, g[i]), F, EXP2, &bad), b[i]);
        out[(size_t)r * d + i] = v;
        oo |= mag(v);
    }
    if (bad) set_err(err, DERR_RANGE);
    if (or_out) {                            // the next bank's to16 shift: the OR of the row's magnitudes
        oo = warp_or64(oo);
        __syncthreads();                     // s_or's earlier values were read above
        if (lane == 0) s_or[wid] = oo;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t w = 0;
#pragma unroll
            for (int k = 0; k < NT / 32; k++) w |= s_or[k];
            or_out[r] = w;
        }
    }
}

// Pythia's q/k/v split (pythia_base2.py:116-134): one warp per (row, part of 3H), parts ordered per head q, k, v.
// q and k: the first `rot` dims turned by the position (pairs (i, i + rot/2), cos/sin at 2^-30; inputs past 2^31
// are where the reference asserts), then to16 over the head; v to the value store as it is.
// turn=float (pythia_base2.py:118-120): cosf/sinf, float64 cos and sin of the angles made on the host, replace the
// integer turn: round(a c - b s), round(b c + a s). arrival=float: the turned q (qraw [rows][d]) and k (kv.kraw) at
// full width as well.
__global__ void k_heads_pythia(const int64_t* __restrict__ QKV, int rows, const int32_t* __restrict__ row_slot,
                               const int32_t* __restrict__ row_pos, int layer, KV kv, int rot,
                               const int32_t* __restrict__ COS, const int32_t* __restrict__ SIN, int32_t* __restrict__ q16,
                               int32_t* __restrict__ qexp, uint32_t* err, const double* __restrict__ cosf,
                               const double* __restrict__ sinf, int64_t* __restrict__ qraw, uint64_t* stamp) {
    griddep_wait();
    stamp_begin(stamp);
    griddep_launch();
    const int r = blockIdx.x, part = blockIdx.y, lane = threadIdx.x;
    const int H = kv.H, d = H * 64, h = part / 3, kind = part % 3;
    if (r >= rows) return;
    const int64_t* x = QKV + (size_t)r * 3 * d + (size_t)part * 64;
    int64_t v0 = x[lane], v1 = x[lane + 32];
    const int slot = row_slot[r], pos = row_pos[r];
    if (pos < 0 || pos >= kv.lim) { if (lane == 0) set_err(err, DERR_POS); return; }   // never index past the tables
    if (kind < 2) {
        const int half = rot >> 1;                                       // rot == 16: pairs (t, t + 8) in lanes 0..15
        const bool big = !cosf && lane < rot && mag(v0) >= (1ull << 31);
        if (__any_sync(0xffffffffu, big) && lane == 0) set_err(err, DERR_RANGE);
        const int64_t other = __shfl_xor_sync(0xffffffffu, v0, half);   // lane t < half holds a, lane t + half holds b
        if (cosf) {
            if (lane < rot) {
                const int t = lane < half ? lane : lane - half;
                const double c = cosf[(size_t)pos * half + t], s = sinf[(size_t)pos * half + t];
                const double me = i2d(v0), ot = i2d(other);
                v0 = lane < half ? rint64(__dsub_rn(__dmul_rn(me, c), __dmul_rn(ot, s)))      // a c - b s
                                 : rint64(__dadd_rn(__dmul_rn(me, c), __dmul_rn(ot, s)));     // b c + a s
            }
        } else if (lane < rot) {
            const int t = lane < half ? lane : lane - half;
            const int64_t c = COS[(size_t)pos * half + t], s = SIN[(size_t)pos * half + t];
            if (lane < half) v0 = rshift(wsub(wmul(v0, c), wmul(other, s)), 30);          // a*c - b*s
            else v0 = rshift(wadd(wmul(v0, c), wmul(other, s)), 30);                       // b*c + a*s
        }
        const int sh = to16_shift(warp_or64(mag(v0) | mag(v1)));
        const int64_t a0 = rshift(v0, sh), a1 = rshift(v1, sh);
        if (kind == 0 && qraw) { qraw[(size_t)r * d + h * 64 + lane] = v0; qraw[(size_t)r * d + h * 64 + lane + 32] = v1; }
        if (kind == 1 && kv.kraw) {
            const size_t idx = kv_index(slot, layer, h, pos, kv.L, H, kv.ctx);
            kv.kraw[idx * 64 + lane] = v0;
            kv.kraw[idx * 64 + lane + 32] = v1;
        }
        if (kind == 0) {
            q16[(size_t)r * d + h * 64 + lane] = (int32_t)a0;
            q16[(size_t)r * d + h * 64 + lane + 32] = (int32_t)a1;
            if (lane == 0) qexp[r * H + h] = -16 + sh;
        } else {
            const size_t idx = kv_index(slot, layer, h, pos, kv.L, H, kv.ctx);
            kv.k[idx * 64 + lane] = (int16_t)(uint16_t)(uint32_t)a0;
            kv.k[idx * 64 + lane + 32] = (int16_t)(uint16_t)(uint32_t)a1;
            const uint32_t m0 = __ballot_sync(0xffffffffu, a0 == 32768), m1 = __ballot_sync(0xffffffffu, a1 == 32768);
            if (lane == 0) {
                kv.kmask[idx] = (uint64_t)m0 | ((uint64_t)m1 << 32);
                kv.kexp[idx] = -16 + sh;
            }
        }
    } else {
        const size_t idx = kv_index(slot, layer, h, pos, kv.L, H, kv.ctx);
        const bool bad = v0 != (int64_t)(int32_t)v0 || v1 != (int64_t)(int32_t)v1;
        if (__any_sync(0xffffffffu, bad) && lane == 0) set_err(err, DERR_VOVF);
        kv.v[idx * 64 + lane] = (int32_t)v0;
        kv.v[idx * 64 + lane + 32] = (int32_t)v1;
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// bank epilogues (base2.py:62-76, 78-83)
// ---------------------------------------------------------------------------------------------------------------------
struct BankArgs {
    const int32_t* x16;     // [rows][nin]
    const int16_t* w;       // [nin][nout]
    int nin, nout, rows;
    EpiArgs epi;
    int flt = 0;                    // float stage switches of this bank's epilogue (FE_* bits), 0: integer
    const double* sig = nullptr;    // gauge=float: per row sqrt(var + 1e-5) of the stream at 2^-16
};

// the bank epilogue with float stages (base2.py:66-69 gauged bank, :110-113 head, :79-80 bend; pythia_base2.py:144-146
// bend): pile * 2^(we + ex) / sig at 2^-16 rounded, the bias after (layer banks) or before the rounding (head)
template <int EPI>
B2_DEV void epi_store_float(const BankArgs& a, int r, int j, int64_t pile) {
    const EpiArgs& e = a.epi;
    const int orow = e.out_map ? e.out_map[r] : r;
    int64_t* o = e.out + (size_t)orow * e.ldo + j;
    const int64_t es = wadd(wadd((int64_t)e.e[j], (int64_t)e.ex[r]), 16);
    int64_t v;
    if ((EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE) && (a.flt & (FE_GAUGE | FE_GAUGE_HEAD))) {
        const double val = __ddiv_rn(__dmul_rn(i2d(pile), scalbn(1.0, (int)(es - 16))), a.sig[r]);
        v = (a.flt & FE_GAUGE_HEAD) ? rint64(__dmul_rn(__dadd_rn(val, __ddiv_rn(i2d(e.b[j]), 65536.0)), 65536.0))
                                    : wadd(rint64(__dmul_rn(val, 65536.0)), e.b[j]);
    } else if (EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE) {
        v = wadd(power(pile, wsub(wmul(es, 65536), e.LS[r]), e.EXP2), e.b[j]);
    } else {
        v = wadd(rshift(pile, -es), e.b[j]);
    }
    if (EPI == EPI_GAUGED_EDGE || EPI == EPI_PLAIN_EDGE)
        v = (a.flt & FE_EDGE_TANH) ? edge_tanh(v) : (a.flt & FE_EDGE_ERF) ? edge_erf(v) : edge(v, e.PHI);
    *o = EPI == EPI_PLAIN_ADD ? wadd(*o, v) : v;
}

// CUDA-core bank product: one thread per output column, RT rows per CTA, the pile exact in int64.
template <int EPI, int RT>
__global__ void __launch_bounds__(256) k_bank_simt(BankArgs a) {
    griddep_wait();
    griddep_launch();
    __shared__ int32_t xs[RT][64];
    const int j = blockIdx.x * 256 + threadIdx.x;
    const int r0 = blockIdx.y * RT;
    int64_t acc[RT];
#pragma unroll
    for (int rr = 0; rr < RT; rr++) acc[rr] = 0;
    for (int k0 = 0; k0 < a.nin; k0 += 64) {
        for (int t = threadIdx.x; t < RT * 64; t += 256) {
            int rr = t >> 6, kk = t & 63, r = r0 + rr;
            xs[rr][kk] = (r < a.rows && k0 + kk < a.nin) ? a.x16[(size_t)r * a.nin + k0 + kk] : 0;
        }
        __syncthreads();
        if (j < a.nout) {
            const int kmax = a.nin - k0 < 64 ? a.nin - k0 : 64;
            const int16_t* wp = a.w + (size_t)k0 * a.nout + j;
            for (int kk = 0; kk < kmax; kk++) {
                int w = __ldg(wp + (size_t)kk * a.nout);
#pragma unroll
                for (int rr = 0; rr < RT; rr++) acc[rr] += (long long)w * (long long)xs[rr][kk];
            }
        }
        __syncthreads();
    }
    if (j >= a.nout) return;
    if (a.flt) {
        for (int rr = 0; rr < RT; rr++)
            if (r0 + rr < a.rows) epi_store_float<EPI>(a, r0 + rr, j, acc[rr]);
        return;
    }
#pragma unroll
    for (int rr = 0; rr < RT; rr++)
        if (r0 + rr < a.rows) epi_store<EPI>(a.epi, r0 + rr, j, acc[rr]);
}

// ---------------------------------------------------------------------------------------------------------------------
// q/k/v split (the Metal engine's heads16, base2_stream.swift:112-119; base2.py:93 to16 of q and k per head):
// one warp per (row, part of 3H). q16 -> per-row buffer; k16 + exponent -> key store (int16, with a bit mask of
// the entries equal to +32768, which int16 cannot hold); v -> value store as int32 (checked).
// ---------------------------------------------------------------------------------------------------------------------

__global__ void k_heads(const int64_t* __restrict__ QKV, int rows, const int32_t* __restrict__ row_slot,
                        const int32_t* __restrict__ row_pos, int layer, KV kv, int32_t* __restrict__ q16,
                        int32_t* __restrict__ qexp, uint32_t* err) {
    griddep_wait();
    griddep_launch();
    const int r = blockIdx.x, part = blockIdx.y, lane = threadIdx.x;
    const int H = kv.H, d = H * 64;
    if (r >= rows) return;
    const int64_t* x = QKV + (size_t)r * 3 * d + (size_t)part * 64;
    int64_t v0 = x[lane], v1 = x[lane + 32];
    const int slot = row_slot[r], pos = row_pos[r];
    if (part < 2 * H) {
        int sh = to16_shift(warp_or64(mag(v0) | mag(v1)));
        int64_t a0 = rshift(v0, sh), a1 = rshift(v1, sh);
        if (part < H) {
            q16[(size_t)r * d + part * 64 + lane] = (int32_t)a0;
            q16[(size_t)r * d + part * 64 + lane + 32] = (int32_t)a1;
            if (lane == 0) qexp[r * H + part] = -16 + sh;
        } else {
            if (pos < 0 || pos >= kv.lim) { if (lane == 0) set_err(err, DERR_POS); return; }
            size_t idx = kv_index(slot, layer, part - H, pos, kv.L, H, kv.ctx);
            kv.k[idx * 64 + lane] = (int16_t)(uint16_t)(uint32_t)a0;
            kv.k[idx * 64 + lane + 32] = (int16_t)(uint16_t)(uint32_t)a1;
            if (kv.kraw) { kv.kraw[idx * 64 + lane] = v0; kv.kraw[idx * 64 + lane + 32] = v1; }   // arrival=float
            uint32_t m0 = __ballot_sync(0xffffffffu, a0 == 32768), m1 = __ballot_sync(0xffffffffu, a1 == 32768);
            if (lane == 0) {
                kv.kmask[idx] = (uint64_t)m0 | ((uint64_t)m1 << 32);
                kv.kexp[idx] = -16 + sh;
            }
        }
    } else {
        if (pos < 0 || pos >= kv.lim) { if (lane == 0) set_err(err, DERR_POS); return; }
        size_t idx = kv_index(slot, layer, part - 2 * H, pos, kv.L, H, kv.ctx);
        bool bad = v0 != (int64_t)(int32_t)v0 || v1 != (int64_t)(int32_t)v1;
        if (__any_sync(0xffffffffu, bad) && lane == 0) set_err(err, DERR_VOVF);
        kv.v[idx * 64 + lane] = (int32_t)v0;
        kv.v[idx * 64 + lane + 32] = (int32_t)v1;
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// the arrival (base2.py:85-100; Metal attend, base2_stream.swift:120-133), one CTA of NW warps per (row, head):
//   pass 1: scores sc[s] = rshift(q16 . k16[s], -(eq + ek[s] - 3 + 10)) for s <= pos, kept in shared memory;
//   the clock starts at the largest score; pass 2: a = ARR[start - sc] (0 past the table), Z = sum a,
//   num = sum a * v; out = power(num, -log2fix(Z)).
// Shared memory: 8 bytes per key (dynamic).
// ---------------------------------------------------------------------------------------------------------------------
struct AttnArgs {
    const int32_t* row_slot;
    const int32_t* row_pos;
    int rows, layer;
    KV kv;
    const int32_t* q16;     // [rows][d]
    const int32_t* qexp;    // [rows][H]
    const int32_t* ARR;
    int alen;
    const int32_t* LOG2;
    const int32_t* EXP2;
    int64_t* out;           // [rows][d]
    uint32_t* err;
    uint64_t* or_out;       // optional [rows]: OR of |out| per row (the next bank's to16 shift)
    int64_t half;           // Pythia: log2(head size) / 2 at 2^-16 (the score's 1/sqrt(64) as a power)
    const int64_t* qf;      // arrival=float: the queries at full width, row r's head h at qf[r * ldq + h * 64]
    int ldq;
    uint64_t* trace = nullptr;   // optional (profiling aid): %globaltimer stamps [CTA][8] (k_attend_bulk)
    uint64_t* stamp = nullptr;   // b2_profile mode 2
    int early = 0;               // decode: keys before a row's own position come from earlier steps (k_attend_bulk
                                 // copies them before its dependency wait, the row's own key after it)
};

// the score of one key: GPT-2 rshift(q.k, -(eq + ek - 3 + 10)) (base2.py:94); Pythia power(q.k, (eq + ek + 10)*65536
// - HALF) (pythia_base2.py:135; |q.k| <= 64 * 2^30 < 2^45, the int64 power, whose left shift the reference bounds by
// 2^62: DERR_RANGE past it)
template <bool PY>
B2_DEV int64_t score(int64_t dot, int64_t eq, int64_t ek, const AttnArgs& a) {
    if (PY) {
        const int64_t F = (eq + ek + 10) * 65536 - a.half, s = 16 - (F >> 16);
        const int64_t p = dot * (int64_t)__ldg(a.EXP2 + (F & 0xFFFF));
        if (s < 0 && (s <= -62 || mag(p) >= (1ull << (62 + s)))) set_err(a.err, DERR_RANGE);
        return rshift(p, s);
    }
    return rshift(dot, -(eq + ek - 3 + 10));
}


template <int NW, bool PY>
__global__ void __launch_bounds__(NW * 32) k_attend(AttnArgs a) {
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    extern __shared__ int64_t sc[];           // [pos + 1]
    __shared__ int32_t qs[64];
    __shared__ int64_t red[NW][66];
    const int r = blockIdx.x, h = blockIdx.y;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int H = a.kv.H, d = H * 64;
    const int slot = a.row_slot[r], p = a.row_pos[r];
    if (p < 0 || p >= a.kv.lim) return;      // flagged by k_heads (DERR_POS); never read past the store
    const int nk = p + 1;
    if (threadIdx.x < 64) qs[threadIdx.x] = a.q16[(size_t)r * d + h * 64 + threadIdx.x];
    __syncthreads();
    const int64_t eq = a.qexp[r * H + h];
    const size_t base = kv_index(slot, a.layer, h, 0, a.kv.L, H, a.kv.ctx);
    const int16_t* K = a.kv.k + base * 64;
    const int32_t* Vv = a.kv.v + base * 64;
    const uint64_t* KM = a.kv.kmask + base;
    const int32_t* KE = a.kv.kexp + base;

    // ---- pass 1: lane holds 8 dims ((lane&7)*8..) of keys chunk*32 + (lane>>3) + 4i, i = 0..7
    int qr[8];
#pragma unroll
    for (int t = 0; t < 8; t++) qr[t] = qs[(lane & 7) * 8 + t];
    int64_t lmax = INT64_MIN;
    for (int c = wid; c * 32 < nk; c += NW) {
        int64_t part[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int key = c * 32 + (lane >> 3) + 4 * i;
            part[i] = 0;
            if (key < nk) {
                int4 raw = __ldg(reinterpret_cast<const int4*>(K + (size_t)key * 64 + (lane & 7) * 8));
                const int16_t* kk = reinterpret_cast<const int16_t*>(&raw);
                int64_t s = 0;
#pragma unroll
                for (int t = 0; t < 8; t++) s += (long long)qr[t] * (long long)kk[t];
                part[i] = s;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            part[i] += __shfl_xor_sync(0xffffffffu, part[i], 1);
            part[i] += __shfl_xor_sync(0xffffffffu, part[i], 2);
            part[i] += __shfl_xor_sync(0xffffffffu, part[i], 4);
        }
        if ((lane & 7) == 0) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                int key = c * 32 + (lane >> 3) + 4 * i;
                if (key < nk) {
                    int64_t dot = part[i];
                    uint64_t m = __ldg(KM + key);
                    while (m) { int t = __ffsll((long long)m) - 1; m &= m - 1; dot += 65536LL * qs[t]; }
                    int64_t s = score<PY>(dot, eq, (int64_t)__ldg(KE + key), a);
                    sc[key] = s;
                    lmax = s > lmax ? s : lmax;
                }
            }
        }
    }
    lmax = warp_max64(lmax);
    if (lane == 0) red[wid][0] = lmax;
    __syncthreads();
    int64_t start = red[0][0];
#pragma unroll
    for (int k = 1; k < NW; k++) start = red[k][0] > start ? red[k][0] : start;
    __syncthreads();

    // ---- pass 2: lane holds dims 2*lane, 2*lane+1; warps take keys round-robin, 4 in flight
    int64_t n0 = 0, n1 = 0, Z = 0;
    uint64_t vmax = 0;      // Pythia: the largest |v| met (pythia_base2.py:139 asserts max|v| * Z < 2^62)
    for (int s0 = wid * 4; s0 < nk; s0 += NW * 4) {
        int64_t av[4];
        int2 vv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            int s = s0 + u;
            av[u] = 0;
            vv[u] = make_int2(0, 0);
            if (s < nk) {
                av[u] = arrival(wsub(start, sc[s]), a.ARR, a.alen, a.err);
                if (av[u]) vv[u] = __ldg(reinterpret_cast<const int2*>(Vv + (size_t)s * 64) + lane);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            Z = wadd(Z, av[u]);
            n0 = wadd(n0, wmul(av[u], vv[u].x));
            n1 = wadd(n1, wmul(av[u], vv[u].y));
            if (PY && av[u]) vmax = max(vmax, max(mag(vv[u].x), mag(vv[u].y)));
        }
    }
    red[wid][2 * lane] = n0;
    red[wid][2 * lane + 1] = n1;
    if (lane == 0) red[wid][64] = Z;
    if (PY) { vmax = warp_max_u64(vmax); if (lane == 0) red[wid][65] = (int64_t)vmax; }
    __syncthreads();
    if (wid == 0) {
        int64_t t0 = 0, t1 = 0, zz = 0;
        uint64_t vm = 0;
#pragma unroll
        for (int k = 0; k < NW; k++) {
            t0 = wadd(t0, red[k][2 * lane]); t1 = wadd(t1, red[k][2 * lane + 1]); zz = wadd(zz, red[k][64]);
            if (PY) vm = max(vm, (uint64_t)red[k][65]);
        }
        int64_t F = -log2fix(zz, a.LOG2);
        int64_t* o = a.out + (size_t)r * d + h * 64;
        bool bad = PY && (unsigned __int128)vm * (unsigned __int128)(uint64_t)zz >= ((unsigned __int128)1 << 62);
        const int64_t v0 = PY ? power_exact(t0, F, a.EXP2, &bad) : power(t0, F, a.EXP2);
        const int64_t v1 = PY ? power_exact(t1, F, a.EXP2, &bad) : power(t1, F, a.EXP2);
        if (PY && bad) set_err(a.err, DERR_RANGE);
        o[2 * lane] = v0;
        o[2 * lane + 1] = v1;
        if (a.or_out) {
            const uint64_t w = warp_or64(mag(v0) | mag(v1));
            if (lane == 0) atomicOr((unsigned long long*)&a.or_out[r], (unsigned long long)w);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// the arrival with the stream's keys and their metadata for this head brought into shared memory by three bulk
// async copies at once (the whole run of positions 0..pos is contiguous in the store) and its values prefetched into
// L2 by a fourth, then:
//   pass 1  scores (8 lanes per key, 16-byte shared loads), the largest;   pass 1b  a = ARR[start - sc], Z = sum a;
//   pass 2  num = sum a * v (2 dims per lane, warps split the keys, values read from L2, four keys in flight);
//   out = power(num, -log2fix(Z)).
// Shared memory: 152 bytes per key (positions rounded up to 4), so that a decode step's (row, head) CTAs fit on the
// GPU at once. Used while the context fits; k_attend otherwise.
// ---------------------------------------------------------------------------------------------------------------------
constexpr int ATT_BYTES_PER_KEY = 128 + 8 + 4 + 8 + 4;

template <int NW, bool PY, int CS>
__global__ void __launch_bounds__(NW * 32) k_attend_bulk(AttnArgs a) {
    uint64_t* const tr = a.trace && CS == 1 ? a.trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 8 : nullptr;
#define ASTAMP(k_) \
    if (tr && threadIdx.x == 0) tr[k_] = gtime();
    ASTAMP(0)
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ uint64_t bar;
    __shared__ int32_t qs[64];
    __shared__ int64_t red[NW][66];
    __shared__ int64_t s_max, s_part[66];          // CS > 1: this CTA's largest score; its sums (64 dims, Z, max |v|)
    const int r = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int H = a.kv.H, d = H * 64;
    // decode (a.early): the row table and every key before the row's own position were written at least two launches
    // back (the step's first kernel, earlier steps), so they are read, and the keys copied, before the dependency wait;
    // L2 reads, never the non-coherent path. The row's own key (this step's qkv bank) is read after the wait.
    if (!a.early) {
        griddep_wait();
        stamp_begin(a.stamp);
        griddep_launch();
    }
    const int slot = __ldcg(a.row_slot + r), p = __ldcg(a.row_pos + r);
    if (p < 0 || p >= a.kv.lim) return;      // flagged by the qkv bank (DERR_POS); never read past the store (the
                                             // whole cluster returns: the row is the same for all its CTAs)
    const int nk = p + 1;
    // CS > 1: the CTAs of a cluster share the row's keys, rank c taking [k0, k0 + nl) (chunks of a multiple of 4 keys)
    const int c = CS > 1 ? (int)cluster_rank() : 0;
    const int chunk = CS > 1 ? (((nk + CS - 1) / CS + 3) & ~3) : nk;
    const int k0 = c * chunk, nl = max(0, min(nk - k0, chunk));
    const int nkr = (nl + 3) & ~3;           // keys this CTA copies and holds (from k0, a multiple of 4)
    int16_t* Ks = reinterpret_cast<int16_t*>(sm);
    uint64_t* KMs = reinterpret_cast<uint64_t*>(sm + (size_t)nkr * 128);
    int32_t* KEs = reinterpret_cast<int32_t*>(sm + (size_t)nkr * 136);
    int64_t* SCs = reinterpret_cast<int64_t*>(sm + (size_t)nkr * 140);
    int32_t* AVs = reinterpret_cast<int32_t*>(sm + (size_t)nkr * 148);
    const size_t base = kv_index(slot, a.layer, h, 0, a.kv.L, H, a.kv.ctx) + k0;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(&bar, (uint32_t)nkr * (128 + 8 + 4));
        if (nkr) {
            bulk_g2s(Ks, a.kv.k + base * 64, (uint32_t)nkr * 128, &bar);
            bulk_g2s(KMs, a.kv.kmask + base, (uint32_t)nkr * 8, &bar);
            bulk_g2s(KEs, a.kv.kexp + base, (uint32_t)nkr * 4, &bar);
            bulk_prefetch_l2(a.kv.v + base * 64, (uint32_t)nkr * 256);
        }
    }
    if (a.early) {
        griddep_wait();
        stamp_begin(a.stamp);
        griddep_launch();
    }
    ASTAMP(1)
    const int pl = p - k0;                   // the row's own key, local index (this CTA's when 0 <= pl < nl)
    const bool own = a.early && wid == 0 && pl >= 0 && pl < nl;
    uint32_t okw = 0;
    unsigned long long okm = 0;
    int32_t oke = 0;
    if (own) {                               // read now, with q; stored after the bulk copy that may cover its slot
        const size_t e = base + pl;
        okw = __ldcg(reinterpret_cast<const unsigned int*>(a.kv.k + e * 64) + lane);
        if (lane == 0) {
            okm = __ldcg((const unsigned long long*)a.kv.kmask + e);
            oke = __ldcg(a.kv.kexp + e);
        }
    }
    if (tid < 64) qs[tid] = a.q16[(size_t)r * d + h * 64 + tid];
    const int64_t eq = a.qexp[r * H + h];
    // a wait that gives up flags the call (DERR_TIMEOUT); a cluster's CTAs still meet at every barrier
    const bool copied = mbar_wait(&bar, 0, a.err);
    if (CS == 1 && !copied) return;
    if (own) {
        reinterpret_cast<uint32_t*>(Ks + (size_t)pl * 64)[lane] = okw;
        if (lane == 0) {
            KMs[pl] = okm;
            KEs[pl] = oke;
        }
    }
    __syncthreads();
    ASTAMP(2)

    // ---- pass 1: lane holds 8 dims ((lane&7)*8..) of key cc*4 + (lane>>3)
    int qr[8];
#pragma unroll
    for (int t = 0; t < 8; t++) qr[t] = qs[(lane & 7) * 8 + t];
    int64_t lmax = INT64_MIN;
    for (int cc = wid; cc * 4 < nl; cc += NW) {
        const int key = cc * 4 + (lane >> 3);
        int64_t part = 0;
        if (key < nl) {
            const int4 raw = reinterpret_cast<const int4*>(Ks + (size_t)key * 64)[lane & 7];
            const int16_t* kk = reinterpret_cast<const int16_t*>(&raw);
#pragma unroll
            for (int t = 0; t < 8; t++) part += (long long)qr[t] * (long long)kk[t];
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        if ((lane & 7) == 0 && key < nl) {
            uint64_t m = KMs[key];
            while (m) { const int t = __ffsll((long long)m) - 1; m &= m - 1; part += 65536LL * qs[t]; }
            const int64_t s = score<PY>(part, eq, (int64_t)KEs[key], a);
            SCs[key] = s;
            lmax = s > lmax ? s : lmax;
        }
    }
    lmax = warp_max64(lmax);
    if (lane == 0) red[wid][65] = lmax;
    __syncthreads();
    ASTAMP(3)
    int64_t start = red[0][65];
#pragma unroll
    for (int k = 1; k < NW; k++) start = red[k][65] > start ? red[k][65] : start;
    if (CS > 1) {                            // the row's largest score over the cluster's CTAs
        if (tid == 0) s_max = start;
        cluster_sync();
        const uint32_t off = saddr(&s_max);
#pragma unroll
        for (int q = 0; q < CS; q++) {
            const int64_t m = ld_dsmem(mapa(off, (uint32_t)q));
            start = m > start ? m : start;
        }
    }

    // ---- pass 1b: the arrival weights and their total
    int64_t z = 0;
    for (int s = tid; s < nl; s += NW * 32) {
        const int64_t av = arrival(wsub(start, SCs[s]), a.ARR, a.alen, a.err);
        AVs[s] = (int32_t)av;
        z = wadd(z, av);
    }
    z = warp_sum64(z);
    __syncthreads();                 // red[][65] read by everyone; AVs complete
    ASTAMP(4)
    if (lane == 0) red[wid][64] = z;

    // ---- pass 2: lane holds dims 2*lane, 2*lane+1; warps take keys round-robin, four keys' values in flight
    //      (a key whose weight is 0 adds 0, as skipping it would; Pythia's largest |v| only over weighted keys)
    int64_t n0 = 0, n1 = 0;
    uint64_t vmax = 0;
    const int2* Vg = reinterpret_cast<const int2*>(a.kv.v + base * 64);
    int s = wid;
    for (; s + 3 * NW < nl; s += 4 * NW) {
        int2 vv[4];
        int64_t av[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            av[u] = AVs[s + u * NW];
            vv[u] = Vg[(size_t)(s + u * NW) * 32 + lane];
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            n0 = wadd(n0, wmul(av[u], vv[u].x));
            n1 = wadd(n1, wmul(av[u], vv[u].y));
            if (PY && av[u]) vmax = max(vmax, max(mag(vv[u].x), mag(vv[u].y)));
        }
    }
    for (; s < nl; s += NW) {
        const int64_t av = AVs[s];
        if (!av) continue;
        const int2 vv = Vg[(size_t)s * 32 + lane];
        n0 = wadd(n0, wmul(av, vv.x));
        n1 = wadd(n1, wmul(av, vv.y));
        if (PY) vmax = max(vmax, max(mag(vv.x), mag(vv.y)));
    }
    red[wid][2 * lane] = n0;
    red[wid][2 * lane + 1] = n1;
    if (PY) { vmax = warp_max_u64(vmax); if (lane == 0) red[wid][65] = (int64_t)vmax; }
    __syncthreads();
    ASTAMP(5)
    int64_t t0 = 0, t1 = 0, zz = 0;
    uint64_t vm = 0;
    if (wid == 0) {
#pragma unroll
        for (int k = 0; k < NW; k++) {
            t0 = wadd(t0, red[k][2 * lane]); t1 = wadd(t1, red[k][2 * lane + 1]); zz = wadd(zz, red[k][64]);
            if (PY) vm = max(vm, (uint64_t)red[k][65]);
        }
    }
    if (CS > 1) {                            // the cluster's sums (wrapping int64 adds: any order gives the same bits)
        if (wid == 0) {
            s_part[2 * lane] = t0;
            s_part[2 * lane + 1] = t1;
            if (lane == 0) { s_part[64] = zz; s_part[65] = (int64_t)vm; }
        }
        cluster_sync();
        if (c == 0 && wid == 0) {
            t0 = t1 = zz = 0;
            vm = 0;
            const uint32_t o0 = saddr(&s_part[2 * lane]), o1 = saddr(&s_part[2 * lane + 1]), oz = saddr(&s_part[64]),
                           ov = saddr(&s_part[65]);
#pragma unroll
            for (int q = 0; q < CS; q++) {
                t0 = wadd(t0, ld_dsmem(mapa(o0, (uint32_t)q)));
                t1 = wadd(t1, ld_dsmem(mapa(o1, (uint32_t)q)));
                zz = wadd(zz, ld_dsmem(mapa(oz, (uint32_t)q)));
                if (PY) vm = max(vm, (uint64_t)ld_dsmem(mapa(ov, (uint32_t)q)));
            }
        }
    }
    if (wid == 0 && c == 0) {
        const int64_t F = -log2fix(zz, a.LOG2);
        int64_t* o = a.out + (size_t)r * d + h * 64;
        bool bad = PY && (unsigned __int128)vm * (unsigned __int128)(uint64_t)zz >= ((unsigned __int128)1 << 62);
        const int64_t v0 = PY ? power_exact(t0, F, a.EXP2, &bad) : power(t0, F, a.EXP2);
        const int64_t v1 = PY ? power_exact(t1, F, a.EXP2, &bad) : power(t1, F, a.EXP2);
        if (PY && bad) set_err(a.err, DERR_RANGE);
        o[2 * lane] = v0;
        o[2 * lane + 1] = v1;
        if (a.or_out) {
            const uint64_t w = warp_or64(mag(v0) | mag(v1));
            if (lane == 0) atomicOr((unsigned long long*)&a.or_out[r], (unsigned long long)w);
        }
        ASTAMP(6)
    }
    if (CS > 1) cluster_sync();              // no CTA leaves while rank 0 may still read its sums
#undef ASTAMP
}

// ---------------------------------------------------------------------------------------------------------------------
// the arrival in a prompt pass (base2.py:85-100; pythia_base2.py:125-141): a block of up to QB consecutive prompt
// positions of one stream per CTA and head, so that each key / value tile brought into shared memory serves all QB
// queries (per-row arrivals would read every earlier key once per row):
//   pass 1  the score of every (query, key <= the query's position) pair into shared memory, each query's largest;
//   pass 2  a = ARR[start - sc] (0 past the table), Z = sum a, per query;
//   pass 3  num = sum a * v over value tiles, out = power(num, -log2fix(Z)).
// The arithmetic is k_attend's, query by query (wrapping int64 sums; Pythia's exact power and range checks).
// Shared memory: QB x max_ctx int64 (scores, then arrival weights) + the tiles (prefill_smem()).
// ---------------------------------------------------------------------------------------------------------------------
struct PrefillBlock {
    int row0, nr, slot, pos0;      // rows row0 .. row0 + nr - 1 are positions pos0 .. of stream slot `slot`
};
constexpr int PF_KT = 64;          // keys per tile
constexpr int PF_KROW = 66;        // int16 per key row in shared memory (64 + 2: conflict-free row-per-lane reads)
inline size_t prefill_smem(int qb, int nkmax) {
    return (size_t)qb * nkmax * 8 + (size_t)qb * 64 * 4 + (size_t)PF_KT * PF_KROW * 2 + PF_KT * 8 + PF_KT * 4 +
           (size_t)PF_KT * 64 * 4;
}

template <int QB, bool PY>
__global__ void __launch_bounds__(256) k_attend_prefill(AttnArgs a, const PrefillBlock* __restrict__ blocks, int nkmax) {
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int64_t s_max[QB][2], s_eq[QB], s_Z[QB];
    __shared__ uint64_t s_vm[QB];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const PrefillBlock blk = blocks[blockIdx.x];
    const int h = blockIdx.y, H = a.kv.H, d = H * 64;
    const int nr = blk.nr, pos0 = blk.pos0, nk = pos0 + nr;
    if (pos0 < 0 || nr < 1 || nr > QB || nk > a.kv.lim || nk > nkmax) return;   // flagged by the heads kernel
    int64_t* S = reinterpret_cast<int64_t*>(sm);                          // [QB][nkmax]
    int32_t* Qs = reinterpret_cast<int32_t*>(S + (size_t)QB * nkmax);      // [QB][64]
    int16_t* Kt = reinterpret_cast<int16_t*>(Qs + QB * 64);               // [PF_KT][PF_KROW]
    uint64_t* KMt = reinterpret_cast<uint64_t*>(Kt + PF_KT * PF_KROW);    // [PF_KT]
    int32_t* KEt = reinterpret_cast<int32_t*>(KMt + PF_KT);               // [PF_KT]
    int32_t* Vt = KEt + PF_KT;                                            // [PF_KT][64]
    for (int i = tid; i < QB * 64; i += 256) {
        const int q = i >> 6, t = i & 63;
        Qs[i] = q < nr ? a.q16[(size_t)(blk.row0 + q) * d + h * 64 + t] : 0;
    }
    if (tid < QB) {
        s_eq[tid] = tid < nr ? (int64_t)a.qexp[(blk.row0 + tid) * H + h] : 0;
        s_vm[tid] = 0;
    }
    const size_t base = kv_index(blk.slot, a.layer, h, 0, a.kv.L, H, a.kv.ctx);

    // ---- pass 1: thread (key kl of the tile, query group qg): queries qg, qg + 4, .. ----
    constexpr int QPT = QB / 4;
    const int kl = tid & 63, qg = tid >> 6;
    int64_t lmax[QPT];
#pragma unroll
    for (int i = 0; i < QPT; i++) lmax[i] = INT64_MIN;
    for (int k0 = 0; k0 < nk; k0 += PF_KT) {
        __syncthreads();                                                  // the previous tile is consumed
        {
            const int r = tid >> 2, c = tid & 3, key = k0 + r;
            uint32_t* dst = reinterpret_cast<uint32_t*>(Kt + r * PF_KROW) + c * 8;
            int4 v0 = make_int4(0, 0, 0, 0), v1 = make_int4(0, 0, 0, 0);
            if (key < nk) {
                const int4* src = reinterpret_cast<const int4*>(a.kv.k + (base + key) * 64) + c * 2;
                v0 = src[0];
                v1 = src[1];
            }
            dst[0] = v0.x; dst[1] = v0.y; dst[2] = v0.z; dst[3] = v0.w;
            dst[4] = v1.x; dst[5] = v1.y; dst[6] = v1.z; dst[7] = v1.w;
            if (tid < PF_KT) {
                const int kk = k0 + tid;
                KMt[tid] = kk < nk ? a.kv.kmask[base + kk] : 0;
                KEt[tid] = kk < nk ? a.kv.kexp[base + kk] : 0;
            }
        }
        __syncthreads();
        const int key = k0 + kl;
        if (key < nk) {
            uint32_t kw[32];
            const uint32_t* kr = reinterpret_cast<const uint32_t*>(Kt + kl * PF_KROW);
#pragma unroll
            for (int w = 0; w < 32; w++) kw[w] = kr[w];
            const uint64_t mk0 = KMt[kl];
            const int64_t ek = KEt[kl];
#pragma unroll
            for (int i = 0; i < QPT; i++) {
                const int q = qg + 4 * i;
                if (q >= nr || key > pos0 + q) continue;                 // causal: keys up to the query's own position
                const int32_t* qr = Qs + q * 64;
                int64_t d4[4] = {0, 0, 0, 0};                          // four independent sums (latency)
#pragma unroll
                for (int w = 0; w < 32; w++) {
                    // |q|, |k| <= 32768: each product fits int32 (a pair's sum may not: (-32768)^2 * 2 = 2^31)
                    d4[(2 * w) & 3] += (int64_t)(qr[2 * w] * (int32_t)(int16_t)(kw[w] & 0xFFFF));
                    d4[(2 * w + 1) & 3] += (int64_t)(qr[2 * w + 1] * (int32_t)(int16_t)(kw[w] >> 16));
                }
                int64_t dot = (d4[0] + d4[1]) + (d4[2] + d4[3]);
                uint64_t mk = mk0;
                while (mk) { const int t = __ffsll((long long)mk) - 1; mk &= mk - 1; dot += 65536LL * qr[t]; }
                const int64_t sc = score<PY>(dot, s_eq[q], ek, a);
                S[(size_t)q * nkmax + key] = sc;
                lmax[i] = sc > lmax[i] ? sc : lmax[i];
            }
        }
    }
    // each query's largest score: its 64 threads are warps 2 qg and 2 qg + 1
#pragma unroll
    for (int i = 0; i < QPT; i++) {
        const int64_t m = warp_max64(lmax[i]);
        if (lane == 0) s_max[qg + 4 * i][wid & 1] = m;
    }
    __syncthreads();

    // ---- pass 2: arrival weights in place of the scores, Z per query (256 / QB threads per query) ----
    constexpr int TPQ = 256 / QB;
    {
        const int q = tid / TPQ, sub = tid % TPQ;
        int64_t z = 0;
        if (q < nr) {
            const int64_t start = s_max[q][0] > s_max[q][1] ? s_max[q][0] : s_max[q][1];
            for (int key = sub; key <= pos0 + q; key += TPQ) {
                const int64_t av = arrival(wsub(start, S[(size_t)q * nkmax + key]), a.ARR, a.alen, a.err);
                S[(size_t)q * nkmax + key] = av;
                z = wadd(z, av);
            }
        }
#pragma unroll
        for (int o = TPQ / 2; o > 0; o >>= 1) z = wadd(z, __shfl_xor_sync(0xffffffffu, z, o));
        if (sub == 0 && q < QB) s_Z[q] = z;
    }

    // ---- pass 3: num = sum a v; thread (query q, DPT dims) ----
    constexpr int DPT = 64 / TPQ;
    const int q = tid / TPQ, dg = tid % TPQ;
    int64_t num[DPT];
#pragma unroll
    for (int j = 0; j < DPT; j++) num[j] = 0;
    uint64_t vm = 0;
    for (int k0 = 0; k0 < nk; k0 += PF_KT) {
        __syncthreads();                                                  // pass 2 / the previous value tile is done
        for (int i = tid; i < PF_KT * 16; i += 256) {
            const int r = i >> 4, c = i & 15, key = k0 + r;
            reinterpret_cast<int4*>(Vt)[i] =
                key < nk ? reinterpret_cast<const int4*>(a.kv.v + (base + key) * 64)[c] : make_int4(0, 0, 0, 0);
        }
        __syncthreads();
        if (q < nr) {
            const int kend = min(PF_KT, pos0 + q + 1 - k0);
            for (int r = 0; r < kend; r++) {
                const int64_t av = S[(size_t)q * nkmax + k0 + r];
                if (!av) continue;
                const int32_t* vr = Vt + r * 64 + dg * DPT;
#pragma unroll
                for (int j = 0; j < DPT; j++) {
                    num[j] = wadd(num[j], wmul(av, vr[j]));
                    if (PY) vm = max(vm, mag(vr[j]));
                }
            }
        }
    }
    if (PY) {
        __syncthreads();
        if (q < nr) atomicMax((unsigned long long*)&s_vm[q], (unsigned long long)vm);
        __syncthreads();
    }
    if (q < nr) {
        const int64_t zz = s_Z[q];
        const int64_t F = -log2fix(zz, a.LOG2);
        bool bad = PY && (unsigned __int128)s_vm[q] * (unsigned __int128)(uint64_t)zz >= ((unsigned __int128)1 << 62);
        int64_t* o = a.out + (size_t)(blk.row0 + q) * d + h * 64 + dg * DPT;
#pragma unroll
        for (int j = 0; j < DPT; j++) o[j] = PY ? power_exact(num[j], F, a.EXP2, &bad) : power(num[j], F, a.EXP2);
        if (PY && bad) set_err(a.err, DERR_RANGE);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// the race at the top (base2.py:34-40): argmax with ties to the lowest index; one CTA per scored row
// ---------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_race(const int64_t* __restrict__ logits, int ld, const int32_t* __restrict__ rows_map,
                                               int V, int32_t* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    __shared__ int64_t sv[32];
    __shared__ int si[32];
    const int r = rows_map ? rows_map[blockIdx.x] : blockIdx.x;
    const int64_t* x = logits + (size_t)r * ld;
    int64_t v = INT64_MIN;
    int i = 0x7fffffff;
    for (int t = threadIdx.x; t < V; t += 1024) race_merge(v, i, x[t], t);
    warp_race(v, i);
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = v; si[threadIdx.x >> 5] = i; }
    __syncthreads();
    if (threadIdx.x < 32) {
        v = sv[threadIdx.x];
        i = si[threadIdx.x];
        warp_race(v, i);
        if (threadIdx.x == 0) out[r] = i;
    }
}

// the race over a head epilogue's per-group winners (TcRace): row r's word is the best of v[r][0..nparts), ties to the
// lowest column
__global__ void __launch_bounds__(256) k_race_parts(const int64_t* __restrict__ pv, const int32_t* __restrict__ pi, int ld,
                                                    int nparts, int32_t* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    __shared__ int64_t sv[8];
    __shared__ int si[8];
    const int r = blockIdx.x;
    int64_t v = INT64_MIN;
    int i = 0x7fffffff;
    for (int t = threadIdx.x; t < nparts; t += 256) race_merge(v, i, pv[(size_t)r * ld + t], pi[(size_t)r * ld + t]);
    warp_race(v, i);
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = v; si[threadIdx.x >> 5] = i; }
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < 8 ? sv[threadIdx.x] : INT64_MIN;
        i = threadIdx.x < 8 ? si[threadIdx.x] : 0x7fffffff;
        warp_race(v, i);
        if (threadIdx.x == 0) out[r] = i;
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// row bookkeeping for a decode step: one row per stream slot, at the slot's next position
// ---------------------------------------------------------------------------------------------------------------------
__global__ void k_decode_rows(int n, const int32_t* __restrict__ tok_in, const int32_t* __restrict__ slot_len,
                              const int32_t* __restrict__ slot_tok, int32_t* row_slot, int32_t* row_pos, int32_t* row_tok) {
    griddep_wait();
    griddep_launch();
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    row_slot[s] = s;
    row_pos[s] = slot_len[s];
    row_tok[s] = tok_in ? tok_in[s] : slot_tok[s];
}

// a decode step's first kernel: row s = stream slot s at its next position, R = wte[tok] + wpe[pos], the row's OR
// of magnitudes (the qkv bank's to16 shift) into or_buf[0], and the step's other OR slots or_buf[1..nor) cleared
__global__ void k_embed_decode(int n, const int32_t* __restrict__ slot_len, const int32_t* __restrict__ slot_tok,
                               int32_t* row_slot, int32_t* row_pos, int32_t* row_tok, const int64_t* __restrict__ wte,
                               const int64_t* __restrict__ wpe, int d, int V, int nctx, int64_t* __restrict__ R,
                               uint64_t* or_buf, int nor, int or_ld, int64_t* acc, int32_t* accn, uint32_t* err) {
    griddep_wait();
    griddep_launch();
    __shared__ uint64_t s_or[8];
    const int s = blockIdx.x;
    if (s >= n) return;
    int tok = slot_tok[s], pos = slot_len[s];
    if (threadIdx.x == 0) { row_slot[s] = s; row_pos[s] = pos; row_tok[s] = tok; }
    if (tok < 0 || tok >= V) { if (threadIdx.x == 0) set_err(err, DERR_TOKEN); tok = 0; }
    if (pos < 0 || pos >= nctx) { if (threadIdx.x == 0) set_err(err, DERR_POS); pos = 0; }
    const int64_t* a = wte + (size_t)tok * d;
    const int64_t* b = wpe ? wpe + (size_t)pos * d : nullptr;   // Pythia: no position table
    uint64_t o = 0;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const int64_t v = b ? wadd(__ldg(a + i), __ldg(b + i)) : __ldg(a + i);
        R[(size_t)s * d + i] = v;
        o |= mag(v);
    }
    for (int q = 1 + threadIdx.x; q < nor; q += blockDim.x) or_buf[(size_t)q * or_ld + s] = 0;
    // the in-kernel quantisation's per-row accumulators of every bank input ([2][nor][or_ld] S1, S2; [nor][or_ld])
    if (acc)
        for (int q = threadIdx.x; q < nor; q += blockDim.x) {
            acc[(size_t)q * or_ld + s] = 0;
            acc[(size_t)(nor + q) * or_ld + s] = 0;
            accn[(size_t)q * or_ld + s] = 0;
        }
    o = warp_or64(o);
    if ((threadIdx.x & 31) == 0) s_or[threadIdx.x >> 5] = o;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t all = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) all |= s_or[w];
        or_buf[s] = all;
    }
}


// where a decode step's words go: out[s * ld + (slot_len[s] - base[s])], set once per call (k_gen_begin), so one
// captured step graph serves every call and every position
struct GenDesc {
    int32_t* out;
    int ld;
};

__global__ void k_gen_begin(int n, const int32_t* __restrict__ slot_len, int32_t* base, GenDesc* desc, int32_t* out, int ld) {
    griddep_wait();
    griddep_launch();
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < n) base[s] = slot_len[s];
    if (s == 0) { desc->out = out; desc->ld = ld; }
}

// after the race: the word goes straight back in (base2_stream.swift:143-146); stream lengths advance
// b2_check_wait: the bounded wait of every TMA / bulk-copy completion (mbar_wait) on an mbarrier that expects 16
// bytes no copy will ever bring (a flag nothing sets). The wait gives up after the handle's limit and sets
// DERR_TIMEOUT; nothing faults and the context stays usable.
__global__ void k_wait_check(uint32_t* err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_expect_tx(&bar, 16);
        mbar_wait(&bar, 0, err);
    }
    __syncwarp();
}

// b2_profile mode 2: a unit of work (a decode step, a prompt-pass chunk) begins by clearing its stamp slots ...
__global__ void k_stamp_reset(uint64_t* slots, int n) {
    griddep_wait();
    griddep_launch();
    for (int i = threadIdx.x; i < n; i += blockDim.x) slots[i] = ~0ull;
}
// ... and ends by turning them into durations: a stamped kernel lasted from its start to the next stamped start of any
// class (or to this kernel's own start), so a kernel without a slot is counted in the stamped one before it.
// tot[2c] += ns, tot[2c + 1] += launches of class c.
struct StampUse {
    int n[8];   // slots used per class in this unit of work
};
__global__ void __launch_bounds__(1024) k_stamp_accum(const uint64_t* slots, StampUse use, int per_class, uint64_t* tot) {
    griddep_wait();
    griddep_launch();
    __shared__ uint64_t t_end;
    __shared__ int off[9];
    if (threadIdx.x == 0) {
        t_end = gtime();
        off[0] = 0;
        for (int c = 0; c < 8; c++) off[c + 1] = off[c] + use.n[c];
    }
    __syncthreads();
    const int n = off[8];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int c = 0;
        while (i >= off[c + 1]) c++;
        const uint64_t s = slots[(size_t)c * per_class + (i - off[c])];
        if (s == ~0ull) continue;
        uint64_t next = t_end;
        for (int cc = 0; cc < 8; cc++)
            for (int j = 0; j < use.n[cc]; j++) {
                const uint64_t u = slots[(size_t)cc * per_class + j];
                if (u != ~0ull && u > s && u < next) next = u;
            }
        if (next <= s) continue;
        atomicAdd((unsigned long long*)&tot[2 * c], (unsigned long long)(next - s));
        atomicAdd((unsigned long long*)&tot[2 * c + 1], 1ull);
    }
}

__global__ void k_decode_commit(int n, const int32_t* __restrict__ word, int32_t* slot_len, int32_t* slot_tok,
                                const GenDesc* __restrict__ desc, const int32_t* __restrict__ base) {
    griddep_wait();
    griddep_launch();
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    int w = word[s];
    int len = slot_len[s];
    slot_len[s] = len + 1;
    slot_tok[s] = w;
    int32_t* out = desc->out;
    if (out) out[(size_t)s * desc->ld + (len - base[s])] = w;
}

// ---------------------------------------------------------------------------------------------------------------------
// float stage switches (see b2_float.cuh): the gauge's sigma, Pythia's float norm, the float arrival. One CTA per
// row (per row and head for the arrival); the pairwise sums run in one thread, in numpy's order.
// ---------------------------------------------------------------------------------------------------------------------
// the row at 2^-16 into x[], x - mean into x[], (x - mean)^2 into t[]; returns sqrt(mean t + 1e-5)
// (base2.py:67, pythia_base2.py:103). Block-wide; d <= the shared arrays' length.
template <int NT>
__device__ double row_sigma(const int64_t* __restrict__ R, int d, double* x, double* t) {
    __shared__ double s_mu, s_sg;
    for (int i = threadIdx.x; i < d; i += NT) x[i] = __ddiv_rn(i2d(R[i]), 65536.0);
    __syncthreads();
    if (threadIdx.x == 0) s_mu = __ddiv_rn(pairwise_sum(x, d), (double)d);
    __syncthreads();
    const double mu = s_mu;
    for (int i = threadIdx.x; i < d; i += NT) { const double c = __dsub_rn(x[i], mu); x[i] = c; t[i] = __dmul_rn(c, c); }
    __syncthreads();
    if (threadIdx.x == 0) s_sg = __dsqrt_rn(__dadd_rn(__ddiv_rn(pairwise_sum(t, d), (double)d), 1e-5));
    __syncthreads();
    return s_sg;
}

constexpr int FLT_MAXD = 1024;   // the float norms take rows of up to 1,024 (d = 768 here)

// GPT-2 gauge=float: sig[r] of row src_rows[r] (or r) of R (base2.py:67 and :111)
template <int NT>
__global__ void __launch_bounds__(NT) k_sigma(const int64_t* __restrict__ R, int d, const int32_t* __restrict__ src_rows,
                                             int rows, double* __restrict__ sig) {
    griddep_wait();
    griddep_launch();
    __shared__ double x[FLT_MAXD], t[FLT_MAXD];
    const int r = blockIdx.x;
    if (r >= rows || d > FLT_MAXD) return;
    const double s = row_sigma<NT>(R + (size_t)(src_rows ? src_rows[r] : r) * d, d, x, t);
    if (threadIdx.x == 0) sig[r] = s;
}

// Pythia gauge=float (pythia_base2.py:102-104): round((x - mu) / sg * g * 2^ge * 2^16) + b
template <int NT>
__global__ void __launch_bounds__(NT) k_gauge_ln_float(const int64_t* __restrict__ R, int d,
                                                      const int32_t* __restrict__ src_rows, int rows,
                                                      const int64_t* __restrict__ g, int64_t ge,
                                                      const int64_t* __restrict__ b, int64_t* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    __shared__ double x[FLT_MAXD], t[FLT_MAXD];
    const int r = blockIdx.x;
    if (r >= rows || d > FLT_MAXD) return;
    const double sg = row_sigma<NT>(R + (size_t)(src_rows ? src_rows[r] : r) * d, d, x, t);
    const double sc = scalbn(1.0, (int)ge);
    for (int i = threadIdx.x; i < d; i += NT)
        out[(size_t)r * d + i] =
            wadd(rint64(__dmul_rn(__dmul_rn(__dmul_rn(__ddiv_rn(x[i], sg), i2d(g[i])), sc), 65536.0)), b[i]);
}

// arrival=float (base2.py:89-92, pythia_base2.py:130-133) for row r at position p, head h: s = (q/2^16).(k/2^16)/8
// (the dot exact in 128 bits, rounded once), a = exp(s - max s) / (pairwise sum), out = round(sum_s a v / 2^16 * 2^16)
// with the sum over s in order. 64 threads (one per output dim); dynamic shared memory: 8 bytes per key.
__global__ void __launch_bounds__(64) k_attend_float(AttnArgs a) {
    griddep_wait();
    griddep_launch();
    extern __shared__ double e[];
    __shared__ int64_t qs[64];
    __shared__ double red[2], s_Z;
    const int r = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const int H = a.kv.H, d = H * 64;
    const int slot = a.row_slot[r], p = a.row_pos[r];
    if (p < 0 || p >= a.kv.lim) return;      // flagged by the heads kernel (DERR_POS)
    const int nk = p + 1;
    qs[tid] = a.qf[(size_t)r * a.ldq + h * 64 + tid];
    __syncthreads();
    const size_t base = kv_index(slot, a.layer, h, 0, a.kv.L, H, a.kv.ctx);
    double mx = -INFINITY;
    for (int s = tid; s < nk; s += 64) {
        const int64_t* k = a.kv.kraw + (base + s) * 64;
        __int128 dot = 0;
        for (int t = 0; t < 64; t++) dot += (__int128)qs[t] * (__int128)k[t];
        const double v = __ddiv_rn(scalbn(i128_to_double(dot), -32), 8.0);
        e[s] = v;
        mx = fmax(mx, v);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmax(red[0], red[1]);
    for (int s = tid; s < nk; s += 64) e[s] = exp(__dsub_rn(e[s], mx));
    __syncthreads();
    if (tid == 0) s_Z = pairwise_sum(e, nk);
    __syncthreads();
    const double Z = s_Z;
    for (int s = tid; s < nk; s += 64) e[s] = __ddiv_rn(e[s], Z);
    __syncthreads();
    const int32_t* V = a.kv.v + base * 64 + tid;
    double acc = 0.0;
    for (int s = 0; s < nk; s++) acc = __dadd_rn(acc, __dmul_rn(e[s], __ddiv_rn((double)V[(size_t)s * 64], 65536.0)));
    a.out[(size_t)r * d + h * 64 + tid] = rint64(__dmul_rn(acc, 65536.0));
}

// truncate streams back to lens[s] positions (never forward), last_tok[s] fed next
__global__ void k_rewind(int n, const int32_t* __restrict__ lens, const int32_t* __restrict__ last_tok, int V,
                         int32_t* slot_len, int32_t* slot_tok, uint32_t* err) {
    griddep_wait();
    griddep_launch();
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    int l = lens[s], t = last_tok[s];
    if (l < 1 || l > slot_len[s]) { set_err(err, DERR_POS); return; }
    if (t < 0 || t >= V) { set_err(err, DERR_TOKEN); return; }
    slot_len[s] = l;
    slot_tok[s] = t;
}

// prompt rows for a chunk [r0, r0 + rows) of the concatenated prompts
__global__ void k_prefill_rows(int r0, int rows, const int32_t* __restrict__ row_slot_all,
                               const int32_t* __restrict__ row_pos_all, const int32_t* __restrict__ ids,
                               int32_t* row_slot, int32_t* row_pos, int32_t* row_tok) {
    griddep_wait();
    griddep_launch();
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows) return;
    row_slot[t] = row_slot_all[r0 + t];
    row_pos[t] = row_pos_all[r0 + t];
    row_tok[t] = ids[r0 + t];
}

}  // namespace b2

namespace b2 {

// ---------------------------------------------------------------------------------------------------------------------
// The exact collapsing top read (the reference's top=fr, base2_stream_fr2.swift:23-38, kernels :194-406, host
// :832-898), for decode steps of a few streams whose scores are not stored. A head weight is w = 256 wh + lo with
// wh = w >> 8 (the wh plane) and lo = w & 255 = wl + 128 (the wl plane), so a word's pile is 256 C + L with
// C = sum wh x over the whole plane and L = sum lo x in [255 SN, 255 SP] (SN, SP: the sums of the input's negative
// and positive values). The head's epilogue is non-decreasing in the pile (no wrap: |pile| < 2^42), so every word has
// a low and a high score; T5 is the 5th-best low (larger, then lower slot), and a word whose high is below T5 is below
// five other words' exact scores: only the words still in read their wl rows and get the exact score, and the race
// runs among them (largest, ties to the lowest slot: base2.py:34-40). Bit-exact with the plain race.
// ---------------------------------------------------------------------------------------------------------------------
constexpr int TOPFR_ROWS = 4;    // streams per decode step the collapsing read takes
constexpr int TOPFR_NIN = 768;   // the head's inputs (a lane holds 24 of them)

struct TopFrArgs {
    const int8_t* wh;            // [nout_pad][nin] K-major (word by word)
    const int8_t* wl;
    const int32_t* x16;          // [rows][nin] the head's input, to16'd (k_quant)
    const int32_t* ex;           // [rows]
    const int64_t* LS;           // [rows] (gauged head)
    const int32_t* e;            // [nout]
    const int64_t* b;            // [nout]
    const int32_t* EXP2;
    int nout, rows;
    int64_t* C;                  // [TOPFR_ROWS][nout] every word's coarse sum (sum wh x)
    int64_t* HIS;                // [TOPFR_ROWS][nout] its high score
    int64_t* p5v;                // [TOPFR_ROWS][nparts][5] each coarse CTA's five best lows
    int32_t* p5i;
    int nparts;
    int32_t* list;               // [TOPFR_ROWS][nout] the words still in
    int32_t* cnt;                // [TOPFR_ROWS]
    int64_t* sv;                 // [TOPFR_ROWS][nfin] each finishing CTA's best (score, word)
    int32_t* si;
    int nfin;
    uint64_t* stamp;             // b2_profile mode 2 (the coarse read)
};

// (larger score, then lower slot) first: the race's own order
B2_DEV bool fr_better(int64_t a, int ia, int64_t b, int ib) { return a > b || (a == b && ia < ib); }
B2_DEV void fr_put5(int64_t* v, int* ix, int64_t u, int iu) {
    if (!fr_better(u, iu, v[4], ix[4])) return;
    v[4] = u;
    ix[4] = iu;
#pragma unroll
    for (int k = 4; k > 0; k--)
        if (fr_better(v[k], ix[k], v[k - 1], ix[k - 1])) {
            const int64_t tv = v[k]; v[k] = v[k - 1]; v[k - 1] = tv;
            const int ti = ix[k]; ix[k] = ix[k - 1]; ix[k - 1] = ti;
        }
}
template <int EPI>
B2_DEV int64_t fr_score(int64_t pile, int j, int r, const TopFrArgs& a) {
    const int64_t ex = a.ex[r];
    const int64_t LS = EPI == EPI_GAUGED ? a.LS[r] : 0;
    const int64_t e2 = EPI == EPI_GAUGED ? (int64_t)__ldg(a.EXP2 + (wsub(0, LS) & 0xFFFF)) : 0;
    return epi_value<EPI>(pile, (int64_t)a.e[j], a.b[j], ex, LS, e2, nullptr);
}
// this lane's 24 inputs of row r (inputs 16 lane .. + 16 and 512 + 8 lane .. + 8) and the row's S1, SP, SN
B2_DEV void fr_row(const TopFrArgs& a, int r, int lane, int (&x)[24], int64_t& S1, int64_t& SP, int64_t& SN) {
    const int32_t* xr = a.x16 + (size_t)r * TOPFR_NIN;
    const int4* p = reinterpret_cast<const int4*>(xr + 16 * lane);
    const int4* q = reinterpret_cast<const int4*>(xr + 512 + 8 * lane);
    int4 t[6] = {p[0], p[1], p[2], p[3], q[0], q[1]};
#pragma unroll
    for (int u = 0; u < 6; u++) { x[4 * u] = t[u].x; x[4 * u + 1] = t[u].y; x[4 * u + 2] = t[u].z; x[4 * u + 3] = t[u].w; }
    int64_t s1 = 0, sp = 0, sn = 0;
#pragma unroll
    for (int u = 0; u < 24; u++) { s1 += x[u]; if (x[u] > 0) sp += x[u]; else sn += x[u]; }
    S1 = warp_sum64(s1);
    SP = warp_sum64(sp);
    SN = warp_sum64(sn);
}
// sum over the word's 768 bytes of a plane times the input: lane takes bytes 16 lane .. + 16 and 512 + 8 lane .. + 8
B2_DEV int64_t fr_dot(const int8_t* row, const int (&x)[24], int lane) {
    const int4 u = *reinterpret_cast<const int4*>(row + 16 * lane);
    const int2 v = *reinterpret_cast<const int2*>(row + 512 + 8 * lane);
    const uint32_t wd[6] = {(uint32_t)u.x, (uint32_t)u.y, (uint32_t)u.z, (uint32_t)u.w, (uint32_t)v.x, (uint32_t)v.y};
    int s = 0;                                   // |byte x| <= 2^22, 24 of them < 2^27
#pragma unroll
    for (int k = 0; k < 6; k++)
#pragma unroll
        for (int t = 0; t < 4; t++) s += (int)(int8_t)(wd[k] >> (8 * t)) * x[4 * k + t];
    return warp_sum64((int64_t)s);
}

// (a)-(c): every word's coarse sum and its low and high score; each CTA's five best lows per row. A warp per word.
template <int EPI>
__global__ void __launch_bounds__(256) k_top_coarse(TopFrArgs a) {
    griddep_wait();
    stamp_begin(a.stamp);
    griddep_launch();
    __shared__ int64_t s5v[TOPFR_ROWS][8][5];
    __shared__ int s5i[TOPFR_ROWS][8][5];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int64_t bv[TOPFR_ROWS][5];
    int bi[TOPFR_ROWS][5];
#pragma unroll
    for (int r = 0; r < TOPFR_ROWS; r++)
#pragma unroll
        for (int k = 0; k < 5; k++) { bv[r][k] = INT64_MIN; bi[r][k] = 0x7fffffff; }
    const int gw = blockIdx.x * 8 + wid, nw = gridDim.x * 8;
#pragma unroll
    for (int r = 0; r < TOPFR_ROWS; r++) {
        if (r >= a.rows) break;
        int x[24];
        int64_t S1, SP, SN;
        fr_row(a, r, lane, x, S1, SP, SN);
        for (int j = gw; j < a.nout; j += nw) {
            const int64_t c = fr_dot(a.wh + (size_t)j * TOPFR_NIN, x, lane);
            if (lane == 0) {
                const int64_t lo = fr_score<EPI>(256 * c + 255 * SN, j, r, a);
                const int64_t hi = fr_score<EPI>(256 * c + 255 * SP, j, r, a);
                a.C[(size_t)r * a.nout + j] = c;
                a.HIS[(size_t)r * a.nout + j] = hi;
                fr_put5(bv[r], bi[r], lo, j);
            }
        }
        if (lane == 0)
#pragma unroll
            for (int k = 0; k < 5; k++) { s5v[r][wid][k] = bv[r][k]; s5i[r][wid][k] = bi[r][k]; }
    }
    __syncthreads();
    if (threadIdx.x < TOPFR_ROWS && (int)threadIdx.x < a.rows) {
        const int r = threadIdx.x;
        int64_t v[5];
        int ix[5];
#pragma unroll
        for (int k = 0; k < 5; k++) { v[k] = INT64_MIN; ix[k] = 0x7fffffff; }
        for (int w = 0; w < 8; w++)
#pragma unroll
            for (int k = 0; k < 5; k++) fr_put5(v, ix, s5v[r][w][k], s5i[r][w][k]);
        for (int k = 0; k < 5; k++) {
            a.p5v[((size_t)r * a.nparts + blockIdx.x) * 5 + k] = v[k];
            a.p5i[((size_t)r * a.nparts + blockIdx.x) * 5 + k] = ix[k];
        }
    }
}

// the five best over a warp's lanes, each lane holding its own five best in order: five rounds of the warp's best head,
// popped from the lane that holds it
B2_DEV void fr_merge5(int64_t* v, int* ix) {
    int64_t ov[5];
    int oi[5];
#pragma unroll
    for (int k = 0; k < 5; k++) {
        int64_t bv = v[0];
        int bi = ix[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int64_t cv = __shfl_xor_sync(0xffffffffu, bv, o);
            const int ci = __shfl_xor_sync(0xffffffffu, bi, o);
            if (fr_better(cv, ci, bv, bi)) { bv = cv; bi = ci; }
        }
        if (v[0] == bv && ix[0] == bi) {
#pragma unroll
            for (int q = 0; q < 4; q++) { v[q] = v[q + 1]; ix[q] = ix[q + 1]; }
            v[4] = INT64_MIN;
            ix[4] = 0x7fffffff;
        }
        ov[k] = bv;
        oi[k] = bi;
    }
#pragma unroll
    for (int k = 0; k < 5; k++) { v[k] = ov[k]; ix[k] = oi[k]; }
}

// T5 (the 5th-best low of the row) and the words still in (high >= T5): one CTA per row
__global__ void __launch_bounds__(1024) k_top_select(TopFrArgs a) {
    griddep_wait();
    griddep_launch();
    __shared__ int64_t s5v[32][5];
    __shared__ int s5i[32][5];
    __shared__ int64_t s_t5;
    __shared__ int s_cnt;
    const int r = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int64_t v[5];
    int ix[5];
#pragma unroll
    for (int k = 0; k < 5; k++) { v[k] = INT64_MIN; ix[k] = 0x7fffffff; }
    for (int t = threadIdx.x; t < a.nparts; t += blockDim.x)
#pragma unroll
        for (int k = 0; k < 5; k++) fr_put5(v, ix, a.p5v[((size_t)r * a.nparts + t) * 5 + k], a.p5i[((size_t)r * a.nparts + t) * 5 + k]);
    fr_merge5(v, ix);
    if (lane == 0)
#pragma unroll
        for (int k = 0; k < 5; k++) { s5v[wid][k] = v[k]; s5i[wid][k] = ix[k]; }
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    if (wid == 0) {
#pragma unroll
        for (int k = 0; k < 5; k++) { v[k] = s5v[lane][k]; ix[k] = s5i[lane][k]; }
        fr_merge5(v, ix);
        if (lane == 0) s_t5 = v[4];
    }
    __syncthreads();
    const int64_t t5 = s_t5;
    for (int j0 = 0; j0 < a.nout; j0 += blockDim.x) {
        const int j = j0 + threadIdx.x;
        const bool keep = j < a.nout && a.HIS[(size_t)r * a.nout + j] >= t5;
        const uint32_t m = __ballot_sync(0xffffffffu, keep);
        int base = 0;
        if (lane == 0 && m) base = atomicAdd(&s_cnt, __popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (keep) a.list[(size_t)r * a.nout + base + __popc(m & ((1u << lane) - 1))] = j;
    }
    __syncthreads();
    if (threadIdx.x == 0) a.cnt[r] = s_cnt;
}

// (d): the words still in, exactly: pile = 256 C + sum wl x + 128 S1 (lo = wl + 128), the head's own score, and each
// CTA's best (score, word) per row (k_race_parts then picks the row's word). A warp per word still in.
template <int EPI>
__global__ void __launch_bounds__(256) k_top_finish(TopFrArgs a) {
    griddep_wait();
    griddep_launch();
    __shared__ int64_t sv[8];
    __shared__ int si[8];
    const int r = blockIdx.y, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x[24];
    int64_t S1, SP, SN;
    fr_row(a, r, lane, x, S1, SP, SN);
    const int n = a.cnt[r];
    int64_t best = INT64_MIN;
    int bw = 0x7fffffff;
    for (int k = blockIdx.x * 8 + wid; k < n; k += gridDim.x * 8) {
        const int j = a.list[(size_t)r * a.nout + k];
        const int64_t l = fr_dot(a.wl + (size_t)j * TOPFR_NIN, x, lane);
        const int64_t s = fr_score<EPI>(wadd(wadd(wmul(256, a.C[(size_t)r * a.nout + j]), l), wmul(128, S1)), j, r, a);
        if (fr_better(s, j, best, bw)) { best = s; bw = j; }
    }
    if (lane == 0) { sv[wid] = best; si[wid] = bw; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++) if (fr_better(sv[w], si[w], best, bw)) { best = sv[w]; bw = si[w]; }
        a.sv[(size_t)r * a.nfin + blockIdx.x] = best;
        a.si[(size_t)r * a.nfin + blockIdx.x] = bw;
    }
}

}  // namespace b2
