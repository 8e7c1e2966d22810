/*
 * base2_oracle.c -- TEST INFRASTRUCTURE ONLY. A plain-C restatement of the reference's CPU machine `base2.py`
 * (the integer-only GPT-2), used as the parity checker for the CUDA engine and as the timed CPU baseline.
 * Nothing in the product links or calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU legs do.
 *
 * Every function states the reference lines it follows. Arithmetic is numpy int64 arithmetic exactly as base2.py
 * gets it:
 *   - +, -, * wrap modulo 2^64 (numpy int64 array ops do; hazard: power()'s X*EXP2 does wrap at long contexts);
 *   - np.left_shift by >= 64 gives 0, np.right_shift by >= 64 gives the sign fill (numpy's defined shifts);
 *   - products (base2.py:29-32) are float64 matmuls asserted below 2^52, hence exact; here they are exact int64
 *     sums, which give the same integers whenever base2.py's own assert holds.
 * Signed overflow is undefined in C, so every wrapping operation goes through uint64_t.
 * The float stage switches (gauge=/edge=/arrival=/turn= float) are float64 in the reference's own operation order,
 * each multiply and add rounded on its own (built with -ffp-contract=off), means and sums in numpy's pairwise order.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef int64_t i64;
typedef uint64_t u64;

static inline i64 wadd(i64 a, i64 b) { return (i64)((u64)a + (u64)b); }
static inline i64 wsub(i64 a, i64 b) { return (i64)((u64)a - (u64)b); }
static inline i64 wmul(i64 a, i64 b) { return (i64)((u64)a * (u64)b); }
static inline i64 np_lsh(i64 x, i64 s) { return (s < 0 || s >= 64) ? 0 : (i64)((u64)x << s); }
static inline i64 np_rsh(i64 x, i64 s) { return s >= 64 ? (x < 0 ? -1 : 0) : (s < 0 ? 0 : (x >> s)); }

/* base2.py:18-22 rshift: X x 2^-s rounded to nearest (add half, arithmetic shift); s <= 0 shifts left. */
static inline i64 rshift1(i64 x, i64 s) {
    i64 up = np_lsh(x, s < 0 ? -s : 0);
    i64 sp = s > 0 ? s : 0;
    i64 half = sp > 0 ? np_lsh(1, sp - 1) : 0;
    return np_rsh(wadd(up, half), sp);
}

/* Python int.bit_length() of an int64 value (of its magnitude; 64 for INT64_MIN). */
static inline int bitlen(i64 v) {
    u64 m = v < 0 ? (u64)0 - (u64)v : (u64)v;
    return m ? 64 - __builtin_clzll(m) : 0;
}

/* base2.py:42-48 log2fix: top 1's position t, the next 16 digits m, t*65536 + LOG2[m]. */
static inline i64 log2fix1(i64 v, const i64 *LOG2) {
    int t = bitlen(v) - 1;
    i64 m = t >= 16 ? ((v >> (t - 16)) & 0xFFFF) : (np_lsh(v, 16 - t) & 0xFFFF);
    return (i64)t * 65536 + LOG2[m];
}

/* base2.py:50-53 power: X x 2^(F/65536) = rshift(X * EXP2[F & 0xFFFF], 16 - (F >> 16)), the product wrapping. */
static inline i64 power1(i64 x, i64 F, const i64 *EXP2) {
    i64 I = F >> 16, f = F & 0xFFFF;
    return rshift1(wmul(x, EXP2[f]), 16 - I);
}

/* base2.py:24-27 to16 for one row: sh = max(bit_length(OR |x|) - 15, 0); x16 = rshift(x, sh). Returns sh. */
static int to16_row(const i64 *x, int n, i64 *x16) {
    u64 o = 0;
    for (int i = 0; i < n; i++) o |= (u64)(x[i] < 0 ? wsub(0, x[i]) : x[i]);
    int top = bitlen((i64)o);
    int sh = top - 15 > 0 ? top - 15 : 0;
    for (int i = 0; i < n; i++) x16[i] = rshift1(x[i], sh);
    return sh;
}

/* base2.py:78-83 edge: idx = rshift(h, 4) + 32768 picks the share (0 below, 65536 above); rshift(h * share, 16). */
static inline i64 edge1(i64 h, const i64 *PHI) {
    i64 idx = wadd(rshift1(h, 16 - 12), 32768);
    i64 share = idx < 0 ? 0 : (idx > 65535 ? 65536 : PHI[idx]);
    return rshift1(wmul(h, share), 16);
}

/* base2.py:34-40 race: the largest value; among equal largest, the lowest index. */
static i64 race1(const i64 *v, i64 n) {
    i64 best = 0;
    for (i64 i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* element-wise entry points (the pinning tests call these against base2.py's own outputs)                       */
/* ------------------------------------------------------------------------------------------------------------ */
void b2o_rshift(const i64 *x, const i64 *s, i64 n, i64 *y) { for (i64 i = 0; i < n; i++) y[i] = rshift1(x[i], s[i]); }
void b2o_log2fix(const i64 *v, i64 n, const i64 *LOG2, i64 *y) { for (i64 i = 0; i < n; i++) y[i] = log2fix1(v[i], LOG2); }
void b2o_power(const i64 *x, const i64 *F, i64 n, const i64 *EXP2, i64 *y) { for (i64 i = 0; i < n; i++) y[i] = power1(x[i], F[i], EXP2); }
void b2o_edge(const i64 *h, i64 n, const i64 *PHI, i64 *y) { for (i64 i = 0; i < n; i++) y[i] = edge1(h[i], PHI); }
i64 b2o_race(const i64 *v, i64 n) { return race1(v, n); }
void b2o_to16(const i64 *X, i64 rows, i64 n, i64 e0, i64 *x16, i64 *ex) {
    for (i64 r = 0; r < rows; r++) ex[r] = e0 + to16_row(X + r * n, (int)n, x16 + r * n);
}

/* base2.py:55-60 gauge_log for one row of 768: x16, ex, LS = (log2fix(V) >> 1) - LOG768 + ex*65536,
 * V = 768*S2 - S1^2 + (EPS40 >> (40 + 2 ex)). n is the row length; the 768 is the reference's constant. */
static i64 gauge_row(const i64 *x, int n, i64 *x16, i64 *ex_out, const i64 *LOG2, i64 log768, i64 eps40) {
    i64 ex = -16 + to16_row(x, n, x16);
    i64 S1 = 0, S2 = 0;
    for (int i = 0; i < n; i++) { S1 = wadd(S1, x16[i]); S2 = wadd(S2, wmul(x16[i], x16[i])); }
    i64 V = wsub(wmul(768, S2), wmul(S1, S1));
    i64 sh = 40 + 2 * ex;
    V = wadd(V, sh >= 0 ? np_rsh(eps40, sh) : np_lsh(eps40, -sh));
    *ex_out = ex;
    return wadd(wsub(log2fix1(V, LOG2) >> 1, log768), wmul(ex, 65536));
}
void b2o_gauge_log(const i64 *R, i64 rows, i64 n, const i64 *LOG2, i64 log768, i64 eps40, i64 *x16, i64 *ex, i64 *LS) {
    for (i64 r = 0; r < rows; r++) LS[r] = gauge_row(R + r * n, (int)n, x16 + r * n, ex + r, LOG2, log768, eps40);
}

/* ------------------------------------------------------------------------------------------------------------ */
/* float stage switches: shared pieces                                                                            */
/* ------------------------------------------------------------------------------------------------------------ */
enum { F_GAUGE = 1, F_EDGE = 2, F_ARRIVAL = 4, F_TURN = 8 };
typedef __int128 i128;

/* numpy's pairwise sum, the order np.add.reduce / np.mean use along a contiguous axis (numpy's pairwise_sum):
 * fewer than 8 terms in order; up to 128 in eight interleaved partial sums folded ((0+1)+(2+3))+((4+5)+(6+7)) and
 * then the remainder in order; more: split at half the count rounded down to a multiple of 8. */
double b2f_pairwise(const double *a, i64 n) {
    if (n < 8) {
        double r = 0.0;
        for (i64 i = 0; i < n; i++) r += a[i];
        return r;
    }
    if (n <= 128) {
        double r[8];
        for (int j = 0; j < 8; j++) r[j] = a[j];
        i64 i = 8;
        for (; i < n - (n % 8); i += 8)
            for (int j = 0; j < 8; j++) r[j] += a[i + j];
        double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; i++) res += a[i];
        return res;
    }
    i64 n2 = n / 2;
    n2 -= n2 % 8;
    return b2f_pairwise(a, n2) + b2f_pairwise(a + n2, n - n2);
}

/* the row at 2^-16, its mean and sqrt(mean((x - mean)^2) + 1e-5) (base2.py:67, pythia_base2.py:103). x, t: n
 * doubles of scratch; on return x holds x - mean. */
static double row_sigma(const i64 *R, int n, double *x, double *t) {
    for (int i = 0; i < n; i++) x[i] = (double)R[i] / 65536.0;
    const double mu = b2f_pairwise(x, n) / (double)n;
    for (int i = 0; i < n; i++) { x[i] = x[i] - mu; t[i] = x[i] * x[i]; }
    return sqrt(b2f_pairwise(t, n) / (double)n + 1e-5);
}

/* an exact 128-bit dot product as the nearest double (ties to even) */
double b2f_i128_to_double(i128 x) {
    if (x >= (i128)INT64_MIN && x <= (i128)INT64_MAX) return (double)(i64)x;
    const int neg = x < 0;
    unsigned __int128 u = neg ? (unsigned __int128)0 - (unsigned __int128)x : (unsigned __int128)x;
    int top = 127;
    while (!((u >> top) & 1)) top--;
    const int sh = top - 62;                                 /* keep 63 bits */
    u64 keep = (u64)(u >> sh);
    const int sticky = (u & (((unsigned __int128)1 << sh) - 1)) != 0;
    u64 mant = keep >> 10, rem = keep & 1023;                /* 53 bits + 10 to round away */
    if (rem > 512 || (rem == 512 && (sticky || (mant & 1)))) mant++;
    const double r = ldexp((double)mant, sh + 10);
    return neg ? -r : r;
}

/* base2.py:79-80, edge=float: 0.5 h (1 + tanh(0.7978845608028654 (h + 0.044715 h^3))) at 2^-16, rounded */
static i64 edge_tanh1(i64 H) {
    const double h = (double)H / 65536.0;
    const double t = 0.7978845608028654 * (h + 0.044715 * pow(h, 3.0));
    return (i64)rint(0.5 * h * (1.0 + tanh(t)) * 65536.0);
}
/* pythia_base2.py:144-146, edge=float: h 0.5 (1 + erf(h / sqrt 2)) at 2^-16, rounded */
static i64 edge_erf1(i64 H) {
    const double h = (double)H / 65536.0;
    return (i64)rint(h * 0.5 * (1.0 + erf(h / 1.4142135623730951)) * 65536.0);
}
void b2f_edge(const i64 *h, i64 n, int erf_form, i64 *y) {
    for (i64 i = 0; i < n; i++) y[i] = erf_form ? edge_erf1(h[i]) : edge_tanh1(h[i]);
}

/* base2.py:89-92 / pythia_base2.py:130-133, arrival=float, for the last row of a causal run over positions 0..p:
 * s = (q / 2^16).(k / 2^16) / 8 (the dot exact, then rounded once), a = exp(s - max s) / (its pairwise sum),
 * out = round(sum_s a_s (v_s / 2^16) * 2^16) with the sum over s in order. q, K rows (stride ldk), V rows (stride
 * ldv) at full width; e: p+1 doubles of scratch. */
static void arrival_float_row(const i64 *q, const i64 *K, size_t ldk, const i64 *V, size_t ldv, int p, int hd,
                              i64 *out, double *e) {
    double mx = -INFINITY;
    for (int s = 0; s <= p; s++) {
        i128 dot = 0;
        for (int t = 0; t < hd; t++) dot += (i128)q[t] * (i128)K[(size_t)s * ldk + t];
        e[s] = ldexp(b2f_i128_to_double(dot), -32) / 8.0;
        if (e[s] > mx) mx = e[s];
    }
    for (int s = 0; s <= p; s++) e[s] = exp(e[s] - mx);
    const double Z = b2f_pairwise(e, p + 1);
    for (int s = 0; s <= p; s++) e[s] = e[s] / Z;
    for (int t = 0; t < hd; t++) {
        double acc = 0.0;
        for (int s = 0; s <= p; s++) acc = acc + e[s] * ((double)V[(size_t)s * ldv + t] / 65536.0);
        out[t] = (i64)rint(acc * 65536.0);
    }
}

/* ------------------------------------------------------------------------------------------------------------ */
/* the model                                                                                                     */
/* ------------------------------------------------------------------------------------------------------------ */
typedef struct {
    const int16_t *w;     /* [nin][nout] (reference layout, base2_gpu.py:11) */
    const i64 *e, *b;     /* [nout] */
    int nin, nout;
} bank_t;

typedef struct {
    int L, d, H, hd, F, V, ctx;
    bank_t bank[64 * 4 + 1];  /* layer*4 + {qkv, proj, fc, mproj}; head at 4*L */
    const i64 *wte, *wpe, *PHI, *ARR, *LOG2, *EXP2;
    i64 alen, log768, eps40;
    int flags;                /* F_GAUGE | F_EDGE | F_ARRIVAL: stages back to float64 (base2.py:10-11) */
} model_t;

void *b2o_create(int L, int d, int H, int F, int V, int ctx) {
    model_t *m = (model_t *)calloc(1, sizeof(model_t));
    m->L = L; m->d = d; m->H = H; m->hd = d / H; m->F = F; m->V = V; m->ctx = ctx;
    return m;
}
void b2o_destroy(void *m) { free(m); }
void b2o_set_flags(void *mv, int flags) { ((model_t *)mv)->flags = flags; }
void b2o_set_bank(void *mv, int idx, const int16_t *w, const i64 *e, const i64 *b, int nin, int nout) {
    model_t *m = (model_t *)mv;
    m->bank[idx].w = w; m->bank[idx].e = e; m->bank[idx].b = b; m->bank[idx].nin = nin; m->bank[idx].nout = nout;
}
void b2o_set_tables(void *mv, const i64 *wte, const i64 *wpe, const i64 *PHI, const i64 *ARR, i64 alen,
                    const i64 *LOG2, const i64 *EXP2, i64 log768, i64 eps40) {
    model_t *m = (model_t *)mv;
    m->wte = wte; m->wpe = wpe; m->PHI = PHI; m->ARR = ARR; m->alen = alen; m->LOG2 = LOG2; m->EXP2 = EXP2;
    m->log768 = log768; m->eps40 = eps40;
}

/* base2.py:29-32 product for one row: pile[j] = sum_i x16[i] * w[i][j], exact. Columns split over threads when
 * `par` is set (single-stream runs); a multi-stream run parallelises over streams instead. */
static void product_row(const i64 *x16, const bank_t *bk, i64 *pile, int par) {
    const int nin = bk->nin, nout = bk->nout;
    const int CH = 1024;
    int nch = (nout + CH - 1) / CH;
#pragma omp parallel for schedule(static) if (par)
    for (int c = 0; c < nch; c++) {
        int j0 = c * CH, j1 = j0 + CH < nout ? j0 + CH : nout;
        i64 acc[1024];
        for (int j = 0; j < j1 - j0; j++) acc[j] = 0;
        for (int i = 0; i < nin; i++) {
            i64 xi = x16[i];
            if (!xi) continue;
            const int16_t *wr = bk->w + (size_t)i * nout + j0;
            for (int j = 0; j < j1 - j0; j++) acc[j] += xi * (i64)wr[j];
        }
        for (int j = 0; j < j1 - j0; j++) pile[j0 + j] = acc[j];
    }
}

/* base2.py:62-71 gauged_bank for one row; with gauge=float base2.py:66-69 (layer banks) or :110-113 (head: the
 * bias at 2^-16 added before the rounding). */
static void gauged_row_h(const model_t *m, const bank_t *bk, const i64 *R, i64 *out, i64 *x16, i64 *pile, int par,
                         int head) {
    i64 ex;
    i64 LS = gauge_row(R, m->d, x16, &ex, m->LOG2, m->log768, m->eps40);
    product_row(x16, bk, pile, par);
    if (m->flags & F_GAUGE) {
        double *x = (double *)malloc(sizeof(double) * 2 * m->d);
        const double sig = row_sigma(R, m->d, x, x + m->d);
        free(x);
        for (int j = 0; j < bk->nout; j++) {
            const double val = (double)pile[j] * ldexp(1.0, (int)(bk->e[j] + ex)) / sig;
            out[j] = head ? (i64)rint((val + (double)bk->b[j] / 65536.0) * 65536.0)
                          : wadd((i64)rint(val * 65536.0), bk->b[j]);
        }
        return;
    }
    for (int j = 0; j < bk->nout; j++) {
        i64 F = wsub(wmul(wadd(wadd(bk->e[j], ex), 16), 65536), LS);
        out[j] = wadd(power1(pile[j], F, m->EXP2), bk->b[j]);
    }
}
static void gauged_row(const model_t *m, const bank_t *bk, const i64 *R, i64 *out, i64 *x16, i64 *pile, int par) {
    gauged_row_h(m, bk, R, out, x16, pile, par, 0);
}

/* base2.py:73-76 plain_bank for one row, added into R (base2.py:105-106 R = R + plain_bank(...)). */
static void plain_row_add(const model_t *m, const bank_t *bk, const i64 *X, i64 *R, i64 *x16, i64 *pile, int par) {
    i64 ex = -16 + to16_row(X, bk->nin, x16);
    product_row(x16, bk, pile, par);
    for (int j = 0; j < bk->nout; j++)
        R[j] = wadd(R[j], wadd(rshift1(pile[j], -wadd(wadd(bk->e[j], ex), 16)), bk->b[j]));
}

void b2o_gauged_bank(void *mv, int idx, const i64 *R, int rows, i64 *out) {
    model_t *m = (model_t *)mv; const bank_t *bk = &m->bank[idx];
    i64 *x16 = (i64 *)malloc(sizeof(i64) * bk->nin), *pile = (i64 *)malloc(sizeof(i64) * bk->nout);
    for (int r = 0; r < rows; r++) gauged_row(m, bk, R + (size_t)r * bk->nin, out + (size_t)r * bk->nout, x16, pile, 1);
    free(x16); free(pile);
}
void b2o_plain_bank(void *mv, int idx, const i64 *X, int rows, i64 *out) {
    model_t *m = (model_t *)mv; const bank_t *bk = &m->bank[idx];
    i64 *x16 = (i64 *)malloc(sizeof(i64) * bk->nin), *pile = (i64 *)malloc(sizeof(i64) * bk->nout);
    for (int r = 0; r < rows; r++) {
        i64 *o = out + (size_t)r * bk->nout;
        memset(o, 0, sizeof(i64) * bk->nout);
        plain_row_add(m, bk, X + (size_t)r * bk->nin, o, x16, pile, 1);
    }
    free(x16); free(pile);
}

/* the per-stream key/value store: what attention at a later position reads of an earlier one */
typedef struct {
    i64 *k16;   /* [L][ctx][d]   to16'd keys per head part */
    i64 *ek;    /* [L][ctx][H]   their exponents */
    i64 *v;     /* [L][ctx][d]   values at full width (base2.py:98 reads v[:p+1] unshifted) */
    i64 *kraw;  /* [L][ctx][d]   keys at full width (arrival=float only; NULL otherwise) */
} cache_t;

static int cache_alloc(const model_t *m, cache_t *c, int ctx) {
    size_t n = (size_t)m->L * ctx;
    c->k16 = (i64 *)malloc(sizeof(i64) * n * m->d);
    c->ek = (i64 *)malloc(sizeof(i64) * n * m->H);
    c->v = (i64 *)malloc(sizeof(i64) * n * m->d);
    c->kraw = (m->flags & F_ARRIVAL) ? (i64 *)malloc(sizeof(i64) * n * m->d) : NULL;
    return c->k16 && c->ek && c->v && (c->kraw || !(m->flags & F_ARRIVAL));
}
static void cache_free(cache_t *c) { free(c->k16); free(c->ek); free(c->v); free(c->kraw); }

/* base2.py:85-100 attention, integer arrival, for the position p of one stream given the keys/values of 0..p.
 * q: this position's 768 query values (int64). Writes 768 outputs. sc: scratch of >= p+1. */
static void attend_row(const model_t *m, const cache_t *c, int l, int ctx, int p, const i64 *q, i64 *out, i64 *sc) {
    const int d = m->d, hd = m->hd;
    if (m->flags & F_ARRIVAL) {      /* base2.py:89-92 */
        double *e = (double *)sc;    /* sc holds >= p+1 i64, the same size */
        for (int h = 0; h < m->H; h++)
            arrival_float_row(q + h * hd, c->kraw + ((size_t)l * ctx) * d + h * hd, d,
                              c->v + ((size_t)l * ctx) * d + h * hd, d, p, hd, out + h * hd, e);
        return;
    }
    i64 q16[256];
    for (int h = 0; h < m->H; h++) {
        i64 eq = -16 + to16_row(q + h * hd, hd, q16);
        const i64 *K = c->k16 + ((size_t)l * ctx) * d + h * hd;
        const i64 *EK = c->ek + ((size_t)l * ctx) * m->H + h;
        const i64 *Vv = c->v + ((size_t)l * ctx) * d + h * hd;
        for (int s = 0; s <= p; s++) {
            i64 dot = 0;
            const i64 *k = K + (size_t)s * d;
            for (int t = 0; t < hd; t++) dot += q16[t] * k[t];
            sc[s] = rshift1(dot, -(eq + EK[(size_t)s * m->H] - 3 + 10));
        }
        i64 start = sc[race1(sc, p + 1)];
        i64 Z = 0, num[256];
        for (int t = 0; t < hd; t++) num[t] = 0;
        for (int s = 0; s <= p; s++) {
            i64 dd = wsub(start, sc[s]);
            /* numpy: ARR[min(d, len-1)] where d < len; a negative d indexes from the end (d >= -len) */
            i64 a = dd >= m->alen ? 0 : (dd >= 0 ? m->ARR[dd] : (dd >= -m->alen ? m->ARR[m->alen + dd] : 0));
            if (!a) continue;
            Z = wadd(Z, a);
            const i64 *v = Vv + (size_t)s * d;
            for (int t = 0; t < hd; t++) num[t] = wadd(num[t], wmul(a, v[t]));
        }
        i64 F = -log2fix1(Z, m->LOG2);
        for (int t = 0; t < hd; t++) out[h * hd + t] = power1(num[t], F, m->EXP2);
    }
}

typedef struct { i64 *R, *qkv, *att, *hid, *x16, *pile, *sc; } scratch_t;

static int scratch_alloc(const model_t *m, scratch_t *s, int ctx) {
    int wmax = m->V > m->F ? m->V : m->F;
    s->R = (i64 *)malloc(sizeof(i64) * m->d);
    s->qkv = (i64 *)malloc(sizeof(i64) * 3 * m->d);
    s->att = (i64 *)malloc(sizeof(i64) * m->d);
    s->hid = (i64 *)malloc(sizeof(i64) * m->F);
    s->x16 = (i64 *)malloc(sizeof(i64) * (m->F > m->d ? m->F : m->d));
    s->pile = (i64 *)malloc(sizeof(i64) * wmax);
    s->sc = (i64 *)malloc(sizeof(i64) * ctx);
    return s->R && s->qkv && s->att && s->hid && s->x16 && s->pile && s->sc;
}
static void scratch_free(scratch_t *s) { free(s->R); free(s->qkv); free(s->att); free(s->hid); free(s->x16); free(s->pile); free(s->sc); }

/* One new position p of one stream through the 12 layers (base2.py:103-106), keys/values appended to the cache;
 * if `logits` is given, the head's scores for this position (base2.py:107-114). Returns the race's word or -1. */
static int position(const model_t *m, cache_t *c, scratch_t *s, int ctx, int p, int id, i64 *logits, int par) {
    const int d = m->d, H = m->H, hd = m->hd;
    for (int i = 0; i < d; i++) s->R[i] = wadd(m->wte[(size_t)id * d + i], m->wpe[(size_t)p * d + i]);
    for (int l = 0; l < m->L; l++) {
        gauged_row(m, &m->bank[4 * l + 0], s->R, s->qkv, s->x16, s->pile, par);
        for (int h = 0; h < H; h++) {
            i64 *k16 = c->k16 + ((size_t)l * ctx + p) * d + h * hd;
            c->ek[((size_t)l * ctx + p) * H + h] = -16 + to16_row(s->qkv + d + h * hd, hd, k16);
        }
        memcpy(c->v + ((size_t)l * ctx + p) * d, s->qkv + 2 * d, sizeof(i64) * d);
        if (c->kraw) memcpy(c->kraw + ((size_t)l * ctx + p) * d, s->qkv + d, sizeof(i64) * d);
        attend_row(m, c, l, ctx, p, s->qkv, s->att, s->sc);
        plain_row_add(m, &m->bank[4 * l + 1], s->att, s->R, s->x16, s->pile, par);
        gauged_row(m, &m->bank[4 * l + 2], s->R, s->hid, s->x16, s->pile, par);
        for (int j = 0; j < m->F; j++) s->hid[j] = (m->flags & F_EDGE) ? edge_tanh1(s->hid[j]) : edge1(s->hid[j], m->PHI);
        plain_row_add(m, &m->bank[4 * l + 3], s->hid, s->R, s->x16, s->pile, par);
    }
    if (!logits) return -1;
    gauged_row_h(m, &m->bank[4 * m->L], s->R, logits, s->x16, s->pile, par, 1);
    return (int)race1(logits, m->V);
}

static int nthreads(int want) {
#ifdef _OPENMP
    if (want > 0) return want;
    return omp_get_max_threads();
#else
    (void)want; return 1;
#endif
}

/* A 64-bit digest of one row of scores: the sum over v of logit[v] * key(v) modulo 2^64, key(v) = splitmix64(v) | 1
 * (the SplitMix64 finaliser of Steele, Lea and Flood, 2014). Odd keys make any single differing score change the
 * digest. Lets a parity test compare every generated position of every stream without storing the scores. */
static inline u64 hkey(u64 v) {
    u64 z = v + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return (z ^ (z >> 31)) | 1ull;
}
u64 b2o_logit_hash(const i64 *lg, i64 V) {
    u64 h = 0;
    for (i64 v = 0; v < V; v++) h += (u64)lg[v] * hkey((u64)v);
    return h;
}

/* Greedy generation for B independent streams of equal prompt length P (base2.py:122-123: each new word is the
 * race at the last position, fed back in). tokens: [B][n_new]; logits (optional): [B][n_new][V], the scores each
 * token was raced on; hashes (optional): [B][n_new], their digests (b2o_logit_hash). Streams run in parallel over
 * threads; a single stream splits each bank over threads. Returns 0, or -1 when memory is short or a position
 * passes the context. */
static int gen_core(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, i64 *logits, u64 *hashes,
                    int threads) {
    const model_t *m = (const model_t *)mv;
    int ctx = P + n_new;
    if (ctx > m->ctx || P < 1) return -1;
    int nt = nthreads(threads), err = 0;
    int par = B == 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (B > 1)
    for (int b = 0; b < B; b++) {
        cache_t c; scratch_t s;
        i64 *lg = (i64 *)malloc(sizeof(i64) * m->V);
        if (!cache_alloc(m, &c, ctx) || !scratch_alloc(m, &s, ctx) || !lg) { err = -1; continue; }
        for (int p = 0; p < P - 1; p++) position(m, &c, &s, ctx, p, ids[(size_t)b * P + p], NULL, par);
        int tok = ids[(size_t)b * P + P - 1];
        for (int t = 0; t < n_new; t++) {
            tok = position(m, &c, &s, ctx, P - 1 + t, tok, lg, par);
            tokens[(size_t)b * n_new + t] = tok;
            if (logits) memcpy(logits + ((size_t)b * n_new + t) * m->V, lg, sizeof(i64) * m->V);
            if (hashes) hashes[(size_t)b * n_new + t] = b2o_logit_hash(lg, m->V);
        }
        cache_free(&c); scratch_free(&s); free(lg);
    }
    return err;
}
int b2o_generate(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, i64 *logits, int threads) {
    return gen_core(mv, ids, B, P, n_new, tokens, logits, NULL, threads);
}
int b2o_generate_digest(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, u64 *hashes,
                        int threads) {
    return gen_core(mv, ids, B, P, n_new, tokens, NULL, hashes, threads);
}

/* Teacher-forced scores (the judge5.py:15-23 pattern): one stream's P ids, the head's scores at positions
 * [first, last). logits: [(last-first)][V]. */
int b2o_scores(void *mv, const int32_t *ids, int P, int first, int last, i64 *logits) {
    const model_t *m = (const model_t *)mv;
    if (P > m->ctx || first < 0 || last > P || first >= last) return -1;
    cache_t c; scratch_t s;
    if (!cache_alloc(m, &c, P) || !scratch_alloc(m, &s, P)) return -1;
    for (int p = 0; p < P; p++)
        position(m, &c, &s, P, p, ids[p], (p >= first && p < last) ? logits + (size_t)(p - first) * m->V : NULL, 1);
    cache_free(&c); scratch_free(&s);
    return 0;
}

/* base2.py:122-124 exactly as the reference runs it: every new word recomputes the whole prefix from scratch
 * (no key/value store kept between words). One stream; used only as the timed CPU baseline. */
int b2o_greedy_recompute(void *mv, const int32_t *ids, int P, int n_new, int32_t *tokens, int threads) {
    const model_t *m = (const model_t *)mv;
    int ctx = P + n_new;
    if (ctx > m->ctx) return -1;
    (void)threads;
    int32_t *seq = (int32_t *)malloc(sizeof(int32_t) * ctx);
    i64 *lg = (i64 *)malloc(sizeof(i64) * m->V);
    memcpy(seq, ids, sizeof(int32_t) * P);
    int n = P;
    for (int t = 0; t < n_new; t++) {
        cache_t c; scratch_t s;
        if (!cache_alloc(m, &c, n) || !scratch_alloc(m, &s, n)) return -1;
        int tok = -1;
        for (int p = 0; p < n; p++) tok = position(m, &c, &s, n, p, seq[p], p == n - 1 ? lg : NULL, 1);
        cache_free(&c); scratch_free(&s);
        tokens[t] = tok;
        seq[n++] = tok;
    }
    free(seq); free(lg);
    return 0;
}

/* b2o_greedy_recompute over B streams of equal prompt length, streams in parallel over threads (each stream as
 * base2.py runs it: the whole prefix recomputed for every new word). tokens [B][n_new]. */
int b2o_generate_recompute(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, int threads) {
    const model_t *m = (const model_t *)mv;
    if (P + n_new > m->ctx) return -1;
    int nt = nthreads(threads), err = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int b = 0; b < B; b++) {
        int ctx = P + n_new;
        int32_t *seq = (int32_t *)malloc(sizeof(int32_t) * ctx);
        i64 *lg = (i64 *)malloc(sizeof(i64) * m->V);
        memcpy(seq, ids + (size_t)b * P, sizeof(int32_t) * P);
        int n = P;
        for (int t = 0; t < n_new && !err; t++) {
            cache_t c; scratch_t s;
            if (!cache_alloc(m, &c, n) || !scratch_alloc(m, &s, n)) { err = -1; break; }
            int tok = -1;
            for (int p = 0; p < n; p++) tok = position(m, &c, &s, n, p, seq[p], p == n - 1 ? lg : NULL, 0);
            cache_free(&c); scratch_free(&s);
            tokens[(size_t)b * n_new + t] = tok;
            seq[n++] = tok;
        }
        free(seq); free(lg);
    }
    return err;
}

/* base2.py:85-100 over a whole sequence's QKV [P][3d] (the reference's own attention() shape): out [P][d]. */
int b2o_attention(void *mv, const i64 *QKV, int P, i64 *out) {
    const model_t *m = (const model_t *)mv;
    const int d = m->d, H = m->H, hd = m->hd;
    model_t one = *m; one.L = 1;
    cache_t c; i64 *sc = (i64 *)malloc(sizeof(i64) * P);
    if (!cache_alloc(&one, &c, P) || !sc) return -1;
    for (int p = 0; p < P; p++) {
        for (int h = 0; h < H; h++)
            c.ek[(size_t)p * H + h] = -16 + to16_row(QKV + (size_t)p * 3 * d + d + h * hd, hd, c.k16 + (size_t)p * d + h * hd);
        memcpy(c.v + (size_t)p * d, QKV + (size_t)p * 3 * d + 2 * d, sizeof(i64) * d);
        if (c.kraw) memcpy(c.kraw + (size_t)p * d, QKV + (size_t)p * 3 * d + d, sizeof(i64) * d);
    }
    for (int p = 0; p < P; p++) attend_row(&one, &c, 0, P, p, QKV + (size_t)p * 3 * d, out + (size_t)p * d, sc);
    cache_free(&c); free(sc);
    return 0;
}

/* ============================================================================================================ */
/* Pythia-160M: the reference's foundation0/pythia_base2.py (size=160m, plates=finished, order=plain)           */
/* ============================================================================================================ */

/* pythia_base2.py:87-90 power for one element, exactly (Python big ints): X*EXP2[f] then the rounded shift by
 * 16 - I. Returns -1 when the result leaves int64 (where the reference's .astype(np.int64) raises). */
static int power_exact1(i64 x, i64 F, const i64 *EXP2, i64 *out) {
    i64 I = F >> 16, f = F & 0xFFFF, s = 16 - I;
    i128 p = (i128)x * (i128)EXP2[f], r;
    if (s <= 0) {
        if (p == 0) r = 0;
        else if (-s >= 64) return -1;
        else {
            r = p << (-s);
            if ((r >> (-s)) != p) return -1;
        }
    } else if (s >= 100) {
        r = 0;                                /* |p| < 2^81: (p + 2^(s-1)) >> s is 0 */
    } else {
        r = (p + ((i128)1 << (s - 1))) >> s;  /* floor shift, as Python's >> */
    }
    if (r > (i128)INT64_MAX || r < (i128)INT64_MIN) return -1;
    *out = (i64)r;
    return 0;
}

/* pythia_base2.py:87-90 over an array: the int64 path when every |X| < 2^45, else the exact path. Returns -1 on an
 * exact result outside int64. */
int b2p_power(const i64 *x, const i64 *F, i64 n, const i64 *EXP2, i64 *y) {
    int big = 0;
    for (i64 i = 0; i < n; i++) if ((x[i] < 0 ? (u64)0 - (u64)x[i] : (u64)x[i]) >= ((u64)1 << 45)) big = 1;
    for (i64 i = 0; i < n; i++) {
        if (!big) y[i] = power1(x[i], F[i], EXP2);
        else if (power_exact1(x[i], F[i], EXP2, &y[i])) return -1;
    }
    return 0;
}

typedef struct {
    int L, d, H, hd, F, V, ctx, rot;
    bank_t bank[64 * 4 + 1];                   /* layer*4 + {qkv, proj, fc, mproj}; head at 4*L (bias zeros) */
    const i64 *ng[64 * 2 + 1], *nb[64 * 2 + 1]; /* ln1.l = 2l, ln2.l = 2l+1, lnf = 2L: gains (16-bit) and offsets */
    i64 nge[64 * 2 + 1];
    const int16_t *emb; const i64 *embe;       /* embed_in [V][d] and its per-word power of two */
    const i64 *PHI, *ARR, *LOG2, *EXP2, *COS, *SIN;
    i64 alen, eps40, half;
    int flags;                                 /* F_GAUGE | F_TURN | F_EDGE | F_ARRIVAL (pythia_base2.py:20) */
    double *cosf, *sinf;                       /* turn=float: cos/sin of pos * 10000^(-2i/rot), [ctx][rot/2] */
} pmodel_t;

void *b2p_create(int L, int d, int H, int F, int V, int ctx, int rot) {
    pmodel_t *m = (pmodel_t *)calloc(1, sizeof(pmodel_t));
    m->L = L; m->d = d; m->H = H; m->hd = d / H; m->F = F; m->V = V; m->ctx = ctx; m->rot = rot;
    return m;
}
/* pythia_base2.py:118-120: ang = pos * 10000^(-(0, 2, .., rot-2) / rot), its cos and sin (the C library's, which
 * are numpy's float64 cos/sin) */
void b2p_set_flags(void *mv, int flags) {
    pmodel_t *m = (pmodel_t *)mv;
    m->flags = flags;
    free(m->cosf); free(m->sinf); m->cosf = m->sinf = NULL;
    if (!(flags & F_TURN)) return;
    const int r = m->rot / 2;
    m->cosf = (double *)malloc(sizeof(double) * (size_t)m->ctx * r);
    m->sinf = (double *)malloc(sizeof(double) * (size_t)m->ctx * r);
    for (int t = 0; t < r; t++) {
        const double inv = pow(10000.0, (double)(-2 * t) / (double)m->rot);
        for (int p = 0; p < m->ctx; p++) {
            const double ang = (double)p * inv;
            m->cosf[(size_t)p * r + t] = cos(ang);
            m->sinf[(size_t)p * r + t] = sin(ang);
        }
    }
}
void b2p_destroy(void *mv) {
    pmodel_t *m = (pmodel_t *)mv;
    free(m->cosf); free(m->sinf); free(m);
}
void b2p_set_bank(void *mv, int idx, const int16_t *w, const i64 *e, const i64 *b, int nin, int nout) {
    pmodel_t *m = (pmodel_t *)mv;
    m->bank[idx].w = w; m->bank[idx].e = e; m->bank[idx].b = b; m->bank[idx].nin = nin; m->bank[idx].nout = nout;
}
void b2p_set_norm(void *mv, int idx, const i64 *g, i64 ge, const i64 *b) {
    pmodel_t *m = (pmodel_t *)mv;
    m->ng[idx] = g; m->nge[idx] = ge; m->nb[idx] = b;
}
void b2p_set_tables(void *mv, const int16_t *emb, const i64 *embe, const i64 *PHI, const i64 *ARR, i64 alen,
                    const i64 *LOG2, const i64 *EXP2, const i64 *COS, const i64 *SIN, i64 eps40, i64 half) {
    pmodel_t *m = (pmodel_t *)mv;
    m->emb = emb; m->embe = embe; m->PHI = PHI; m->ARR = ARR; m->alen = alen; m->LOG2 = LOG2; m->EXP2 = EXP2;
    m->COS = COS; m->SIN = SIN; m->eps40 = eps40; m->half = half;
}

/* pythia_base2.py:100-110 gauge for one row: c = d*x16 - S1, V = d*S2 - S1^2 + (EPS40 >> (40 + 2 ex)),
 * LS = log2fix(V) >> 1, out = power(c*g, (ge + 16)*65536 - LS) + b (exact power). */
static int gauge_ln_row(const pmodel_t *m, int idx, const i64 *R, i64 *out, i64 *x16) {
    const int d = m->d;
    if (m->flags & F_GAUGE) {          /* pythia_base2.py:102-104 */
        double *x = (double *)malloc(sizeof(double) * 2 * d);
        const double sg = row_sigma(R, d, x, x + d), sc = ldexp(1.0, (int)m->nge[idx]);
        for (int i = 0; i < d; i++)
            out[i] = wadd((i64)rint(x[i] / sg * (double)m->ng[idx][i] * sc * 65536.0), m->nb[idx][i]);
        free(x);
        return 0;
    }
    i64 ex = -16 + to16_row(R, d, x16);
    i64 S1 = 0, S2 = 0;
    for (int i = 0; i < d; i++) { S1 = wadd(S1, x16[i]); S2 = wadd(S2, wmul(x16[i], x16[i])); }
    i64 V = wadd(wsub(wmul(d, S2), wmul(S1, S1)), np_rsh(m->eps40, 40 + 2 * ex));
    i64 LS = log2fix1(V, m->LOG2) >> 1;
    i64 F = wsub(wmul(wadd(m->nge[idx], 16), 65536), LS);
    for (int i = 0; i < d; i++) {
        i64 c = wsub(wmul(d, x16[i]), S1);
        if (power_exact1(wmul(c, m->ng[idx][i]), F, m->EXP2, &out[i])) return -1;
        out[i] = wadd(out[i], m->nb[idx][i]);
    }
    return 0;
}

/* pythia_base2.py:112-114 plain for one row into out (bias b may be NULL: the head) */
static void plain_row(const pmodel_t *m, const bank_t *bk, const i64 *X, i64 *out, i64 *x16, i64 *pile, int par) {
    i64 ex = -16 + to16_row(X, bk->nin, x16);
    product_row(x16, bk, pile, par);
    for (int j = 0; j < bk->nout; j++)
        out[j] = wadd(rshift1(pile[j], -wadd(wadd(bk->e[j], ex), 16)), bk->b ? bk->b[j] : 0);
}

/* pythia_base2.py:116-123 turn for one head part of one position: pairs (i, i + rot/2), cos/sin at 2^-30 */
static int turn_row(const pmodel_t *m, const i64 *x, int pos, i64 *y) {
    const int r = m->rot / 2;
    for (int t = 0; t < m->hd; t++) y[t] = x[t];
    if (m->flags & F_TURN) {           /* pythia_base2.py:118-120 */
        for (int t = 0; t < r; t++) {
            const double c = m->cosf[(size_t)pos * r + t], s = m->sinf[(size_t)pos * r + t];
            const double a = (double)x[t], b = (double)x[t + r];
            y[t] = (i64)rint(a * c - b * s);
            y[t + r] = (i64)rint(b * c + a * s);
        }
        return 0;
    }
    for (int t = 0; t < m->rot; t++) if ((x[t] < 0 ? -x[t] : x[t]) >= ((i64)1 << 31)) return -1;
    for (int t = 0; t < r; t++) {
        i64 c = m->COS[(size_t)pos * r + t], s = m->SIN[(size_t)pos * r + t], a = x[t], b = x[t + r];
        y[t] = rshift1(wsub(wmul(a, c), wmul(b, s)), 30);
        y[t + r] = rshift1(wadd(wmul(b, c), wmul(a, s)), 30);
    }
    return 0;
}

/* the per-stream store for Pythia: k16, its exponent, v (full width) per layer */
static int pcache_alloc(const pmodel_t *m, cache_t *c, int ctx) {
    size_t n = (size_t)m->L * ctx;
    c->k16 = (i64 *)malloc(sizeof(i64) * n * m->d);
    c->ek = (i64 *)malloc(sizeof(i64) * n * m->H);
    c->v = (i64 *)malloc(sizeof(i64) * n * m->d);
    c->kraw = (m->flags & F_ARRIVAL) ? (i64 *)malloc(sizeof(i64) * n * m->d) : NULL;   /* turned keys, full width */
    return c->k16 && c->ek && c->v && (c->kraw || !(m->flags & F_ARRIVAL));
}

/* pythia_base2.py:125-141 attention at position p of one stream, given qkv (this position's [3d], per head q, k, v
 * in Pythia's order) and the store (k16 turned and to16'd, v raw) for 0..p already filled by the caller. */
static int pattend_row(const pmodel_t *m, const cache_t *c, int l, int ctx, int p, const i64 *qkv, i64 *out, i64 *sc) {
    const int d = m->d, hd = m->hd;
    i64 qt[256], q16[256];
    if (m->flags & F_ARRIVAL) {        /* pythia_base2.py:130-133 */
        double *e = (double *)sc;
        for (int h = 0; h < m->H; h++) {
            if (turn_row(m, qkv + h * 3 * hd, p, qt)) return -1;
            arrival_float_row(qt, c->kraw + ((size_t)l * ctx) * d + h * hd, d, c->v + ((size_t)l * ctx) * d + h * hd, d,
                              p, hd, out + h * hd, e);
        }
        return 0;
    }
    for (int h = 0; h < m->H; h++) {
        if (turn_row(m, qkv + h * 3 * hd, p, qt)) return -1;
        i64 eq = -16 + to16_row(qt, hd, q16);
        const i64 *K = c->k16 + ((size_t)l * ctx) * d + h * hd;
        const i64 *EK = c->ek + ((size_t)l * ctx) * m->H + h;
        const i64 *Vv = c->v + ((size_t)l * ctx) * d + h * hd;
        i64 lev = INT64_MIN;
        for (int s = 0; s <= p; s++) {
            i64 dot = 0;
            const i64 *k = K + (size_t)s * d;
            for (int t = 0; t < hd; t++) dot += q16[t] * k[t];
            i64 F = wsub(wmul(eq + EK[(size_t)s * m->H] + 10, 65536), m->half);
            if (power_exact1(dot, F, m->EXP2, &sc[s])) return -1;
            if (sc[s] > lev) lev = sc[s];
        }
        i64 Z = 0, num[256];
        for (int t = 0; t < hd; t++) num[t] = 0;
        for (int s = 0; s <= p; s++) {
            i64 dd = wsub(lev, sc[s]);
            i64 a = dd < m->alen ? m->ARR[dd < 0 ? 0 : dd] : 0;
            if (!a) continue;
            Z = wadd(Z, a);
            const i64 *v = Vv + (size_t)s * d;
            for (int t = 0; t < hd; t++) num[t] = wadd(num[t], wmul(a, v[t]));
        }
        i64 F = -log2fix1(Z, m->LOG2);
        for (int t = 0; t < hd; t++) if (power_exact1(num[t], F, m->EXP2, &out[h * hd + t])) return -1;
    }
    return 0;
}

typedef struct { i64 *R, *G, *qkv, *att, *hid, *x16, *pile, *sc, *At, *Mo; } pscratch_t;

static int pscratch_alloc(const pmodel_t *m, pscratch_t *s, int ctx) {
    int wmax = m->V > m->F ? m->V : m->F;
    s->R = (i64 *)malloc(sizeof(i64) * m->d); s->G = (i64 *)malloc(sizeof(i64) * m->d);
    s->qkv = (i64 *)malloc(sizeof(i64) * 3 * m->d); s->att = (i64 *)malloc(sizeof(i64) * m->d);
    s->hid = (i64 *)malloc(sizeof(i64) * m->F); s->x16 = (i64 *)malloc(sizeof(i64) * (m->F > m->d ? m->F : m->d));
    s->pile = (i64 *)malloc(sizeof(i64) * wmax); s->sc = (i64 *)malloc(sizeof(i64) * ctx);
    s->At = (i64 *)malloc(sizeof(i64) * m->d); s->Mo = (i64 *)malloc(sizeof(i64) * m->d);
    return s->R && s->G && s->qkv && s->att && s->hid && s->x16 && s->pile && s->sc && s->At && s->Mo;
}
static void pscratch_free(pscratch_t *s) {
    free(s->R); free(s->G); free(s->qkv); free(s->att); free(s->hid); free(s->x16); free(s->pile); free(s->sc);
    free(s->At); free(s->Mo);
}

/* One new position of one stream (pythia_base2.py:151-160): returns the race's word (logits given) or -1 (none),
 * -2 on a value the reference would reject (an exact power outside int64, a turn input past 2^31). */
static int pposition(const pmodel_t *m, cache_t *c, pscratch_t *s, int ctx, int p, int id, i64 *logits, int par) {
    const int d = m->d, H = m->H, hd = m->hd;
    for (int i = 0; i < d; i++) s->R[i] = rshift1((i64)m->emb[(size_t)id * d + i], -(m->embe[id] + 16));
    for (int l = 0; l < m->L; l++) {
        /* attention branch */
        if (gauge_ln_row(m, 2 * l, s->R, s->G, s->x16)) return -2;
        plain_row(m, &m->bank[4 * l + 0], s->G, s->qkv, s->x16, s->pile, par);
        for (int h = 0; h < H; h++) {
            i64 kt[256];
            if (turn_row(m, s->qkv + h * 3 * hd + hd, p, kt)) return -2;
            c->ek[((size_t)l * ctx + p) * H + h] = -16 + to16_row(kt, hd, c->k16 + ((size_t)l * ctx + p) * d + h * hd);
            if (c->kraw) memcpy(c->kraw + ((size_t)l * ctx + p) * d + h * hd, kt, sizeof(i64) * hd);
            memcpy(c->v + ((size_t)l * ctx + p) * d + h * hd, s->qkv + h * 3 * hd + 2 * hd, sizeof(i64) * hd);
        }
        if (pattend_row(m, c, l, ctx, p, s->qkv, s->att, s->sc)) return -2;
        plain_row(m, &m->bank[4 * l + 1], s->att, s->At, s->x16, s->pile, par);
        /* MLP branch, from the same R */
        if (gauge_ln_row(m, 2 * l + 1, s->R, s->G, s->x16)) return -2;
        plain_row(m, &m->bank[4 * l + 2], s->G, s->hid, s->x16, s->pile, par);
        for (int j = 0; j < m->F; j++) s->hid[j] = (m->flags & F_EDGE) ? edge_erf1(s->hid[j]) : edge1(s->hid[j], m->PHI);
        plain_row(m, &m->bank[4 * l + 3], s->hid, s->Mo, s->x16, s->pile, par);
        for (int i = 0; i < d; i++) s->R[i] = wadd(wadd(s->R[i], s->At[i]), s->Mo[i]);
    }
    if (!logits) return -1;
    if (gauge_ln_row(m, 2 * m->L, s->R, s->G, s->x16)) return -2;
    plain_row(m, &m->bank[4 * m->L], s->G, logits, s->x16, s->pile, par);
    return (int)race1(logits, m->V);
}

/* greedy words for B streams of equal prompt length (the loop of pythia_base2.py:175), logits and their digests
 * (b2o_logit_hash) optional */
static int pgen_core(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, i64 *logits, u64 *hashes,
                     int threads) {
    const pmodel_t *m = (const pmodel_t *)mv;
    int ctx = P + n_new;
    if (ctx > m->ctx || P < 1) return -1;
    int nt = nthreads(threads), err = 0, par = B == 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (B > 1)
    for (int b = 0; b < B; b++) {
        cache_t c; pscratch_t s;
        i64 *lg = (i64 *)malloc(sizeof(i64) * m->V);
        if (!pcache_alloc(m, &c, ctx) || !pscratch_alloc(m, &s, ctx) || !lg) { err = -1; continue; }
        for (int p = 0; p < P - 1 && !err; p++)
            if (pposition(m, &c, &s, ctx, p, ids[(size_t)b * P + p], NULL, par) == -2) err = -2;
        int tok = ids[(size_t)b * P + P - 1];
        for (int t = 0; t < n_new && !err; t++) {
            tok = pposition(m, &c, &s, ctx, P - 1 + t, tok, lg, par);
            if (tok == -2) { err = -2; break; }
            tokens[(size_t)b * n_new + t] = tok;
            if (logits) memcpy(logits + ((size_t)b * n_new + t) * m->V, lg, sizeof(i64) * m->V);
            if (hashes) hashes[(size_t)b * n_new + t] = b2o_logit_hash(lg, m->V);
        }
        cache_free(&c); pscratch_free(&s); free(lg);
    }
    return err;
}
int b2p_generate(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, i64 *logits, int threads) {
    return pgen_core(mv, ids, B, P, n_new, tokens, logits, NULL, threads);
}
int b2p_generate_digest(void *mv, const int32_t *ids, int B, int P, int n_new, int32_t *tokens, u64 *hashes,
                        int threads) {
    return pgen_core(mv, ids, B, P, n_new, tokens, NULL, hashes, threads);
}

/* teacher-forced scores at positions [first, last) of one stream (pythia_base2.py:151-160 with last) */
int b2p_scores(void *mv, const int32_t *ids, int P, int first, int last, i64 *logits) {
    const pmodel_t *m = (const pmodel_t *)mv;
    if (P > m->ctx || first < 0 || last > P || first >= last) return -1;
    cache_t c; pscratch_t s;
    if (!pcache_alloc(m, &c, P) || !pscratch_alloc(m, &s, P)) return -1;
    int rc = 0;
    for (int p = 0; p < P && !rc; p++)
        if (pposition(m, &c, &s, P, p, ids[p], (p >= first && p < last) ? logits + (size_t)(p - first) * m->V : NULL, 1) == -2)
            rc = -2;
    cache_free(&c); pscratch_free(&s);
    return rc;
}

/* element entry points for the pinning tests */
int b2p_gauge(void *mv, int idx, const i64 *R, int rows, i64 *out) {
    const pmodel_t *m = (const pmodel_t *)mv;
    i64 *x16 = (i64 *)malloc(sizeof(i64) * m->d);
    int rc = 0;
    for (int r = 0; r < rows && !rc; r++) rc = gauge_ln_row(m, idx, R + (size_t)r * m->d, out + (size_t)r * m->d, x16);
    free(x16);
    return rc;
}
int b2p_turn(void *mv, const i64 *X, const i64 *pos, int rows, i64 *Y) {
    const pmodel_t *m = (const pmodel_t *)mv;
    for (int r = 0; r < rows; r++) if (turn_row(m, X + (size_t)r * m->hd, (int)pos[r], Y + (size_t)r * m->hd)) return -1;
    return 0;
}
int b2p_plain(void *mv, int idx, const i64 *X, int rows, i64 *out) {
    const pmodel_t *m = (const pmodel_t *)mv;
    const bank_t *bk = &m->bank[idx];
    i64 *x16 = (i64 *)malloc(sizeof(i64) * bk->nin), *pile = (i64 *)malloc(sizeof(i64) * bk->nout);
    for (int r = 0; r < rows; r++) plain_row(m, bk, X + (size_t)r * bk->nin, out + (size_t)r * bk->nout, x16, pile, 1);
    free(x16); free(pile);
    return 0;
}
/* pythia_base2.py:125-141 over a whole sequence's QKV [P][3d] */
int b2p_attention(void *mv, const i64 *QKV, int P, i64 *out) {
    const pmodel_t *m = (const pmodel_t *)mv;
    const int d = m->d, H = m->H, hd = m->hd;
    pmodel_t one = *m; one.L = 1;
    cache_t c; i64 *sc = (i64 *)malloc(sizeof(i64) * P);
    if (!pcache_alloc(&one, &c, P) || !sc) return -1;
    for (int p = 0; p < P; p++)
        for (int h = 0; h < H; h++) {
            i64 kt[256];
            if (turn_row(m, QKV + (size_t)p * 3 * d + h * 3 * hd + hd, p, kt)) return -2;
            c.ek[(size_t)p * H + h] = -16 + to16_row(kt, hd, c.k16 + (size_t)p * d + h * hd);
            if (c.kraw) memcpy(c.kraw + (size_t)p * d + h * hd, kt, sizeof(i64) * hd);
            memcpy(c.v + (size_t)p * d + h * hd, QKV + (size_t)p * 3 * d + h * 3 * hd + 2 * hd, sizeof(i64) * hd);
        }
    int rc = 0;
    for (int p = 0; p < P && !rc; p++) rc = pattend_row(&one, &c, 0, P, p, QKV + (size_t)p * 3 * d, out + (size_t)p * d, sc);
    cache_free(&c); free(sc);
    return rc;
}
