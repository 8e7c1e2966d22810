// b2_arith.cuh -- the machine's integer arithmetic on the device, bit-for-bit the reference's numpy int64 semantics.
//
// The reference machine (base2.py) computes in numpy int64, so:
//   * +, -, * wrap modulo 2^64 (power()'s X * EXP2 does wrap at long contexts, base2.py:53);
//   * np.left_shift by >= 64 gives 0, np.right_shift by >= 64 gives the sign fill;
//   * rshift(X, s) (base2.py:18-22) adds 2^(s-1) then shifts arithmetically; s <= 0 shifts left.
// Signed overflow is undefined behaviour in C++, so every wrapping operation is done on uint64_t.
#pragma once
#include <stdint.h>

#define B2_DEV __device__ __forceinline__

namespace b2 {

B2_DEV int64_t wadd(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
B2_DEV int64_t wsub(int64_t a, int64_t b) { return (int64_t)((uint64_t)a - (uint64_t)b); }
B2_DEV int64_t wmul(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }
B2_DEV int64_t np_lsh(int64_t x, int64_t s) { return (s < 0 || s >= 64) ? 0 : (int64_t)((uint64_t)x << s); }
B2_DEV int64_t np_rsh(int64_t x, int64_t s) { return s >= 64 ? (x < 0 ? -1 : 0) : (s < 0 ? 0 : (x >> s)); }

// base2.py:18-22
B2_DEV int64_t rshift(int64_t x, int64_t s) {
    if (s > 0 && s < 64) return (int64_t)((uint64_t)x + (1ull << (s - 1))) >> s;   // the common case, same bits
    int64_t up = np_lsh(x, s < 0 ? -s : 0);
    int64_t sp = s > 0 ? s : 0;
    int64_t half = sp > 0 ? np_lsh(1, sp - 1) : 0;
    return np_rsh(wadd(up, half), sp);
}

// Python int.bit_length() of an int64 (of its magnitude; 64 for INT64_MIN)
B2_DEV int bitlen(int64_t v) {
    uint64_t m = v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v;
    return 64 - __clzll((long long)m);
}
B2_DEV int bitlen_u(uint64_t m) { return 64 - __clzll((long long)m); }

// |x| as the OR-able magnitude (numpy np.abs wraps INT64_MIN onto itself)
B2_DEV uint64_t mag(int64_t x) { return x < 0 ? (uint64_t)0 - (uint64_t)x : (uint64_t)x; }

// to16's shift from the OR of a row's magnitudes (base2.py:24-27): max(bit_length - 15, 0).
// The OR is interpreted as numpy int64 (bit 63 set means a negative number), as base2.py's int(v).bit_length() does.
B2_DEV int to16_shift(uint64_t orv) {
    int top = bitlen((int64_t)orv);
    return top > 15 ? top - 15 : 0;
}

// base2.py:42-48
B2_DEV int64_t log2fix(int64_t v, const int32_t* __restrict__ LOG2) {
    int t = bitlen(v) - 1;
    int64_t m = t >= 16 ? ((v >> (t - 16)) & 0xFFFF) : (np_lsh(v, 16 - t) & 0xFFFF);
    return (int64_t)t * 65536 + (int64_t)__ldg(LOG2 + m);
}

// base2.py:50-53
B2_DEV int64_t power(int64_t x, int64_t F, const int32_t* __restrict__ EXP2) {
    int64_t I = F >> 16, f = F & 0xFFFF;
    return rshift(wmul(x, (int64_t)__ldg(EXP2 + f)), 16 - I);
}

// pythia_base2.py:87-90: power with Python's whole numbers (the reference leaves int64 past |X| >= 2^45): the
// product in 128 bits, the rounded shift, the result back in int64. *bad is set when it does not fit (where the
// reference's astype(np.int64) raises). Equals power() whenever power() does not wrap.
B2_DEV int64_t power_exact(int64_t x, int64_t F, const int32_t* __restrict__ EXP2, bool* bad) {
    const int64_t I = F >> 16, f = F & 0xFFFF, s = 16 - I;
    const __int128 p = (__int128)x * (__int128)__ldg(EXP2 + f);
    __int128 r;
    if (s <= 0) {
        if (p == 0) return 0;
        if (-s >= 64) { *bad = true; return 0; }
        r = p << (-s);
        if ((r >> (-s)) != p) { *bad = true; return 0; }
    } else if (s >= 100) {
        r = 0;                                    // |p| < 2^81
    } else {
        r = (p + ((__int128)1 << (s - 1))) >> s;  // floor, as Python's >>
    }
    if (r > (__int128)INT64_MAX || r < (__int128)INT64_MIN) { *bad = true; return 0; }
    return (int64_t)r;
}

// base2.py:78-83 (integer bend)
B2_DEV int64_t edge(int64_t h, const int32_t* __restrict__ PHI) {
    int64_t idx = wadd(rshift(h, 16 - 12), 32768);
    int64_t share = idx < 0 ? 0 : (idx > 65535 ? 65536 : (int64_t)__ldg(PHI + idx));
    return rshift(wmul(h, share), 16);
}

// the gauge's V = 768*S2 - S1^2 + (EPS40 >> (40 + 2 ex)) and LS (base2.py:57-60)
B2_DEV int64_t gauge_LS(int64_t S1, int64_t S2, int ex, const int32_t* __restrict__ LOG2, int64_t log768, int64_t eps40) {
    int64_t V = wsub(wmul(768, S2), wmul(S1, S1));
    int64_t sh = 40 + 2 * (int64_t)ex;
    V = wadd(V, sh >= 0 ? np_rsh(eps40, sh) : np_lsh(eps40, -sh));
    return wadd(wsub(log2fix(V, LOG2) >> 1, log768), wmul(ex, 65536));
}

// ---- warp / block reductions ---------------------------------------------------------------------------------------
B2_DEV uint64_t warp_or64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
B2_DEV int64_t warp_sum64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = wadd(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
B2_DEV int64_t warp_max64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) { int64_t u = __shfl_xor_sync(0xffffffffu, v, o); v = u > v ? u : v; }
    return v;
}
B2_DEV uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) { uint64_t u = __shfl_xor_sync(0xffffffffu, v, o); v = u > v ? u : v; }
    return v;
}
// (value, index) keep-larger with ties to the lower index: the race (base2.py:34-40)
B2_DEV void race_merge(int64_t& v, int& i, int64_t ov, int oi) {
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}
B2_DEV void warp_race(int64_t& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        int64_t ov = __shfl_xor_sync(0xffffffffu, v, o);
        int oi = __shfl_xor_sync(0xffffffffu, i, o);
        race_merge(v, i, ov, oi);
    }
}

}  // namespace b2
