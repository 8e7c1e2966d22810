// b2_float.cuh -- the float stage switches on the device (base2.py:10-11 gauge=/edge=/arrival= float, base2.py:66-69,
// 79-80, 89-92, 110-113; Pythia's gauge=/turn=/edge=/arrival= float, pythia_base2.py:20, 102-104, 118-120, 130-133,
// 144-146). Float64 in the reference's own order of operations. Every add, multiply and divide is an explicitly
// rounded intrinsic (__dadd_rn, __dmul_rn, ...) so the compiler cannot contract a multiply and an add into one fused
// operation, which numpy's separate ufunc passes never do; means and sums follow numpy's pairwise summation order.
// The basic operations and sqrt are correctly rounded here as in numpy, so a stage built only from them (the gauge,
// the turn with host-made cos/sin tables) gives the reference's integers exactly; tanh, pow, erf and exp are
// CUDA's, within a few units in the last place of the C library's, so those stages can differ from the reference
// by one in rare places.
#pragma once
#include <stdint.h>
#include "b2_arith.cuh"

namespace b2 {

enum { FL_GAUGE = 1, FL_EDGE = 2, FL_ARRIVAL = 4, FL_TURN = 8 };   // B2_*_FLOAT in base2.h

// the bank epilogue's float stages (BankArgs::flt)
enum { FE_GAUGE = 1, FE_GAUGE_HEAD = 2, FE_EDGE_TANH = 4, FE_EDGE_ERF = 8 };

B2_DEV double i2d(int64_t x) { return __ll2double_rn(x); }
B2_DEV int64_t rint64(double x) { return (int64_t)rint(x); }   // numpy's round: half to even

// numpy's pairwise sum of a[0..n) (numpy's pairwise_sum; the order np.sum / np.mean take along a contiguous axis):
// fewer than 8 terms in order; up to 128 in eight interleaved partial sums folded ((0+1)+(2+3))+((4+5)+(6+7)) then
// the remainder in order; more: split at half the count rounded down to a multiple of 8 (recursion depth <= 6 for
// the 3,072-long rows here).
static __device__ __noinline__ double pairwise_sum(const double* a, int n) {
    if (n < 8) {
        double s = 0.0;
        for (int i = 0; i < n; i++) s = __dadd_rn(s, a[i]);
        return s;
    }
    if (n <= 128) {
        double r[8];
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] = a[j];
        int i = 8;
        for (; i < n - (n % 8); i += 8)
#pragma unroll
            for (int j = 0; j < 8; j++) r[j] = __dadd_rn(r[j], a[i + j]);
        double s = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                             __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
        for (; i < n; i++) s = __dadd_rn(s, a[i]);
        return s;
    }
    int n2 = n / 2;
    n2 -= n2 % 8;
    const double left = pairwise_sum(a, n2);
    return __dadd_rn(left, pairwise_sum(a + n2, n - n2));
}

// an exact 128-bit integer as the nearest double (ties to even); the same steps as the oracle's
B2_DEV double i128_to_double(__int128 x) {
    if (x >= (__int128)INT64_MIN && x <= (__int128)INT64_MAX) return i2d((int64_t)x);
    const bool neg = x < 0;
    const unsigned __int128 u = neg ? (unsigned __int128)0 - (unsigned __int128)x : (unsigned __int128)x;
    const uint64_t hi = (uint64_t)(u >> 64);
    const int top = 127 - __clzll((long long)hi);             // hi != 0 here
    const int sh = top - 62;
    const uint64_t keep = (uint64_t)(u >> sh);
    const bool sticky = (u & (((unsigned __int128)1 << sh) - 1)) != 0;
    uint64_t mant = keep >> 10;
    const uint64_t rem = keep & 1023;
    if (rem > 512 || (rem == 512 && (sticky || (mant & 1)))) mant++;
    const double r = scalbn(__ull2double_rn(mant), sh + 10);
    return neg ? -r : r;
}

// base2.py:79-80: 0.5 h (1 + tanh(0.7978845608028654 (h + 0.044715 h^3))) at 2^-16, rounded
B2_DEV int64_t edge_tanh(int64_t H) {
    const double h = __ddiv_rn(i2d(H), 65536.0);
    const double t = __dmul_rn(0.7978845608028654, __dadd_rn(h, __dmul_rn(0.044715, pow(h, 3.0))));
    return rint64(__dmul_rn(__dmul_rn(__dmul_rn(0.5, h), __dadd_rn(1.0, tanh(t))), 65536.0));
}
// pythia_base2.py:144-146: h 0.5 (1 + erf(h / sqrt 2)) at 2^-16, rounded
B2_DEV int64_t edge_erf(int64_t H) {
    const double h = __ddiv_rn(i2d(H), 65536.0);
    const double e = erf(__ddiv_rn(h, 1.4142135623730951));
    return rint64(__dmul_rn(__dmul_rn(__dmul_rn(h, 0.5), __dadd_rn(1.0, e)), 65536.0));
}

}  // namespace b2
