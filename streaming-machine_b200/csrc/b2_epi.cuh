// b2_epi.cuh -- pieces shared by every bank-product kernel (CUDA-core and tensor-core): the device error word and
// what a bank does with a finished pile (base2.py:62-83).
#pragma once
#include <stdint.h>
#include "b2_arith.cuh"

namespace b2 {

// sticky device error bits (read back by b2_sync)
enum : uint32_t {
    DERR_TOKEN = 1u,     // a token id outside [0, vocab)
    DERR_POS = 2u,       // a position at or past the store's context (or the position table)
    DERR_VOVF = 4u,      // a V value outside int32 (the value store holds int32)
    DERR_INDEX = 8u,     // an arrival-table index below -len (where base2.py raises IndexError)
    DERR_TIMEOUT = 16u,  // a bounded wait in a tensor-core kernel gave up (the results of that call are void)
    DERR_RANGE = 32u,    // a value where the reference raises: an exact power outside int64, a turn input past 2^31
};

B2_DEV void set_err(uint32_t* err, uint32_t bit) { atomicOr(err, bit); }

// the per-stream key/value store (one per engine)
struct KV {
    int16_t* k;        // [slot][L][H][ctx][64]
    uint64_t* kmask;   // [slot][L][H][ctx]  bit t: k16[t] == +32768
    int32_t* kexp;     // [slot][L][H][ctx]
    int32_t* v;        // [slot][L][H][ctx][64]
    int L, H, ctx;     // ctx: the positions' stride (a multiple of 16, so every (slot, layer, head) run is 16-byte aligned)
    int lim;           // positions actually allocated to a stream (max_ctx); a position at or past it is an error
    int64_t* kraw = nullptr;   // arrival=float only: the keys at full width, [slot][L][H][ctx][64]
};

// position of (slot, layer, head, pos) in the key/value store: [slot][layer][head][pos]
B2_DEV size_t kv_index(int slot, int layer, int head, int pos, int L, int H, int ctx) {
    return (((size_t)slot * L + layer) * H + head) * (size_t)ctx + pos;
}

enum { EPI_GAUGED = 0, EPI_GAUGED_EDGE = 1, EPI_PLAIN_ADD = 2, EPI_PLAIN_OUT = 3, EPI_PLAIN_EDGE = 4 };

// what a bank does with a finished pile (row r, output column j)
struct EpiArgs {
    const int32_t* ex;      // [rows] the input's power of two
    const int64_t* LS;      // [rows] the gauge (gauged banks)
    const int32_t* e;       // [nout] the column's power of two
    const int64_t* b;       // [nout] bias
    int64_t* out;           // [out row][ldo]
    int ldo;
    const int32_t* out_map; // optional row -> out row
    const int32_t* EXP2;
    const int32_t* PHI;
};

// the same arithmetic with the row's quantities already at hand: exr = the input's power of two, LSr = the gauge,
// e2r = EXP2[(-LSr) & 0xFFFF] (power()'s table read depends only on the row, since F = 65536*(e_j + exr + 16) - LSr).
template <int EPI>
B2_DEV int64_t epi_value(int64_t pile, int64_t e_j, int64_t b_j, int64_t exr, int64_t LSr, int64_t e2r,
                         const int32_t* __restrict__ PHI) {
    int64_t es = wadd(wadd(e_j, exr), 16);
    if (EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE) {
        int64_t F = wsub(wmul(es, 65536), LSr);
        int64_t v = wadd(rshift(wmul(pile, e2r), 16 - (F >> 16)), b_j);
        return EPI == EPI_GAUGED_EDGE ? edge(v, PHI) : v;
    }
    const int64_t v = wadd(rshift(pile, -es), b_j);
    return EPI == EPI_PLAIN_EDGE ? edge(v, PHI) : v;     // pythia_base2.py:156 edge(plain(..., fc))
}

// PDL: wait for the kernels this one depends on (no-op without programmatic launch), and let the next one start
B2_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B2_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <int EPI>
B2_DEV void epi_store(const EpiArgs& a, int r, int j, int64_t pile) {
    int orow = a.out_map ? a.out_map[r] : r;
    int64_t* o = a.out + (size_t)orow * a.ldo + j;
    int64_t es = wadd(wadd((int64_t)a.e[j], (int64_t)a.ex[r]), 16);
    if (EPI == EPI_GAUGED || EPI == EPI_GAUGED_EDGE) {
        int64_t F = wsub(wmul(es, 65536), a.LS[r]);        // base2.py:70
        int64_t v = wadd(power(pile, F, a.EXP2), a.b[j]);  // base2.py:71
        if (EPI == EPI_GAUGED_EDGE) v = edge(v, a.PHI);    // base2.py:106 edge(gauged_bank(...))
        *o = v;
    } else {
        int64_t v = wadd(rshift(pile, -es), a.b[j]);       // base2.py:76
        if (EPI == EPI_PLAIN_EDGE) v = edge(v, a.PHI);
        *o = EPI == EPI_PLAIN_ADD ? wadd(*o, v) : v;       // base2.py:105-106 R = R + ...
    }
}

// ARR read as base2.py:97 does it: ARR[min(d, len-1)] where d < len, else 0. d is never negative unless a score
// wrapped; numpy would then index from the table's end (d >= -len) or raise (d < -len, flagged here).
B2_DEV int64_t arrival(int64_t d, const int32_t* __restrict__ ARR, int alen, uint32_t* err) {
    if (d >= alen) return 0;
    if (d >= 0) return (int64_t)__ldg(ARR + d);
    if (d >= -(int64_t)alen) return (int64_t)__ldg(ARR + (alen + d));
    set_err(err, DERR_INDEX);
    return 0;
}

}  // namespace b2
