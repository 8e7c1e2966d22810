// b2_tc.cuh -- the bank product on the 5th-generation tensor cores (tcgen05.mma kind::i8, accumulators in TMEM,
// operands staged by TMA). Interface used by b2_engine.cu; kernels in b2_tc.cu.
//
// Exactness. A weight w (|w| <= 32767) and an activation x16 (-32768..32768) are each split into two signed bytes:
//     w = 256*wh + wls + 128         wh = w >> 8,            wls = (w & 255) - 128
//     x = 256*xh + xls + 128 (+256)  xh = min(x >> 8, 127),  xls = (x & 255) - 128   (+256 only for x = +32768)
// Three int32 accumulators per output, A1 = sum wh*xh, A2 = sum wh*xls + wls*xh, A3 = sum wls*xls, are exact
// (|A| < 2^27 for 3072 inputs), and the pile (base2.py:29-32) is recovered exactly in int64:
//     pile = 65536*A1 + 256*A2 + A3 + 128*sum(w) + 128*sum(x_repr) - 16384*nin + 256*sum_{x_i = 32768} w_i
// where x_repr is x with +32768 read as 32512. The last term runs over a per-row list of the (rare) +32768 entries.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "b2_epi.cuh"

namespace b2 {

struct TcMap { alignas(64) unsigned char bytes[128]; };

// A bank in the tensor-core layout: the two weight planes, K-major ([out][in]), padded to 128 outputs.
struct TcBank {
    int ready = 0;
    int prebuilt = 0;            // the planes and corrections were uploaded (tc_bank_upload), not built from w
    int nin = 0, nout = 0, nout_pad = 0;
    int8_t* wh = nullptr;        // [nout_pad][nin]
    int8_t* wl = nullptr;        // [nout_pad][nin]
    int64_t* colcorr = nullptr;  // [nout_pad]  128*sum_i w[i][j] - 16384*nin
    int64_t* colcorr_kb = nullptr;  // [nin/128][nout_pad] the same per 128-input block
    const int16_t* w16 = nullptr;  // the reference-layout bank [nin][nout] (for the +32768 correction)
    TcMap map_wh, map_wl;        // box: 128 bytes of K x 128 outputs
    TcMap map_wh64, map_wl64;    // box: 128 bytes of K x 64 outputs (k_bank_wide)
    int16_t* wt = nullptr;       // heads (nout > 4096): the weights as 64-column tiles, [tile][nin][64] int16 (zeros past
                                 // nout), so that the GEMV head reads each tile as one contiguous 96 KB block
    TcMap map_w16;               // over wt as [tiles * nin][64], box 64 columns x 256 rows (k_head_gemv)
    int map_w16_ok = 0;
};

// Row-side buffers: the activations' planes and their corrections.
struct TcRows {
    int rows_cap = 0, kmax = 0;
    int8_t* xh = nullptr;       // [rows_cap][kmax]
    int8_t* xl = nullptr;       // [rows_cap][kmax]
    int64_t* rowcorr = nullptr; // [rows_cap]  128*sum_i x_repr[i]
    int32_t* nsat = nullptr;    // [rows_cap]  entries equal to +32768
    int16_t* sat = nullptr;     // [rows_cap][kmax] their indices
    uint32_t* err = nullptr;    // device error word (shared with the engine)
    struct { int k, bn; TcMap h, l, h32, l32; } maps[4];   // per K: boxes of 64 and of 32 rows
    int nmaps = 0;
};


// the qkv bank's heads16 done in its decode epilogue (instead of storing q/k/v and a separate split kernel): q16 and
// its exponent per head, k16 / mask / exponent and v appended to the key/value store at each row's position
struct TcHeads {
    int32_t* q16;
    int32_t* qexp;
    KV kv;
    const int32_t* row_slot;
    const int32_t* row_pos;
    int layer;
    int pythia = 0;                  // Pythia's parts (q, k, v per head) and its turn of q and k (16 dims)
    const int32_t* COS = nullptr;    // [n_ctx][8] at 2^-30 (Pythia)
    const int32_t* SIN = nullptr;
};

// a decode bank's rows quantised inside k_bank_wide instead of by a quant kernel before it: the rows' int64 values
// and their ORs (complete when the kernel starts), per-row accumulators for S1, S2 and the +32768 count (zero when
// the kernel starts), and an arrival counter per 32-row half (only ever increases). tc_bank fills in the planes.
struct TcQuant {
    const int64_t* X = nullptr;
    int ldx = 0;
    const uint64_t* xor_in = nullptr;
    int64_t* S1 = nullptr;
    int64_t* S2 = nullptr;
    int32_t* nsat = nullptr;
    unsigned long long* ctr = nullptr;   // [2]
    const int32_t* LOG2 = nullptr;
    int64_t log768 = 0, eps40 = 0;
    int unsplit = 0;                     // 1: one CTA per tile even where the bank would take a CTA pair (a choice made
                                         // per handle, never per launch: the arrival counter needs it fixed per site)
    int8_t* xh = nullptr;
    int8_t* xl = nullptr;
    int16_t* sat = nullptr;
    int kmax = 0;
};

// the race fused into a bank's epilogue (the head, greedy decoding): per row, the largest value over each 32-column
// group and its column (ties to the lowest), v[row * ld + group], i[row * ld + group]; ld >= 4 * (nout_pad / 128)
struct TcRace {
    int64_t* v = nullptr;
    int32_t* i = nullptr;
    int ld = 0;
};

int tc_min_rows_default();
int tc_init();
int tc_bank_build(TcBank& t, const int16_t* w, int nin, int nout);
// a layout computed ahead of time (host arrays: wh, wl [nout_pad][nin], cc [nout_pad], cckb [nin/128][nout_pad]); the
// next tc_bank_build of the same shape keeps it instead of building one
int tc_bank_upload(TcBank& t, int nin, int nout, const int8_t* wh, const int8_t* wl, const int64_t* cc, const int64_t* cckb);
int tc_bank_download(const TcBank& t, int8_t* wh, int8_t* wl, int64_t* cc, int64_t* cckb);
void tc_bank_free(TcBank& t);
int tc_rows_alloc(TcRows& r, int rows_cap, int kmax, uint32_t* err);
void tc_rows_free(TcRows& r);
// heads (optional, EPI_GAUGED): do heads16 in the epilogue when the split-K decode kernel runs; *heads_done tells
// whether k_bank_wide takes this bank for `rows` decode rows (the in-kernel quantisation needs it)
bool wide_fits(const TcBank& t, int rows, int* wz = nullptr);
int tc_bank(const TcBank& t, TcRows& r, int epi, int rows, const int32_t* ex, const int64_t* LS, const int32_t* e,
            const int64_t* b, int64_t* out, int ldo, const int32_t* out_map, const int32_t* EXP2, const int32_t* PHI,
            cudaStream_t st, bool pdl, const TcHeads* heads = nullptr, bool* heads_done = nullptr,
            uint64_t* trace = nullptr, const TcQuant* quant = nullptr, uint64_t* or_out = nullptr,
            const TcRace* race = nullptr, uint64_t* stamp = nullptr);

// the head of a decode step of <= 2 rows as a CUDA-core GEMV (k_head_gemv): X [rows][ldx] int64 quantised in the kernel
// (its OR, to16, and for EPI_GAUGED the gauge), the race in its epilogue into race (and the scores into out when out is
// given); the bank must have map_w16_ok (a head built with more than 4,096 outputs)
int tc_head_gemv(const TcBank& t, int epi, const int64_t* X, int ldx, int rows, const int32_t* e, const int64_t* b,
                 const int32_t* EXP2, const int32_t* LOG2, int64_t log768, int64_t eps40, const TcRace& race,
                 int64_t* out, int ldo, uint32_t* err, int grid, cudaStream_t st, bool pdl, uint64_t* stamp);

// layer 0's qkv bank of a decode step from the stored rows Tw [vocab][nout] = wte . W and Tp [n_ctx][nout] = wpe . W
// (valid when every embedded value is below 2^15; the gauged epilogue and heads16 as the bank does them)
int tc_entry_qkv(const TcBank& t, const int64_t* Tw, const int64_t* Tp, const int32_t* row_tok, const int64_t* wte,
                 const int64_t* wpe, int vocab, int nctx, int rows, const int32_t* e, const int64_t* b, const int32_t* EXP2,
                 const TcQuant& q, const TcHeads& hd, uint32_t* err, cudaStream_t st, bool pdl, uint64_t* stamp);
// the largest |x| of n int64 values into *out (device; *out must start at 0)
int tc_absmax(const int64_t* x, size_t n, unsigned long long* out, cudaStream_t st);

}  // namespace b2
