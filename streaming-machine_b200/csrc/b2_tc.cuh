// b2_tc.cuh -- the bank product on the 5th-generation tensor cores (tcgen05, kind::i8). Interface used by
// b2_engine.cu; the kernels live in b2_tc.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2 {

// A bank in the tensor-core layout: w = 256*wh + (wl + 128) + ... split into two signed int8 planes, K-major.
struct TcBank {
    int ready = 0;
    int nin = 0, nout = 0, nout_pad = 0;
    int8_t* wh = nullptr;       // [nout_pad][nin]  w >> 8
    int8_t* wl = nullptr;       // [nout_pad][nin]  (w & 255) - 128
    int64_t* colsum = nullptr;  // [nout]  sum_i w[i][j]
    alignas(64) unsigned char tmap_wh[128];
    alignas(64) unsigned char tmap_wl[128];
};

// Row-side buffers: the activations' planes and their corrections.
struct TcRows {
    int max_rows = 0, kmax = 0;
    int8_t* xh = nullptr;       // [max_rows_pad][kmax]
    int8_t* xl = nullptr;       // [max_rows_pad][kmax]
    int64_t* rowsum = nullptr;  // [max_rows]  sum_i x_repr[i]
    int32_t* nsat = nullptr;    // [max_rows]  entries equal to +32768
    int16_t* sat = nullptr;     // [max_rows][kmax] their indices
    int64_t* pile = nullptr;    // split-K accumulation [max_rows][max nout]
    uint32_t* tiles = nullptr;  // split-K arrival counters
};

int tc_min_rows_default();
int tc_bank_build(TcBank& t, const int16_t* w, int nin, int nout);
void tc_bank_free(TcBank& t);
int tc_rows_alloc(TcRows& r, int max_rows, int kmax);
void tc_rows_free(TcRows& r);
void tc_planes(TcRows& r, const int32_t* x16, int n, int rows, cudaStream_t st);
int tc_bank(const TcBank& t, TcRows& r, int epi, int rows, const int32_t* ex, const int64_t* LS, const int32_t* e,
            const int64_t* b, int64_t* out, int ldo, const int32_t* out_map, const int32_t* EXP2, const int32_t* PHI,
            cudaStream_t st);

}  // namespace b2
