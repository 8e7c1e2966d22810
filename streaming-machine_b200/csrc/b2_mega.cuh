// b2_mega.cuh -- the GPT-2 decode step for up to 64 streams as one persistent kernel (b2_mega.cu). Interface used by
// b2_engine.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_epi.cuh"
#include "b2_tc.cuh"

namespace b2 {

// one layer bank as the decode-step kernel takes it: its tensor-core planes (maps), epilogue data and how its output
// tiles and K range are spread over a cluster of MEGA_CS CTAs (tpc tiles side by side, each split over ks CTAs
// holding kps K blocks of 128 inputs each)
struct MegaBank {
    const int32_t* e;
    const int64_t* b;
    const int64_t* colcorr_kb;   // [nin / 128][nout_pad]
    const int16_t* w16;          // [nin][nout] the bank as converted (the rare +32768 correction)
    int nin, nout, nout_pad, ntiles;
    int tpc, ks, kps;
};

constexpr int MEGA_CS = 6;       // CTAs per cluster

struct MegaArgs {
    const TcMap* maps;           // [4L][2] wh, wl tensor maps (device memory, 64-byte aligned)
    const MegaBank* banks;       // [4L]
    int L, H, d, F, rows;
    // the streams: row r is stream slot r; its position and word come from slot_len / slot_tok
    const int32_t* slot_len;
    const int32_t* slot_tok;
    int32_t* row_slot;
    int32_t* row_pos;
    int32_t* row_tok;
    const int64_t* wte;
    const int64_t* wpe;
    int vocab, nctx;
    // activations (rows x d, rows x F) and, per bank input, the OR of |x| over each row ([4L][64])
    int64_t* R;
    int64_t* ATT;
    int64_t* HID;
    uint64_t* OR;
    int32_t* q16;
    int32_t* qexp;
    KV kv;
    const int32_t* EXP2;
    const int32_t* PHI;
    const int32_t* LOG2;
    const int32_t* ARR;
    int alen;
    int64_t log768, eps40;
    int att_slot_bytes, att_slots;   // the arrival's per-(row, head) shared-memory buffers
    uint32_t* bar;                   // grid barrier counter, zero at launch
    uint32_t* err;
    uint64_t* trace;                 // optional: %globaltimer stamps [CTA][phase][MEGA_STAMPS] (a profiling aid)
};

constexpr int MEGA_STAMPS = 16;
constexpr int MEGA_MAX_PHASES = 64;

struct MegaPlan {
    int ready = 0;
    int nclusters = 0;
    size_t smem = 0;
    TcMap* maps = nullptr;       // device
    MegaBank* banks = nullptr;   // device
    uint32_t* bar = nullptr;     // device
};

// builds the per-bank table and tensor maps for the layer banks (tc[0 .. 4L)), sizes the grid
int mega_plan(MegaPlan& p, const TcBank* tc, const int32_t* const* e, const int64_t* const* b, int L);
void mega_free(MegaPlan& p);
// bytes of shared memory the arrival needs per (row, head) at this context; 0 if the kernel cannot take it
int mega_att_slot_bytes(int max_ctx);
int mega_launch(const MegaPlan& p, MegaArgs a, cudaStream_t st);

}  // namespace b2
