// b2_engine.cu -- libbase2cuda.so: the C ABI (include/base2.h) over the machine's sm_100a kernels.
//
// One handle = one model on one GPU + a set of stream slots, each with its own key/value store. Work is organised in
// ROWS: a row is (stream slot, position, token). A prompt pass is many rows per stream (chunked); a decode step is
// one row per stream. Every kernel reads the row table from device memory, so a decode step is position-agnostic on
// the host and can be replayed from a CUDA graph.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/base2.h"
#include "b2_kernels.cuh"
#include "b2_tc.cuh"

using namespace b2;

namespace {

struct DevBank {
    int nin = 0, nout = 0;
    int16_t* w = nullptr;   // [nin][nout] (reference layout, CUDA-core path)
    int32_t* e = nullptr;
    int64_t* b = nullptr;
    TcBank tc;              // tensor-core layout (hi/lo int8 planes), see b2_tc.cuh
};

}  // namespace

struct b2_handle {
    b2_config cfg{};
    int device = 0, flags = 0;
    std::string err;
    std::vector<DevBank> banks;   // 4 * L + 1 (head last)
    int64_t *wte = nullptr, *wpe = nullptr;
    int32_t *PHI = nullptr, *ARR = nullptr, *LOG2 = nullptr, *EXP2 = nullptr;
    int alen = 0;
    int64_t log768 = 0, eps40 = 0;
    bool have_scalar[2] = {false, false};

    // Pythia (kind B2_PYTHIA, pythia_base2.py): the layer norms kept whole (gain g at 2^ge, offset b), ln1.l at 2l,
    // ln2.l at 2l + 1, lnf at 2L; the turn tables [n_ctx][rot/2] at 2^-30; the score's half power; the word rows
    // (embed.w, one power of two per word in embed.e) held on the host until b2_finalize puts them on the 2^-16 scale
    struct Norm {
        int64_t *g = nullptr, *b = nullptr;
        int64_t ge = 0;
        bool have_ge = false;
    };
    std::vector<Norm> norms;
    int32_t *COS = nullptr, *SIN = nullptr;
    double *cosf = nullptr, *sinf = nullptr;   // turn=float: float64 cos/sin of pos * 10000^(-2i/rot), [n_ctx][rot/2]
    double* sigf = nullptr;                    // gauge=float (GPT-2): per row sqrt(var + 1e-5) [max_rows]
    int64_t* qraw = nullptr;                   // arrival=float (Pythia): turned queries at full width [max_rows][d]
    int64_t cs_len = 0, half = 0, rot = 0;
    bool have_half = false, have_rot = false;
    std::vector<int64_t> emb_w, emb_e;
    bool finalized = false;
    int use_tc = 1;               // tensor-core bank product for row counts >= tc_min_rows
    int tc_min_rows = 1 << 30;    // (set at finalize when the tensor path is available)

    // stream slots + key/value store
    int n_slots = 0, max_ctx = 0;
    KV kv{};
    int32_t *slot_len = nullptr, *slot_tok = nullptr;
    bool primed = false;

    // row buffers
    int max_rows = 0;
    int32_t *row_slot = nullptr, *row_pos = nullptr, *row_tok = nullptr;
    int64_t *R = nullptr, *QKV = nullptr, *ATT = nullptr, *HID = nullptr;
    int64_t* G2 = nullptr;       // Pythia decode: the second norm's rows ([FUSED_ROWS][d])
    int32_t *x16 = nullptr, *ex = nullptr, *q16 = nullptr, *qexp = nullptr;
    int64_t* LS = nullptr;
    TcRows tcr{};
    int32_t *head_rows = nullptr, *race_out = nullptr;
    uint64_t* row_or = nullptr;  // decode: per bank input, the OR of |x| over each row ([4L][FUSED_ROWS])
    int64_t* wq_acc = nullptr;   // decode, rows quantised in the bank kernels: S1, S2 per bank input ([2][4L][FUSED_ROWS])
    int32_t* wq_nsat = nullptr;  // the +32768 count per bank input ([4L][FUSED_ROWS])
    unsigned long long* wq_ctr = nullptr;   // arrival counters per bank input and row half ([4L][2], never reset)
    int wq = 1;                  // decode steps of <= 64 streams quantise in the bank kernels (B2_WQ=0: quant kernels)
    PrefillBlock* pf_blocks = nullptr;   // prompt pass: blocks of consecutive positions of one stream [max_rows]
    int pf_qb = 0;                       // queries per block (16 or 8, by the context's shared memory; 0: per-row)
    int att_bulk = 1;            // the arrival by bulk copies into shared memory (B2_ATT_BULK=0: per-warp loads)
    int early_keys = 1;          // decode arrival: earlier positions' keys copied before the dependency wait (B2_EARLY_KEYS=0)
    int att_split = 1;           // few (row, head) units with long contexts: keys split over a cluster (B2_ATT_SPLIT=0)
    int qkv_unsplit = 0;         // decode qkv banks on one CTA per tile (set per stream allocation, B2_QKV_PAIR=1: never):
                                 // with many rows the arrival that follows runs one CTA per (row, head) and starts on
                                 // the SMs a CTA-pair qkv would hold
    int qkv_pair = 0;            // B2_QKV_PAIR=1
    int gemv_head = 1;           // decode heads at <= 2 rows on the CUDA-core GEMV head (B2_GEMV_HEAD=0: the tile head)
    // the collapsing top read (b2_set_scalar "top_read" 1): decode steps of <= TOPFR_ROWS streams that store no scores
    int top_fr = 0;
    int entry = 0;                  // "entry_tables" 1: layer 0's qkv bank of a decode step from stored rows
    int64_t* entry_w = nullptr;     // [vocab][3d] = wte . W(qkv.0), built at the first b2_alloc_streams after finalize
    int64_t* entry_p = nullptr;     // [n_ctx][3d] = wpe . W(qkv.0)
    int64_t *fr_C = nullptr, *fr_HIS = nullptr, *fr_p5v = nullptr, *fr_sv = nullptr;
    int32_t *fr_p5i = nullptr, *fr_list = nullptr, *fr_cnt = nullptr, *fr_si = nullptr;
    int sms = 148;               // the device's SM count
    int fuse_heads = 1;          // GPT-2 decode: heads16 in the qkv bank's epilogue (B2_FUSE_HEADS=0: its own kernel)
    uint64_t* split_trace = nullptr;  // B2_SPLIT_TRACE=<file>: the split-K bank kernels' stamps of the last step
    uint64_t* att_trace = nullptr;    // B2_ATT_TRACE=<file>: the decode arrival's stamps of the last step ([L][CTA][8])
    std::string att_trace_path;
    std::string split_trace_path;
    int split_idx = 0;                // split-K launches so far in this step
    int64_t* logits = nullptr;   // [n_slots][vocab]
    int64_t* race_v = nullptr;   // decode: the head epilogue's race winners per row and 32-column group
    int32_t* race_i = nullptr;
    int race_ld = 0;
    int want_logits = 1;         // this call's decode steps store the logits (a caller asked for them)
    uint32_t* d_err = nullptr;
    std::vector<void*> allocs;

    // decode steps: where the words go (device descriptor), programmatic launches, the captured step graph
    GenDesc* gen_desc = nullptr;
    int32_t* gen_base = nullptr;
    int pdl = 1;
    int use_graph = 1;
    cudaStream_t cap_stream = nullptr;
    struct StepGraph {
        int n = 0;
        int want_logits = 0;
        cudaGraphExec_t exec = nullptr;
        int64_t cnt[B2_PROF_N] = {0};
    } graph;

    // b2_profile mode 2: start stamps per launch, slots [class][STAMP_PER_CLASS] (device), the per-class summed
    // durations and counts ([B2_PROF_N][2], device), the next free slot of each class in the current unit of work
    uint64_t* stamp_slots = nullptr;
    uint64_t* stamp_tot = nullptr;
    int stamp_next[B2_PROF_N] = {0};

    // launch accounting / per-class event timing (b2_profile mode 1) or in-kernel stamps (mode 2)
    struct Prof {
        int timing = 0;
        int64_t launches = 0;
        int64_t cnt[B2_PROF_N] = {0};
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev[B2_PROF_N];
        std::vector<cudaEvent_t> pool;
    } prof;
};

namespace {

constexpr int FUSED_ROWS = 64;
constexpr size_t ATT_BULK_MAX = 200 * 1024;   // shared memory the bulk-copy arrival may take
constexpr int ATT_NW = 8;                      // warps per (row, head) CTA of the bulk-copy arrival
constexpr int ATT_CS = 8;                      // CTAs per (row, head) cluster when the arrival splits the keys
constexpr size_t PF_SMEM_MAX = 200 * 1024;    // and the prompt pass's query-block arrival
constexpr int SPLIT_TRACE_LAUNCHES = 64, SPLIT_TRACE_SLOT = 160 * 8;   // B2_SPLIT_TRACE: launches x (CTAs x stamps)

int fail(b2_handle* h, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (h) h->err = buf;
    return code;
}

#define CK(call)                                                                                    \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) return fail(h, B2_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

template <class T>
int dalloc(b2_handle* h, T** p, size_t n) {
    void* q = nullptr;
    if (n == 0) n = 1;
    cudaError_t e = cudaMalloc(&q, n * sizeof(T));
    if (e != cudaSuccess) return fail(h, B2_ERR_NOMEM, "cudaMalloc(%zu bytes): %s", n * sizeof(T), cudaGetErrorString(e));
    h->allocs.push_back(q);
    *p = (T*)q;
    return B2_OK;
}

void dfree(b2_handle* h, void* p) {
    if (!p) return;
    for (size_t i = 0; i < h->allocs.size(); i++)
        if (h->allocs[i] == p) { h->allocs.erase(h->allocs.begin() + i); break; }
    cudaFree(p);
}

void drop_graph(b2_handle* h) {
    if (h->graph.exec) cudaGraphExecDestroy(h->graph.exec);
    h->graph = b2_handle::StepGraph{};
}

int bank_index(const b2_handle* h, const char* name) {
    if (!strcmp(name, "head")) return 4 * h->cfg.n_layer;
    static const char* kinds[4] = {"qkv", "proj", "fc", "mproj"};
    for (int k = 0; k < 4; k++) {
        size_t n = strlen(kinds[k]);
        if (!strncmp(name, kinds[k], n) && name[n] == '.') {
            int l = atoi(name + n + 1);
            if (l >= 0 && l < h->cfg.n_layer) return 4 * l + k;
        }
    }
    return -1;
}

// Pythia norm names: "ln1.<l>.<part>", "ln2.<l>.<part>", "lnf.<part>" -> index (2l, 2l + 1, 2L) and the part
int norm_index(const b2_handle* h, const char* name, const char** part) {
    if (h->cfg.kind != B2_PYTHIA) return -1;
    if (!strncmp(name, "lnf.", 4)) { *part = name + 4; return 2 * h->cfg.n_layer; }
    if (strncmp(name, "ln", 2) || (name[2] != '1' && name[2] != '2') || name[3] != '.') return -1;
    char* end = nullptr;
    long l = strtol(name + 4, &end, 10);
    if (end == name + 4 || *end != '.' || l < 0 || l >= h->cfg.n_layer) return -1;
    *part = end + 1;
    return 2 * (int)l + (name[2] - '1');
}

int upload_table32(b2_handle* h, int32_t** dst, const int64_t* src, int64_t n, const char* name) {
    std::vector<int32_t> t((size_t)n);
    for (int64_t i = 0; i < n; i++) {
        if (src[i] < INT32_MIN || src[i] > INT32_MAX) return fail(h, B2_ERR_VALUE, "table %s[%lld] does not fit int32", name, (long long)i);
        t[i] = (int32_t)src[i];
    }
    if (*dst) dfree(h, *dst);
    int rc = dalloc(h, dst, (size_t)n);
    if (rc) return rc;
    CK(cudaMemcpy(*dst, t.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice));
    return B2_OK;
}

int check_launch(b2_handle* h, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(h, B2_ERR_CUDA, "launch %s: %s", what, cudaGetErrorString(e));
    return B2_OK;
}

// every kernel launch goes through these: a launch count per class and, when timing, a pair of events around it
cudaEvent_t prof_event(b2_handle* h) {
    if (!h->prof.pool.empty()) { cudaEvent_t e = h->prof.pool.back(); h->prof.pool.pop_back(); return e; }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}
void prof_begin(b2_handle* h, int cls, cudaStream_t st, int n = 1) {
    h->prof.launches += n;
    h->prof.cnt[cls] += n;
    if (h->prof.timing == 1) {
        cudaEvent_t a = prof_event(h), b = prof_event(h);
        cudaEventRecord(a, st);
        h->prof.ev[cls].push_back({a, b});
    }
}
void prof_end(b2_handle* h, int cls, cudaStream_t st) {
    if (h->prof.timing == 1) cudaEventRecord(h->prof.ev[cls].back().second, st);
}

// mode 2: the stamp slot of the next launch of class cls (nullptr when not stamping or out of slots)
constexpr int STAMP_PER_CLASS = 4096;
uint64_t* stamp_slot(b2_handle* h, int cls) {
    if (h->prof.timing != 2 || !h->stamp_slots || h->stamp_next[cls] >= STAMP_PER_CLASS) return nullptr;
    return h->stamp_slots + (size_t)cls * STAMP_PER_CLASS + h->stamp_next[cls]++;
}

// every launch: counted per class, bracketed by events when timing, programmatic (PDL) unless timing
template <typename... KArgs, typename... Args>
int launch(b2_handle* h, int cls, const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t st, Args... args) {
    prof_begin(h, cls, st);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = (h->pdl && h->prof.timing != 1) ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ((KArgs)args)...);
    prof_end(h, cls, st);
    if (e != cudaSuccess) return fail(h, B2_ERR_CUDA, "launch %s: %s", what, cudaGetErrorString(e));
    return B2_OK;
}

// mode 2: a unit of work (decode step, prompt-pass chunk) clears its slots first and turns them into per-class
// durations last (k_stamp_reset / k_stamp_accum)
int stamp_open(b2_handle* h, cudaStream_t st) {
    if (h->prof.timing != 2 || !h->stamp_slots) return B2_OK;
    for (int c = 0; c < B2_PROF_N; c++) h->stamp_next[c] = 0;
    return launch(h, B2_PROF_OTHER, "stamp_reset", k_stamp_reset, 1, 1024, 0, st, h->stamp_slots,
                  (int)(B2_PROF_N * STAMP_PER_CLASS));   // (a few microseconds: outside every stamped duration)
}
int stamp_close(b2_handle* h, cudaStream_t st) {
    if (h->prof.timing != 2 || !h->stamp_slots) return B2_OK;
    StampUse use{};
    for (int c = 0; c < B2_PROF_N; c++) use.n[c] = h->stamp_next[c];
    return launch(h, B2_PROF_OTHER, "stamp_accum", k_stamp_accum, 1, 1024, 0, st, (const uint64_t*)h->stamp_slots, use,
                  STAMP_PER_CLASS, h->stamp_tot);
}

// the float stages (B2_*_FLOAT) that bank bi's epilogue takes: GPT-2's gauged banks and head (gauge), its fc (tanh
// bend); Pythia's fc (erf bend; Pythia's float gauge is its own norm kernel)
int bank_float_stages(const b2_handle* h, int bi) {
    const int f = h->flags, head = bi == 4 * h->cfg.n_layer, kind = bi % 4;
    if (!f) return 0;
    if (h->cfg.kind == B2_PYTHIA) return (!head && kind == 2 && (f & B2_EDGE_FLOAT)) ? FE_EDGE_ERF : 0;
    int r = 0;
    if (f & B2_GAUGE_FLOAT) r |= head ? FE_GAUGE_HEAD : (kind == 0 || kind == 2) ? FE_GAUGE : 0;
    if ((f & B2_EDGE_FLOAT) && !head && kind == 2) r |= FE_EDGE_TANH;
    return r;
}

// ---- one bank over `rows` rows whose x16/ex/LS are ready -------------------------------------------------------------
// heads (GPT-2's qkv): the split-K decode kernel may do heads16 in its epilogue; *heads_done says whether it did
int run_bank(b2_handle* h, int bi, int epi, int rows, int64_t* out, int ldo, const int32_t* out_map, cudaStream_t st,
             const TcHeads* heads = nullptr, bool* heads_done = nullptr, const TcQuant* quant = nullptr,
             uint64_t* or_out = nullptr, const TcRace* race = nullptr) {
    const DevBank& bk = h->banks[bi];
    if (heads_done) *heads_done = false;
    if (h->use_tc && rows >= h->tc_min_rows && bk.tc.ready) {
        prof_begin(h, B2_PROF_BANK, st);
        uint64_t* tr = nullptr;
        if (h->split_trace && h->split_idx < SPLIT_TRACE_LAUNCHES) tr = h->split_trace + (size_t)h->split_idx * SPLIT_TRACE_SLOT;
        int rc = tc_bank(bk.tc, h->tcr, epi, rows, h->ex, h->LS, bk.e, bk.b, out, ldo, out_map, h->EXP2, h->PHI, st,
                         h->pdl && h->prof.timing != 1, heads, heads_done, tr, quant, or_out, race,
                         stamp_slot(h, B2_PROF_BANK));
        h->split_idx++;
        prof_end(h, B2_PROF_BANK, st);
        if (rc) return fail(h, B2_ERR_CUDA, "tensor-core bank %d: %s", bi, cudaGetErrorString((cudaError_t)rc));
        return check_launch(h, "tc_bank");
    }
    if (quant || or_out || race) return fail(h, B2_ERR_STATE, "bank %d: this epilogue needs the tensor-core banks", bi);
    BankArgs a{h->x16, bk.w, bk.nin, bk.nout, rows, {h->ex, h->LS, bk.e, bk.b, out, ldo, out_map, h->EXP2, h->PHI}};
    a.flt = bank_float_stages(h, bi);
    a.sig = h->sigf;
    constexpr int RT = 8;
    dim3 grid((bk.nout + 255) / 256, (rows + RT - 1) / RT);
    switch (epi) {
        case EPI_GAUGED: return launch(h, B2_PROF_BANK, "bank_simt", k_bank_simt<EPI_GAUGED, RT>, grid, 256, 0, st, a);
        case EPI_GAUGED_EDGE: return launch(h, B2_PROF_BANK, "bank_simt", k_bank_simt<EPI_GAUGED_EDGE, RT>, grid, 256, 0, st, a);
        case EPI_PLAIN_ADD: return launch(h, B2_PROF_BANK, "bank_simt", k_bank_simt<EPI_PLAIN_ADD, RT>, grid, 256, 0, st, a);
        case EPI_PLAIN_EDGE: return launch(h, B2_PROF_BANK, "bank_simt", k_bank_simt<EPI_PLAIN_EDGE, RT>, grid, 256, 0, st, a);
        default: return launch(h, B2_PROF_BANK, "bank_simt", k_bank_simt<EPI_PLAIN_OUT, RT>, grid, 256, 0, st, a);
    }
}

int run_quant_int(b2_handle* h, const int64_t* X, int n, const int32_t* src_rows, int rows, int gauge, cudaStream_t st);

// to16 (+ the gauge) of rows; with gauge=float (GPT-2) the rows' sigma as well (base2.py:67)
int run_quant(b2_handle* h, const int64_t* X, int n, const int32_t* src_rows, int rows, int gauge, cudaStream_t st) {
    int rc = run_quant_int(h, X, n, src_rows, rows, gauge, st);
    if (rc || !gauge || !(h->flags & B2_GAUGE_FLOAT) || h->cfg.kind != B2_GPT2) return rc;
    return launch(h, B2_PROF_QUANT, "sigma", k_sigma<256>, rows, 256, 0, st, X, n, src_rows, rows, h->sigf);
}

int run_quant_int(b2_handle* h, const int64_t* X, int n, const int32_t* src_rows, int rows, int gauge, cudaStream_t st) {
    PlaneOut pl{};
    if (h->use_tc && rows >= h->tc_min_rows)
        pl = PlaneOut{h->tcr.xh, h->tcr.xl, h->tcr.kmax, h->tcr.rowcorr, h->tcr.nsat, h->tcr.sat};
    pl.stamp = stamp_slot(h, B2_PROF_QUANT);
    if (n > 1024)
        return launch(h, B2_PROF_QUANT, "quant", k_quant<512>, rows, 512, 0, st, X, n, src_rows, rows, h->x16, h->ex, h->LS,
                      gauge, h->LOG2, h->log768, h->eps40, pl);
    return launch(h, B2_PROF_QUANT, "quant", k_quant<256>, rows, 256, 0, st, X, n, src_rows, rows, h->x16, h->ex, h->LS,
                  gauge, h->LOG2, h->log768, h->eps40, pl);
}

// the arrival for `rows` rows at layer l: in a prompt pass (blocks given) query blocks sharing key/value tiles;
// otherwise one CTA per (row, head), by bulk copies while a stream's keys fit in shared memory
int run_attend(b2_handle* h, int rows, int l, uint64_t* or_out, cudaStream_t st, int nblocks = 0, bool decode = false) {
    AttnArgs aa{h->row_slot, h->row_pos, rows, l, h->kv, h->q16, h->qexp, h->ARR, h->alen, h->LOG2, h->EXP2, h->ATT, h->d_err,
                or_out, h->half};
    aa.early = decode && h->early_keys;
    aa.stamp = stamp_slot(h, B2_PROF_ATTEND);
    const bool py = h->cfg.kind == B2_PYTHIA;
    const dim3 grid(rows, h->cfg.n_head);
    if (nblocks > 0 && h->pf_qb && !(h->flags & B2_ARRIVAL_FLOAT)) {
        const dim3 g(nblocks, h->cfg.n_head);
        const size_t sm = prefill_smem(h->pf_qb, h->max_ctx);
        const PrefillBlock* bl = h->pf_blocks;
        const int nkm = h->max_ctx;
        if (h->pf_qb == 16)
            return py ? launch(h, B2_PROF_ATTEND, "attend_prefill", k_attend_prefill<16, true>, g, 256, sm, st, aa, bl, nkm)
                      : launch(h, B2_PROF_ATTEND, "attend_prefill", k_attend_prefill<16, false>, g, 256, sm, st, aa, bl, nkm);
        return py ? launch(h, B2_PROF_ATTEND, "attend_prefill", k_attend_prefill<8, true>, g, 256, sm, st, aa, bl, nkm)
                  : launch(h, B2_PROF_ATTEND, "attend_prefill", k_attend_prefill<8, false>, g, 256, sm, st, aa, bl, nkm);
    }
    if (h->flags & B2_ARRIVAL_FLOAT) {
        aa.qf = py ? h->qraw : h->QKV;                    // GPT-2: q is the first third of the qkv row
        aa.ldq = py ? h->cfg.d_model : 3 * h->cfg.d_model;
        return launch(h, B2_PROF_ATTEND, "attend_float", k_attend_float, grid, 64, sizeof(double) * h->max_ctx, st, aa);
    }
    const size_t bulk = (size_t)((h->max_ctx + 3) & ~3) * ATT_BYTES_PER_KEY;
    // few (row, head) units with long contexts: each unit's keys split over a cluster of ATT_CS CTAs, so the launch
    // fills the GPU in one wave with small CTAs (their largest score and sums combined over DSMEM)
    const size_t bulk_cs = (size_t)((((h->max_ctx + ATT_CS - 1) / ATT_CS) + 3) & ~3) * ATT_BYTES_PER_KEY;
    const bool split = h->att_bulk && h->att_split && bulk_cs <= ATT_BULK_MAX &&
                       ((rows * h->cfg.n_head < 2 * h->sms && h->max_ctx >= 256) || bulk > ATT_BULK_MAX);
    if (split) {
        prof_begin(h, B2_PROF_ATTEND, st);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(rows, h->cfg.n_head, ATT_CS);
        cfg.blockDim = dim3(ATT_NW * 32);
        cfg.dynamicSmemBytes = bulk_cs;
        cfg.stream = st;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = ATT_CS;
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = (h->pdl && h->prof.timing != 1) ? 2 : 1;
        const cudaError_t e = py ? cudaLaunchKernelEx(&cfg, k_attend_bulk<ATT_NW, true, ATT_CS>, aa)
                                 : cudaLaunchKernelEx(&cfg, k_attend_bulk<ATT_NW, false, ATT_CS>, aa);
        prof_end(h, B2_PROF_ATTEND, st);
        if (e != cudaSuccess) return fail(h, B2_ERR_CUDA, "launch attend_bulk (split): %s", cudaGetErrorString(e));
        return B2_OK;
    }
    if (h->att_trace && rows <= 64) aa.trace = h->att_trace + (size_t)l * 64 * h->cfg.n_head * 8;
    if (h->att_bulk && bulk <= ATT_BULK_MAX)
        return py ? launch(h, B2_PROF_ATTEND, "attend_bulk", k_attend_bulk<ATT_NW, true, 1>, grid, ATT_NW * 32, bulk, st, aa)
                  : launch(h, B2_PROF_ATTEND, "attend_bulk", k_attend_bulk<ATT_NW, false, 1>, grid, ATT_NW * 32, bulk, st, aa);
    const size_t sm = sizeof(int64_t) * h->max_ctx;
    return py ? launch(h, B2_PROF_ATTEND, "attend", k_attend<4, true>, grid, 128, sm, st, aa)
              : launch(h, B2_PROF_ATTEND, "attend", k_attend<4, false>, grid, 128, sm, st, aa);
}

// Pythia's layer norm (pythia_base2.py:100-110) of rows of X (gathered by src_rows when given) into out [rows][d]
int run_gauge(b2_handle* h, const int64_t* X, const int32_t* src_rows, int rows, int ni, int64_t* out, cudaStream_t st,
              uint64_t* or_out = nullptr, int ni2 = -1, int64_t* out2 = nullptr, uint64_t* or_out2 = nullptr) {
    const b2_handle::Norm& nm = h->norms[ni];
    if (h->flags & B2_GAUGE_FLOAT)
        return launch(h, B2_PROF_QUANT, "gauge_ln_float", k_gauge_ln_float<256>, rows, 256, 0, st, X, h->cfg.d_model,
                      src_rows, rows, (const int64_t*)nm.g, nm.ge, (const int64_t*)nm.b, out);
    GaugeTwo two{};
    if (ni2 >= 0) {
        const b2_handle::Norm& n2 = h->norms[ni2];
        two = GaugeTwo{n2.g, n2.ge, n2.b, out2, or_out2};
    }
    return launch(h, B2_PROF_QUANT, "gauge_ln", k_gauge_ln<256>, dim3(rows, ni2 >= 0 ? 2 : 1), 256, 0, st, X, h->cfg.d_model,
                  src_rows, rows, (const int64_t*)nm.g, nm.ge, (const int64_t*)nm.b, out, (const int32_t*)h->LOG2,
                  (const int32_t*)h->EXP2, h->eps40, h->d_err, stamp_slot(h, B2_PROF_QUANT), or_out, two);
}

// Pythia's layers + head (pythia_base2.py:161-169): the parallel residual R <- R + A(g1 R) + M(g2 R). Both norms read R
// before either branch adds into it; the branch sums go into R in the order mproj, proj (wrapping int64 adds, so the
// order does not change R). Buffers: g1 R in ATT until the qkv bank has read it, g2 R in HID until the fc bank has.
int run_rows_pythia(b2_handle* h, int rows, const int32_t* hrows, const int32_t* hmap, int nhead, int64_t* logits,
                    int32_t* words_by_slot, cudaStream_t st, int nblocks) {
    const b2_config& c = h->cfg;
    const int d = c.d_model, L = c.n_layer, H = c.n_head, F = c.d_ff;
    int rc;
    if ((rc = launch(h, B2_PROF_OTHER, "embed", k_embed, rows, 256, 0, st, h->row_tok, h->row_pos, rows, h->wte,
                     (const int64_t*)nullptr, d, c.vocab, c.n_ctx, h->R, h->d_err)))
        return rc;
    for (int l = 0; l < L; l++) {
        if ((rc = run_gauge(h, h->R, nullptr, rows, 2 * l, h->ATT, st))) return rc;
        if ((rc = run_quant(h, h->ATT, d, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 0, EPI_PLAIN_OUT, rows, h->QKV, 3 * d, nullptr, st))) return rc;
        if ((rc = launch(h, B2_PROF_HEADS, "heads_pythia", k_heads_pythia, dim3(rows, 3 * H), 32, 0, st,
                         (const int64_t*)h->QKV, rows, (const int32_t*)h->row_slot, (const int32_t*)h->row_pos, l, h->kv,
                         (int)h->rot, (const int32_t*)h->COS, (const int32_t*)h->SIN, h->q16, h->qexp, h->d_err,
                         (const double*)h->cosf, (const double*)h->sinf, h->qraw, stamp_slot(h, B2_PROF_HEADS))))
            return rc;
        if ((rc = run_attend(h, rows, l, nullptr, st, nblocks))) return rc;
        if ((rc = run_gauge(h, h->R, nullptr, rows, 2 * l + 1, h->HID, st))) return rc;
        if ((rc = run_quant(h, h->HID, d, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 2, EPI_PLAIN_EDGE, rows, h->HID, F, nullptr, st))) return rc;
        if ((rc = run_quant(h, h->HID, F, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 3, EPI_PLAIN_ADD, rows, h->R, d, nullptr, st))) return rc;
        if ((rc = run_quant(h, h->ATT, d, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 1, EPI_PLAIN_ADD, rows, h->R, d, nullptr, st))) return rc;
    }
    if (nhead <= 0) return B2_OK;
    if ((rc = run_gauge(h, h->R, hrows, nhead, 2 * L, h->ATT, st))) return rc;
    if ((rc = run_quant(h, h->ATT, d, nullptr, nhead, 0, st))) return rc;
    if ((rc = run_bank(h, 4 * L, EPI_PLAIN_OUT, nhead, logits, c.vocab, hmap, st))) return rc;
    return launch(h, B2_PROF_RACE, "race", k_race, nhead, 1024, 0, st, logits, c.vocab, hmap, c.vocab, words_by_slot);
}

// ---- all layers + head for the rows in the row table --------------------------------------------------------------
// head rows: rows [0, nhead) of `hrows` (row indices) are scored; their logits go to out rows hmap (slot ids).
int run_rows(b2_handle* h, int rows, const int32_t* hrows, const int32_t* hmap, int nhead, int64_t* logits,
             int32_t* words_by_slot, cudaStream_t st, int nblocks = 0) {
    if (h->cfg.kind == B2_PYTHIA) return run_rows_pythia(h, rows, hrows, hmap, nhead, logits, words_by_slot, st, nblocks);
    const b2_config& c = h->cfg;
    const int d = c.d_model, L = c.n_layer, H = c.n_head, F = c.d_ff;
    int rc;
    if ((rc = launch(h, B2_PROF_OTHER, "embed", k_embed, rows, 256, 0, st, h->row_tok, h->row_pos, rows, h->wte, h->wpe, d,
                     c.vocab, c.n_ctx, h->R, h->d_err)))
        return rc;
    for (int l = 0; l < L; l++) {
        if ((rc = run_quant(h, h->R, d, nullptr, rows, 1, st))) return rc;
        // decode rows: heads16 in the qkv bank's epilogue where the split-K kernel runs (not with arrival=float,
        // which also needs the keys at full width)
        const TcHeads hd{h->q16, h->qexp, h->kv, h->row_slot, h->row_pos, l};
        bool heads_done = false;
        const bool want_heads = h->fuse_heads && !(h->flags & B2_ARRIVAL_FLOAT);
        if ((rc = run_bank(h, 4 * l + 0, EPI_GAUGED, rows, h->QKV, 3 * d, nullptr, st, want_heads ? &hd : nullptr,
                           &heads_done)))
            return rc;
        if (!heads_done &&
            (rc = launch(h, B2_PROF_HEADS, "heads", k_heads, dim3(rows, 3 * H), 32, 0, st, h->QKV, rows, h->row_slot,
                         h->row_pos, l, h->kv, h->q16, h->qexp, h->d_err)))
            return rc;
        if ((rc = run_attend(h, rows, l, nullptr, st, nblocks))) return rc;
        if ((rc = run_quant(h, h->ATT, d, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 1, EPI_PLAIN_ADD, rows, h->R, d, nullptr, st))) return rc;
        if ((rc = run_quant(h, h->R, d, nullptr, rows, 1, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 2, EPI_GAUGED_EDGE, rows, h->HID, F, nullptr, st))) return rc;
        if ((rc = run_quant(h, h->HID, F, nullptr, rows, 0, st))) return rc;
        if ((rc = run_bank(h, 4 * l + 3, EPI_PLAIN_ADD, rows, h->R, d, nullptr, st))) return rc;
    }
    if (nhead <= 0) return B2_OK;
    if ((rc = run_quant(h, h->R, d, hrows, nhead, 1, st))) return rc;
    if ((rc = run_bank(h, 4 * L, EPI_GAUGED, nhead, logits, c.vocab, hmap, st))) return rc;
    return launch(h, B2_PROF_RACE, "race", k_race, nhead, 1024, 0, st, logits, c.vocab, hmap, c.vocab, words_by_slot);
}

// ---- a decode step with the rows quantised inside the bank kernels (n <= 64 streams, row r = slot r) -------------
// Each bank input's row OR is published by its producer (embed, attention, the banks before: atomicOr), so the
// k_bank_wide CTAs quantise the rows themselves (shared out, then an arrival counter) instead of waiting for a
// quant kernel (the mproj bank's 24 K blocks split over 4-CTA clusters). Only the head keeps a quant kernel.
TcQuant wq_args(b2_handle* h, int site, const int64_t* X, int ldx, const uint64_t* xor_in) {
    TcQuant q;
    q.X = X;
    q.ldx = ldx;
    q.xor_in = xor_in;
    q.S1 = h->wq_acc + (size_t)site * FUSED_ROWS;
    q.S2 = h->wq_acc + (size_t)(4 * h->cfg.n_layer + site) * FUSED_ROWS;
    q.nsat = h->wq_nsat + (size_t)site * FUSED_ROWS;
    q.ctr = h->wq_ctr + (size_t)site * 2;
    q.LOG2 = h->LOG2;
    q.log768 = h->log768;
    q.eps40 = h->eps40;
    return q;
}

// the collapsing top read over the head's quantised rows (k_quant done): coarse sums and bounds of every word, T5 and
// the words still in, their exact scores, the race among them; the words by slot into race_out
constexpr int FR_PARTS = 296, FR_FIN = 148;
bool top_fr_ok(const b2_handle* h, int n) {
    const DevBank& hb = h->banks[4 * h->cfg.n_layer];
    return h->top_fr && !h->want_logits && n <= TOPFR_ROWS && hb.tc.ready && hb.nin == TOPFR_NIN && h->fr_C;
}
int run_top_fr(b2_handle* h, int n, cudaStream_t st) {
    const DevBank& hb = h->banks[4 * h->cfg.n_layer];
    TopFrArgs a{};
    a.wh = hb.tc.wh;
    a.wl = hb.tc.wl;
    a.x16 = h->x16;
    a.ex = h->ex;
    a.LS = h->LS;
    a.e = hb.e;
    a.b = hb.b;
    a.EXP2 = h->EXP2;
    a.nout = hb.nout;
    a.rows = n;
    a.C = h->fr_C;
    a.HIS = h->fr_HIS;
    a.p5v = h->fr_p5v;
    a.p5i = h->fr_p5i;
    a.nparts = FR_PARTS;
    a.list = h->fr_list;
    a.cnt = h->fr_cnt;
    a.sv = h->fr_sv;
    a.si = h->fr_si;
    a.nfin = FR_FIN;
    a.stamp = stamp_slot(h, B2_PROF_BANK);
    const bool py = h->cfg.kind == B2_PYTHIA;
    int rc = py ? launch(h, B2_PROF_BANK, "top_coarse", k_top_coarse<EPI_PLAIN_OUT>, FR_PARTS, 256, 0, st, a)
                : launch(h, B2_PROF_BANK, "top_coarse", k_top_coarse<EPI_GAUGED>, FR_PARTS, 256, 0, st, a);
    if (rc) return rc;
    a.stamp = nullptr;
    if ((rc = launch(h, B2_PROF_RACE, "top_select", k_top_select, n, 1024, 0, st, a))) return rc;
    rc = py ? launch(h, B2_PROF_RACE, "top_finish", k_top_finish<EPI_PLAIN_OUT>, dim3(FR_FIN, n), 256, 0, st, a)
            : launch(h, B2_PROF_RACE, "top_finish", k_top_finish<EPI_GAUGED>, dim3(FR_FIN, n), 256, 0, st, a);
    if (rc) return rc;
    return launch(h, B2_PROF_RACE, "race", k_race_parts, n, 256, 0, st, (const int64_t*)h->fr_sv, (const int32_t*)h->fr_si,
                  FR_FIN, FR_FIN, h->race_out);
}

// the head of a decode step of one or two rows on the CUDA-core GEMV head (its rows quantised in the kernel, the race
// in its epilogue), then the words from the 32-column winners; false when that head does not apply
bool gemv_head_ok(const b2_handle* h, int n) {
    return h->gemv_head && n <= 2 && h->banks[4 * h->cfg.n_layer].tc.map_w16_ok && !top_fr_ok(h, n);
}
int run_gemv_head(b2_handle* h, int epi, const int64_t* X, int n, cudaStream_t st) {
    const DevBank& hb = h->banks[4 * h->cfg.n_layer];
    const TcRace race{h->race_v, h->race_i, h->race_ld};
    prof_begin(h, B2_PROF_BANK, st);
    const int rc = tc_head_gemv(hb.tc, epi, X, h->cfg.d_model, n, hb.e, hb.b, h->EXP2, h->LOG2, h->log768, h->eps40, race,
                                h->want_logits ? h->logits : nullptr, h->cfg.vocab, h->d_err, h->sms, st,
                                h->pdl && h->prof.timing != 1, stamp_slot(h, B2_PROF_BANK));
    prof_end(h, B2_PROF_BANK, st);
    if (rc) return fail(h, B2_ERR_CUDA, "GEMV head: %s", cudaGetErrorString((cudaError_t)rc));
    return launch(h, B2_PROF_RACE, "race", k_race_parts, n, 256, 0, st, (const int64_t*)h->race_v,
                  (const int32_t*)h->race_i, h->race_ld, h->race_ld, h->race_out);
}

int run_decode_wq(b2_handle* h, int n, cudaStream_t st) {
    const b2_config& c = h->cfg;
    const int d = c.d_model, L = c.n_layer, F = c.d_ff;
    uint64_t* OR = h->row_or;   // slot q of the step: OR[q * FUSED_ROWS + row]
    int rc = launch(h, B2_PROF_OTHER, "embed_decode", k_embed_decode, n, 256, 0, st, n, h->slot_len, h->slot_tok,
                    h->row_slot, h->row_pos, h->row_tok, h->wte, h->wpe, d, c.vocab, c.n_ctx, h->R, OR, 4 * L, FUSED_ROWS,
                    h->wq_acc, h->wq_nsat, h->d_err);
    if (rc) return rc;
    for (int l = 0; l < L; l++) {
        uint64_t* o0 = OR + (size_t)(4 * l) * FUSED_ROWS;
        const TcHeads hd{h->q16, h->qexp, h->kv, h->row_slot, h->row_pos, l};
        bool heads_done = false;
        TcQuant q = wq_args(h, 4 * l, h->R, d, o0);
        q.unsplit = h->qkv_unsplit;
        if (l == 0 && h->entry_w) {   // layer 0's qkv from the stored rows (same bits: the pile is Tw[word] + Tp[pos])
            const DevBank& b0 = h->banks[0];
            prof_begin(h, B2_PROF_BANK, st);
            rc = tc_entry_qkv(b0.tc, h->entry_w, h->entry_p, h->row_tok, h->wte, h->wpe, c.vocab, c.n_ctx, n, b0.e, b0.b,
                              h->EXP2, q, hd, h->d_err, st, h->pdl && h->prof.timing != 1, stamp_slot(h, B2_PROF_BANK));
            prof_end(h, B2_PROF_BANK, st);
            if (rc) return fail(h, B2_ERR_CUDA, "entry qkv: %s", cudaGetErrorString((cudaError_t)rc));
            heads_done = true;
        } else if ((rc = run_bank(h, 4 * l, EPI_GAUGED, n, h->QKV, 3 * d, nullptr, st, &hd, &heads_done, &q))) {
            return rc;
        }
        if (!heads_done) return fail(h, B2_ERR_STATE, "qkv bank %d: heads16 not done in its epilogue", l);
        if ((rc = run_attend(h, n, l, o0 + FUSED_ROWS, st, 0, true))) return rc;
        q = wq_args(h, 4 * l + 1, h->ATT, d, o0 + FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 1, EPI_PLAIN_ADD, n, h->R, d, nullptr, st, nullptr, nullptr, &q, o0 + 2 * FUSED_ROWS)))
            return rc;
        q = wq_args(h, 4 * l + 2, h->R, d, o0 + 2 * FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 2, EPI_GAUGED_EDGE, n, h->HID, F, nullptr, st, nullptr, nullptr, &q,
                           o0 + 3 * FUSED_ROWS)))
            return rc;
        uint64_t* next = l + 1 < L ? o0 + 4 * FUSED_ROWS : nullptr;
        q = wq_args(h, 4 * l + 3, h->HID, F, o0 + 3 * FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 3, EPI_PLAIN_ADD, n, h->R, d, nullptr, st, nullptr, nullptr, &q, next))) return rc;
    }
    if (gemv_head_ok(h, n)) return run_gemv_head(h, EPI_GAUGED, h->R, n, st);
    if ((rc = run_quant(h, h->R, d, nullptr, n, 1, st))) return rc;
    if (top_fr_ok(h, n)) return run_top_fr(h, n, st);
    // the race inside the head's epilogue (per 32-column group), the logits stored only when the caller wants them
    const TcRace race{h->race_v, h->race_i, h->race_ld};
    if ((rc = run_bank(h, 4 * L, EPI_GAUGED, n, h->want_logits ? h->logits : nullptr, c.vocab, nullptr, st, nullptr,
                       nullptr, nullptr, nullptr, &race)))
        return rc;
    return launch(h, B2_PROF_RACE, "race", k_race_parts, n, 256, 0, st, (const int64_t*)h->race_v,
                  (const int32_t*)h->race_i, h->race_ld, h->race_ld, h->race_out);
}

// Pythia-160M (pythia_base2.py:161-169) the same way: the norms publish their rows' ORs, the four banks quantise
// their rows in the kernel and qkv's epilogue does the turn and the key/value append, so a layer is 6 launches (both
// norms, qkv + turn + key/value append, arrival, fc + bend, mproj, proj) instead of 12. The second norm's output has its own buffer (G2): fc writes its 3,072 columns into HID
// while other CTAs may still be quantising their rows of its input.
int run_decode_wq_pythia(b2_handle* h, int n, cudaStream_t st) {
    const b2_config& c = h->cfg;
    const int d = c.d_model, L = c.n_layer, H = c.n_head, F = c.d_ff;
    uint64_t* OR = h->row_or;
    int rc = launch(h, B2_PROF_OTHER, "embed_decode", k_embed_decode, n, 256, 0, st, n, h->slot_len, h->slot_tok,
                    h->row_slot, h->row_pos, h->row_tok, h->wte, (const int64_t*)nullptr, d, c.vocab, c.n_ctx, h->R, OR,
                    4 * L, FUSED_ROWS, h->wq_acc, h->wq_nsat, h->d_err);
    if (rc) return rc;
    for (int l = 0; l < L; l++) {
        uint64_t* o0 = OR + (size_t)(4 * l) * FUSED_ROWS;
        // both norms of R (one launch): g1 R -> ATT (qkv's input), g2 R -> G2 (fc's input)
        if ((rc = run_gauge(h, h->R, nullptr, n, 2 * l, h->ATT, st, o0, 2 * l + 1, h->G2, o0 + 2 * FUSED_ROWS))) return rc;
        // attention branch: qkv with the turn and the key/value append in its epilogue (or a heads kernel after it)
        // -> arrival
        TcQuant q = wq_args(h, 4 * l, h->ATT, d, o0);
        q.unsplit = h->qkv_unsplit;
        TcHeads hd{h->q16, h->qexp, h->kv, h->row_slot, h->row_pos, l};
        hd.pythia = 1;
        hd.COS = h->COS;
        hd.SIN = h->SIN;
        bool heads_done = false;
        if ((rc = run_bank(h, 4 * l + 0, EPI_PLAIN_OUT, n, h->QKV, 3 * d, nullptr, st, h->fuse_heads ? &hd : nullptr,
                           &heads_done, &q)))
            return rc;
        if (!heads_done &&
            (rc = launch(h, B2_PROF_HEADS, "heads_pythia", k_heads_pythia, dim3(n, 3 * H), 32, 0, st,
                         (const int64_t*)h->QKV, n, (const int32_t*)h->row_slot, (const int32_t*)h->row_pos, l, h->kv,
                         (int)h->rot, (const int32_t*)h->COS, (const int32_t*)h->SIN, h->q16, h->qexp, h->d_err,
                         (const double*)nullptr, (const double*)nullptr, (int64_t*)nullptr, stamp_slot(h, B2_PROF_HEADS))))
            return rc;
        if ((rc = run_attend(h, n, l, o0 + FUSED_ROWS, st, 0, true))) return rc;
        // MLP branch from the same R: fc + bend -> mproj; then both branches into R (mproj, proj)
        q = wq_args(h, 4 * l + 2, h->G2, d, o0 + 2 * FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 2, EPI_PLAIN_EDGE, n, h->HID, F, nullptr, st, nullptr, nullptr, &q,
                           o0 + 3 * FUSED_ROWS)))
            return rc;
        q = wq_args(h, 4 * l + 3, h->HID, F, o0 + 3 * FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 3, EPI_PLAIN_ADD, n, h->R, d, nullptr, st, nullptr, nullptr, &q))) return rc;
        q = wq_args(h, 4 * l + 1, h->ATT, d, o0 + FUSED_ROWS);
        if ((rc = run_bank(h, 4 * l + 1, EPI_PLAIN_ADD, n, h->R, d, nullptr, st, nullptr, nullptr, &q))) return rc;
    }
    if ((rc = run_gauge(h, h->R, nullptr, n, 2 * L, h->ATT, st))) return rc;
    if (gemv_head_ok(h, n)) return run_gemv_head(h, EPI_PLAIN_OUT, h->ATT, n, st);
    if ((rc = run_quant(h, h->ATT, d, nullptr, n, 0, st))) return rc;
    if (top_fr_ok(h, n)) return run_top_fr(h, n, st);
    const TcRace race{h->race_v, h->race_i, h->race_ld};
    if ((rc = run_bank(h, 4 * L, EPI_PLAIN_OUT, n, h->want_logits ? h->logits : nullptr, c.vocab, nullptr, st, nullptr,
                       nullptr, nullptr, nullptr, &race)))
        return rc;
    return launch(h, B2_PROF_RACE, "race", k_race_parts, n, 256, 0, st, (const int64_t*)h->race_v,
                  (const int32_t*)h->race_i, h->race_ld, h->race_ld, h->race_out);
}

bool wq_pythia_ok(const b2_handle* h, int n) {
    const b2_config& c = h->cfg;
    if (!(h->wq && c.kind == B2_PYTHIA && h->use_tc && h->tc_min_rows <= 1 && n <= FUSED_ROWS && !h->flags))
        return false;
    for (int bi = 0; bi < 4 * c.n_layer; bi++)
        if (!wide_fits(h->banks[bi].tc, n)) return false;
    return true;
}

bool wq_ok(const b2_handle* h, int n) {
    const b2_config& c = h->cfg;
    if (!(h->wq && c.kind == B2_GPT2 && h->use_tc && h->tc_min_rows <= 1 && n <= FUSED_ROWS && !h->flags &&
          h->fuse_heads))
        return false;
    for (int bi = 0; bi < 4 * c.n_layer; bi++)
        if (!wide_fits(h->banks[bi].tc, n)) return false;
    return true;
}

int ensure_ready(b2_handle* h) {
    if (!h) return B2_ERR_ARG;
    if (!h->finalized) return fail(h, B2_ERR_STATE, "b2_finalize has not been called");
    if (!h->n_slots) return fail(h, B2_ERR_STATE, "b2_alloc_streams has not been called");
    CK(cudaSetDevice(h->device));
    return B2_OK;
}

int read_device_error(b2_handle* h) {
    uint32_t e = 0;
    CK(cudaMemcpy(&e, h->d_err, sizeof e, cudaMemcpyDeviceToHost));
    if (!e) return B2_OK;
    CK(cudaMemset(h->d_err, 0, sizeof(uint32_t)));
    if (e & DERR_POS) return fail(h, B2_ERR_CTX, "a position passed the context (device check, bits 0x%x)", e);
    if (e & DERR_VOVF) return fail(h, B2_ERR_VALUE, "a value-store entry did not fit int32 (device check, bits 0x%x)", e);
    if (e & DERR_INDEX) return fail(h, B2_ERR_VALUE, "an arrival index fell below the table (device check, bits 0x%x)", e);
    if (e & DERR_TIMEOUT) {
        // some CTAs of a quantising bank never arrived: its counters are out of step with the launches, so they start
        // again from zero (nothing is in flight: every caller synchronised before reading the error word)
        if (h->wq_ctr) CK(cudaMemset(h->wq_ctr, 0, sizeof(unsigned long long) * 4 * h->cfg.n_layer * 2));
        return fail(h, B2_ERR_DEVICE, "a device kernel's bounded wait gave up (device check, bits 0x%x)", e);
    }
    if (e & DERR_RANGE)
        return fail(h, B2_ERR_VALUE, "a value passed the range the reference asserts (turn input >= 2^31, a power or the "
                    "arrival's sum past int64; device check, bits 0x%x)", e);
    return fail(h, B2_ERR_DEVICE, "a token id was out of range (device check, bits 0x%x)", e);
}

}  // namespace

// =====================================================================================================================
// C ABI
// =====================================================================================================================
extern "C" {

int b2_abi_version(void) { return B2_ABI_VERSION; }

const char* b2_last_error(const b2_handle* h) { return h ? h->err.c_str() : "null handle"; }

int b2_create(const b2_config* cfg, int device, int flags, b2_handle** out) {
    if (!cfg || !out) return B2_ERR_ARG;
    *out = nullptr;
    if (cfg->kind != B2_GPT2 && cfg->kind != B2_PYTHIA) return B2_ERR_ARG;
    if (cfg->n_layer < 1 || cfg->n_layer > 64 || cfg->n_head < 1 || cfg->d_model != cfg->n_head * 64 ||
        cfg->d_model % 256 || cfg->d_ff % 256 || cfg->vocab < 1 || cfg->n_ctx < 1)
        return B2_ERR_ARG;
    const int allowed = B2_GAUGE_FLOAT | B2_EDGE_FLOAT | B2_ARRIVAL_FLOAT | (cfg->kind == B2_PYTHIA ? B2_TURN_FLOAT : 0);
    if (flags & ~allowed) return B2_ERR_ARG;
    if (flags && cfg->d_model > FLT_MAXD) return B2_ERR_ARG;
    b2_handle* h = new b2_handle();
    h->cfg = *cfg;
    h->device = device;
    h->flags = flags;
    h->banks.resize(4 * cfg->n_layer + 1);
    if (cfg->kind == B2_PYTHIA) h->norms.resize(2 * cfg->n_layer + 1);
    if (const char* v = getenv("B2_PDL")) h->pdl = atoi(v);
    if (const char* v = getenv("B2_GRAPH")) h->use_graph = atoi(v);
    if (const char* v = getenv("B2_ATT_BULK")) h->att_bulk = atoi(v);
    if (const char* v = getenv("B2_EARLY_KEYS")) h->early_keys = atoi(v);
    if (const char* v = getenv("B2_ATT_SPLIT")) h->att_split = atoi(v);
    if (const char* v = getenv("B2_QKV_PAIR")) h->qkv_pair = atoi(v);
    if (const char* v = getenv("B2_GEMV_HEAD")) h->gemv_head = atoi(v);
    if (const char* v = getenv("B2_FUSE_HEADS")) h->fuse_heads = atoi(v);
    if (const char* v = getenv("B2_WQ")) h->wq = atoi(v);
    if (const char* v = getenv("B2_SPLIT_TRACE")) h->split_trace_path = v;
    if (const char* v = getenv("B2_ATT_TRACE")) h->att_trace_path = v;
    if (cudaSetDevice(device) != cudaSuccess) { delete h; return B2_ERR_CUDA; }
    if (cudaFuncSetAttribute(k_attend_bulk<ATT_NW, false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_BULK_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_bulk<ATT_NW, true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_BULK_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_bulk<ATT_NW, false, ATT_CS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_BULK_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_bulk<ATT_NW, true, ATT_CS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_BULK_MAX) != cudaSuccess ||
        cudaDeviceGetAttribute(&h->sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_prefill<16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_prefill<16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_prefill<8, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_attend_prefill<8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM_MAX) != cudaSuccess) {
        delete h;
        return B2_ERR_CUDA;
    }
    // the error word [0], then (as a uint64 at [2]) the bounded waits' limit in ns (0: the kernels' default)
    if (dalloc(h, &h->d_err, 4)) { delete h; return B2_ERR_NOMEM; }
    cudaMemset(h->d_err, 0, 4 * sizeof(uint32_t));
    *out = h;
    return B2_OK;
}

int b2_set_bank(b2_handle* h, const char* name, const int16_t* w, const int64_t* e, const int64_t* b, int32_t nin, int32_t nout) {
    if (!h || !name || !w || !e) return fail(h, B2_ERR_ARG, "b2_set_bank: null argument");
    CK(cudaSetDevice(h->device));
    int bi = bank_index(h, name);
    if (bi < 0) return fail(h, B2_ERR_ARG, "b2_set_bank: unknown bank '%s'", name);
    const b2_config& c = h->cfg;
    int k = bi == 4 * c.n_layer ? 4 : bi % 4;
    int want_in[5] = {c.d_model, c.d_model, c.d_model, c.d_ff, c.d_model};
    int want_out[5] = {3 * c.d_model, c.d_model, c.d_ff, c.d_model, c.vocab};
    if (nin != want_in[k] || nout != want_out[k])
        return fail(h, B2_ERR_ARG, "b2_set_bank %s: shape [%d][%d], want [%d][%d]", name, nin, nout, want_in[k], want_out[k]);
    DevBank& bk = h->banks[bi];
    if (bk.w) { dfree(h, bk.w); dfree(h, bk.e); dfree(h, bk.b); bk.w = nullptr; }
    tc_bank_free(bk.tc);
    bk.nin = nin;
    bk.nout = nout;
    int rc;
    if ((rc = dalloc(h, &bk.w, (size_t)nin * nout))) return rc;
    if ((rc = dalloc(h, &bk.e, (size_t)nout))) return rc;
    if ((rc = dalloc(h, &bk.b, (size_t)nout))) return rc;
    std::vector<int32_t> e32(nout);
    for (int j = 0; j < nout; j++) {
        if (e[j] < -200 || e[j] > 200) return fail(h, B2_ERR_VALUE, "bank %s: exponent %lld out of range", name, (long long)e[j]);
        e32[j] = (int32_t)e[j];
    }
    CK(cudaMemcpy(bk.w, w, sizeof(int16_t) * (size_t)nin * nout, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(bk.e, e32.data(), sizeof(int32_t) * nout, cudaMemcpyHostToDevice));
    if (b) CK(cudaMemcpy(bk.b, b, sizeof(int64_t) * nout, cudaMemcpyHostToDevice));
    else CK(cudaMemset(bk.b, 0, sizeof(int64_t) * nout));   // no bias (Pythia's head, pythia_base2.py:56)
    h->finalized = false;
    return B2_OK;
}

int b2_set_bank_layout(b2_handle* h, const char* name, const int8_t* wh, const int8_t* wl, const int64_t* colcorr,
                       const int64_t* colcorr_kb) {
    if (!h || !name || !wh || !wl || !colcorr || !colcorr_kb) return fail(h, B2_ERR_ARG, "b2_set_bank_layout: null argument");
    CK(cudaSetDevice(h->device));
    const int bi = bank_index(h, name);
    if (bi < 0) return fail(h, B2_ERR_ARG, "b2_set_bank_layout: unknown bank '%s'", name);
    DevBank& bk = h->banks[bi];
    if (!bk.w) return fail(h, B2_ERR_STATE, "b2_set_bank_layout %s: b2_set_bank first", name);
    if (h->flags) return fail(h, B2_ERR_STATE, "b2_set_bank_layout: a handle with float stages has no tensor-core layout");
    const int rc = tc_bank_upload(bk.tc, bk.nin, bk.nout, wh, wl, colcorr, colcorr_kb);
    if (rc) return fail(h, B2_ERR_CUDA, "b2_set_bank_layout %s: %s", name, cudaGetErrorString((cudaError_t)rc));
    h->finalized = false;
    return B2_OK;
}

int b2_get_bank_layout(b2_handle* h, const char* name, int8_t* wh, int8_t* wl, int64_t* colcorr, int64_t* colcorr_kb) {
    if (!h || !name || !wh || !wl || !colcorr || !colcorr_kb) return fail(h, B2_ERR_ARG, "b2_get_bank_layout: null argument");
    CK(cudaSetDevice(h->device));
    const int bi = bank_index(h, name);
    if (bi < 0) return fail(h, B2_ERR_ARG, "b2_get_bank_layout: unknown bank '%s'", name);
    if (!h->finalized || !h->banks[bi].tc.ready) return fail(h, B2_ERR_STATE, "b2_get_bank_layout %s: no tensor-core layout", name);
    const int rc = tc_bank_download(h->banks[bi].tc, wh, wl, colcorr, colcorr_kb);
    if (rc) return fail(h, B2_ERR_CUDA, "b2_get_bank_layout %s: %s", name, cudaGetErrorString((cudaError_t)rc));
    return B2_OK;
}

int b2_set_array(b2_handle* h, const char* name, const int64_t* data, int64_t n) {
    if (!h || !name || !data || n <= 0) return fail(h, B2_ERR_ARG, "b2_set_array: bad argument");
    CK(cudaSetDevice(h->device));
    const b2_config& c = h->cfg;
    int rc;
    if (!strcmp(name, "wte") || !strcmp(name, "wpe")) {
        int64_t want = (int64_t)(name[1] == 't' ? c.vocab : c.n_ctx) * c.d_model;
        if (n != want) return fail(h, B2_ERR_ARG, "%s: %lld values, want %lld", name, (long long)n, (long long)want);
        int64_t** dst = name[1] == 't' ? &h->wte : &h->wpe;
        if (*dst) dfree(h, *dst);
        if ((rc = dalloc(h, dst, (size_t)n))) return rc;
        CK(cudaMemcpy(*dst, data, sizeof(int64_t) * n, cudaMemcpyHostToDevice));
    } else if (!strcmp(name, "phi") || !strcmp(name, "log2") || !strcmp(name, "exp2")) {
        if (n != 65536) return fail(h, B2_ERR_ARG, "%s: %lld entries, want 65536", name, (long long)n);
        int32_t** dst = name[0] == 'p' ? &h->PHI : (name[0] == 'l' ? &h->LOG2 : &h->EXP2);
        if ((rc = upload_table32(h, dst, data, n, name))) return rc;
    } else if (!strcmp(name, "arrival")) {
        if (n > (1 << 24)) return fail(h, B2_ERR_ARG, "arrival: too long");
        if ((rc = upload_table32(h, &h->ARR, data, n, name))) return rc;
        h->alen = (int)n;
    } else if (c.kind == B2_PYTHIA && (!strcmp(name, "cos") || !strcmp(name, "sin"))) {
        if (n % c.n_ctx) return fail(h, B2_ERR_ARG, "%s: %lld values, want n_ctx (%d) x rot/2", name, (long long)n, c.n_ctx);
        if ((rc = upload_table32(h, name[0] == 'c' ? &h->COS : &h->SIN, data, n, name))) return rc;
        h->cs_len = n;
    } else if (c.kind == B2_PYTHIA && (!strcmp(name, "embed.w") || !strcmp(name, "embed.e"))) {
        const bool rows = name[6] == 'w';
        const int64_t want = rows ? (int64_t)c.vocab * c.d_model : c.vocab;
        if (n != want) return fail(h, B2_ERR_ARG, "%s: %lld values, want %lld", name, (long long)n, (long long)want);
        (rows ? h->emb_w : h->emb_e).assign(data, data + n);
    } else if (const char* part = nullptr; norm_index(h, name, &part) >= 0 && (!strcmp(part, "g") || !strcmp(part, "b"))) {
        if (n != c.d_model) return fail(h, B2_ERR_ARG, "%s: %lld values, want %d", name, (long long)n, c.d_model);
        b2_handle::Norm& nm = h->norms[norm_index(h, name, &part)];
        int64_t** dst = part[0] == 'g' ? &nm.g : &nm.b;
        if (*dst) dfree(h, *dst);
        if ((rc = dalloc(h, dst, (size_t)n))) return rc;
        CK(cudaMemcpy(*dst, data, sizeof(int64_t) * n, cudaMemcpyHostToDevice));
    } else {
        return fail(h, B2_ERR_ARG, "b2_set_array: unknown array '%s'", name);
    }
    h->finalized = false;
    return B2_OK;
}

int b2_set_scalar(b2_handle* h, const char* name, int64_t v) {
    if (!h || !name) return B2_ERR_ARG;
    if (!strcmp(name, "top_read")) {   // 0: every word's exact score, then the race; 1: the collapsing read
        if (v != 0 && v != 1) return fail(h, B2_ERR_ARG, "top_read = %lld (0 or 1)", (long long)v);
        h->top_fr = (int)v;
        drop_graph(h);
        return B2_OK;
    }
    if (!strcmp(name, "entry_tables")) {   // GPT-2: layer 0's qkv piles of a decode step from stored rows (0 or 1)
        if ((v != 0 && v != 1) || (v && h->cfg.kind != B2_GPT2))
            return fail(h, B2_ERR_ARG, "entry_tables = %lld (0 or 1, GPT-2 only)", (long long)v);
        h->entry = (int)v;
        if (!v) {
            dfree(h, h->entry_w);
            dfree(h, h->entry_p);
            h->entry_w = h->entry_p = nullptr;
        }
        drop_graph(h);
        return B2_OK;
    }
    if (!strcmp(name, "wait_ns")) {   // the bounded device waits' limit (not a model scalar: finalize state unchanged)
        if (v < 0) return fail(h, B2_ERR_ARG, "wait_ns = %lld is negative", (long long)v);
        CK(cudaSetDevice(h->device));
        CK(cudaDeviceSynchronize());
        const uint64_t u = (uint64_t)v;
        CK(cudaMemcpy(h->d_err + 2, &u, sizeof u, cudaMemcpyHostToDevice));
        return B2_OK;
    }
    const char* part = nullptr;
    const int ni = norm_index(h, name, &part);
    if (!strcmp(name, "log2_768")) { h->log768 = v; h->have_scalar[0] = true; }
    else if (!strcmp(name, "eps40")) { h->eps40 = v; h->have_scalar[1] = true; }
    else if (h->cfg.kind == B2_PYTHIA && !strcmp(name, "half_log2_hs")) { h->half = v; h->have_half = true; }
    else if (h->cfg.kind == B2_PYTHIA && !strcmp(name, "rot")) { h->rot = v; h->have_rot = true; }
    else if (ni >= 0 && !strcmp(part, "ge")) {
        if (v < -64 || v > 64) return fail(h, B2_ERR_VALUE, "%s = %lld out of range", name, (long long)v);
        h->norms[ni].ge = v;
        h->norms[ni].have_ge = true;
    } else return fail(h, B2_ERR_ARG, "b2_set_scalar: unknown scalar '%s'", name);
    h->finalized = false;
    return B2_OK;
}

namespace {
// Pythia's own arrays checked, and the word rows put on the stream's scale once: R0 = rshift(embed.w, -(embed.e + 16))
// (pythia_base2.py:163), kept as the [vocab][d] int64 table the embedding kernel reads
int finalize_pythia(b2_handle* h) {
    const b2_config& c = h->cfg;
    for (size_t i = 0; i < h->norms.size(); i++)
        if (!h->norms[i].g || !h->norms[i].b || !h->norms[i].have_ge) return fail(h, B2_ERR_STATE, "norm %zu not set", i);
    if (!h->have_rot || h->rot != 16)
        return fail(h, B2_ERR_ARG, "rot = %lld: the turn kernel takes 16 turned dims per head", (long long)h->rot);
    if (!h->have_half) return fail(h, B2_ERR_STATE, "half_log2_hs not set");
    if (!h->COS || !h->SIN || h->cs_len != (int64_t)c.n_ctx * (h->rot / 2))
        return fail(h, B2_ERR_STATE, "cos/sin missing or not [n_ctx][rot/2]");
    if (h->emb_w.empty() || h->emb_e.empty()) {
        if (h->wte) return B2_OK;    // already built by an earlier finalize
        return fail(h, B2_ERR_STATE, "embed.w / embed.e not set");
    }
    const int d = c.d_model;
    std::vector<int64_t> t((size_t)c.vocab * d);
    for (int v = 0; v < c.vocab; v++) {
        const int64_t s = h->emb_e[v] + 16;   // a left shift by s (the reference's rshift by -s)
        for (int i = 0; i < d; i++) {
            const int64_t x = h->emb_w[(size_t)v * d + i];
            int64_t y;
            if (s >= 0) {
                const uint64_t m = x < 0 ? (uint64_t)0 - (uint64_t)x : (uint64_t)x;
                if (s > 61 || (m >> (62 - s)) != 0)
                    return fail(h, B2_ERR_VALUE, "embed row %d: a value past 2^62 on the stream's scale", v);
                y = (int64_t)((uint64_t)x << s);
            } else {
                const int64_t r = -s;                 // rounded: add half, shift (|x| < 2^15, r <= 62 keeps it exact)
                if (r > 62) return fail(h, B2_ERR_VALUE, "embed row %d: exponent %lld out of range", v, (long long)h->emb_e[v]);
                y = (x + ((int64_t)1 << (r - 1))) >> r;
            }
            t[(size_t)v * d + i] = y;
        }
    }
    if (h->wte) dfree(h, h->wte);
    int rc = dalloc(h, &h->wte, t.size());
    if (rc) return rc;
    CK(cudaMemcpy(h->wte, t.data(), sizeof(int64_t) * t.size(), cudaMemcpyHostToDevice));
    std::vector<int64_t>().swap(h->emb_w);
    std::vector<int64_t>().swap(h->emb_e);
    return B2_OK;
}
}  // namespace

int b2_finalize(b2_handle* h) {
    if (!h) return B2_ERR_ARG;
    CK(cudaSetDevice(h->device));
    dfree(h, h->entry_w);             // stored rows of the old weights
    dfree(h, h->entry_p);
    h->entry_w = h->entry_p = nullptr;
    for (size_t i = 0; i < h->banks.size(); i++)
        if (!h->banks[i].w) return fail(h, B2_ERR_STATE, "bank %zu not set", i);
    if (h->cfg.kind == B2_PYTHIA) {
        int rc = finalize_pythia(h);
        if (rc) return rc;
    } else if (!h->wte || !h->wpe || !h->have_scalar[0]) {
        return fail(h, B2_ERR_STATE, "a table or scalar is missing");
    }
    if (!h->PHI || !h->ARR || !h->LOG2 || !h->EXP2 || !h->have_scalar[1])
        return fail(h, B2_ERR_STATE, "a table or scalar is missing");
    if ((h->flags & B2_TURN_FLOAT) && !h->cosf) {
        // pythia_base2.py:118-120: ang = pos * 10000^(-(0, 2, ..) / rot), cos and sin by the C library (numpy's values)
        const int r = (int)h->rot / 2, n = h->cfg.n_ctx;
        std::vector<double> c((size_t)n * r), s((size_t)n * r);
        for (int t = 0; t < r; t++) {
            const double inv = std::pow(10000.0, (double)(-2 * t) / (double)h->rot);
            for (int p = 0; p < n; p++) {
                const double ang = (double)p * inv;
                c[(size_t)p * r + t] = std::cos(ang);
                s[(size_t)p * r + t] = std::sin(ang);
            }
        }
        int rc;
        if ((rc = dalloc(h, &h->cosf, c.size())) || (rc = dalloc(h, &h->sinf, s.size()))) return rc;
        CK(cudaMemcpy(h->cosf, c.data(), sizeof(double) * c.size(), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(h->sinf, s.data(), sizeof(double) * s.size(), cudaMemcpyHostToDevice));
    }
    // tensor-core layouts of every bank (the float stages run on the CUDA-core bank kernel only)
    int tc_ok = !h->flags && tc_init() == 0;
    for (auto& bk : h->banks) {
        if (!tc_ok) break;
        if (tc_bank_build(bk.tc, bk.w, bk.nin, bk.nout)) tc_ok = 0;
    }
    CK(cudaDeviceSynchronize());
    h->tc_min_rows = tc_ok ? tc_min_rows_default() : (1 << 30);
    if (tc_ok && h->cfg.kind == B2_GPT2 && !h->flags) {
        cudaGetLastError();
        if (!h->split_trace_path.empty() && !h->split_trace) {
            const size_t n = (size_t)SPLIT_TRACE_LAUNCHES * SPLIT_TRACE_SLOT;
            if (cudaMalloc(&h->split_trace, n * sizeof(uint64_t)) != cudaSuccess) h->split_trace = nullptr;
            else cudaMemset(h->split_trace, 0, n * sizeof(uint64_t));
        }
        if (!h->att_trace_path.empty() && !h->att_trace) {
            const size_t n = (size_t)h->cfg.n_layer * 64 * h->cfg.n_head * 8;
            if (cudaMalloc(&h->att_trace, n * sizeof(uint64_t)) != cudaSuccess) h->att_trace = nullptr;
            else cudaMemset(h->att_trace, 0, n * sizeof(uint64_t));
        }
    }
    const char* env = getenv("B2_TC_MIN_ROWS");
    if (env && tc_ok) h->tc_min_rows = atoi(env);
    h->finalized = true;
    return B2_OK;
}

// the stored rows of layer 0's qkv bank (the reference's stored layer-0 entry, base2_entry.py / base2_layer0.py):
// Tw = wte . W and Tp = wpe . W as exact int64 piles, by the bank kernels themselves (plain epilogue with zero
// exponents and biases: an input row below 2^15 has shift 0, so the stored value is the pile). Valid only when every
// embedded value is below 2^15 (max|wte| + max|wpe| < 2^15); otherwise refused.
int build_entry(b2_handle* h) {
    const b2_config& c = h->cfg;
    const int d = c.d_model, n3 = 3 * d;
    const DevBank& bk = h->banks[0];
    if (c.kind != B2_GPT2 || !bk.tc.ready || bk.nin != d || bk.nout != n3)
        return fail(h, B2_ERR_STATE, "entry tables: the tensor-core qkv.0 bank is needed");
    unsigned long long* mx = nullptr;
    int rc = dalloc(h, &mx, 2);
    if (rc) return rc;
    CK(cudaMemset(mx, 0, 2 * sizeof(unsigned long long)));
    if ((rc = tc_absmax(h->wte, (size_t)c.vocab * d, mx, 0)) || (rc = tc_absmax(h->wpe, (size_t)c.n_ctx * d, mx + 1, 0))) {
        dfree(h, mx);
        return fail(h, B2_ERR_CUDA, "entry tables: %s", cudaGetErrorString((cudaError_t)rc));
    }
    unsigned long long m[2] = {0, 0};
    CK(cudaMemcpy(m, mx, sizeof m, cudaMemcpyDeviceToHost));
    dfree(h, mx);
    if (m[0] + m[1] >= 32768)
        return fail(h, B2_ERR_ARG, "entry tables: embedded values reach 2^15 (max |wte| %llu + max |wpe| %llu)", m[0], m[1]);
    int32_t* e0 = nullptr;
    int64_t* b0 = nullptr;
    if ((rc = dalloc(h, &h->entry_w, (size_t)c.vocab * n3)) || (rc = dalloc(h, &h->entry_p, (size_t)c.n_ctx * n3)) ||
        (rc = dalloc(h, &e0, n3)) || (rc = dalloc(h, &b0, n3)))
        return rc;
    CK(cudaMemset(e0, 0, sizeof(int32_t) * n3));
    CK(cudaMemset(b0, 0, sizeof(int64_t) * n3));
    const int64_t* src[2] = {h->wte, h->wpe};
    int64_t* dst[2] = {h->entry_w, h->entry_p};
    const int nrows[2] = {c.vocab, c.n_ctx};
    for (int k = 0; k < 2 && !rc; k++)
        for (int r0 = 0; r0 < nrows[k] && !rc; r0 += h->max_rows) {
            const int rows = std::min(h->max_rows, nrows[k] - r0);
            if ((rc = run_quant(h, src[k] + (size_t)r0 * d, d, nullptr, rows, 0, 0))) break;
            rc = tc_bank(bk.tc, h->tcr, EPI_PLAIN_OUT, rows, h->ex, h->LS, e0, b0, dst[k] + (size_t)r0 * n3, n3, nullptr,
                         h->EXP2, h->PHI, 0, false);
            if (rc) rc = fail(h, B2_ERR_CUDA, "entry tables: %s", cudaGetErrorString((cudaError_t)rc));
        }
    cudaError_t e = cudaDeviceSynchronize();
    dfree(h, e0);
    dfree(h, b0);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(h, B2_ERR_CUDA, "entry tables: %s", cudaGetErrorString(e));
    return read_device_error(h);
}

int b2_alloc_streams(b2_handle* h, int32_t n_streams, int32_t max_ctx) {
    if (!h) return B2_ERR_ARG;
    if (!h->finalized) return fail(h, B2_ERR_STATE, "b2_finalize has not been called");
    if (n_streams < 1 || max_ctx < 1 || max_ctx > h->cfg.n_ctx)
        return fail(h, B2_ERR_ARG, "b2_alloc_streams: n_streams %d, max_ctx %d (model n_ctx %d)", n_streams, max_ctx, h->cfg.n_ctx);
    CK(cudaSetDevice(h->device));
    const b2_config& c = h->cfg;
    // drop old stream/row buffers
    void* old[] = {h->pf_blocks, h->sigf, h->qraw, h->kv.kraw, h->row_or, h->wq_acc, h->wq_nsat, h->wq_ctr, h->fr_C, h->fr_HIS,
                   h->fr_p5v, h->fr_p5i, h->fr_list, h->fr_cnt, h->fr_sv, h->fr_si, h->G2, h->race_v,
                   h->race_i, h->kv.k, h->kv.kmask, h->kv.kexp, h->kv.v, h->slot_len, h->slot_tok, h->row_slot, h->row_pos,
                   h->row_tok, h->R, h->QKV, h->ATT, h->HID, h->x16, h->ex, h->q16, h->qexp, h->LS, h->head_rows,
                   h->race_out, h->logits};
    for (void* p : old) dfree(h, p);
    tc_rows_free(h->tcr);
    drop_graph(h);
    dfree(h, h->gen_desc);
    dfree(h, h->gen_base);
    h->n_slots = 0;
    h->sigf = nullptr;
    h->qraw = nullptr;
    h->kv.kraw = nullptr;
    h->pf_blocks = nullptr;
    const int L = c.n_layer, H = c.n_head, d = c.d_model, F = c.d_ff;
    const int ctx_stride = (max_ctx + 15) / 16 * 16;
    size_t nkv = (size_t)n_streams * L * H * ctx_stride;
    int rc;
    h->kv.L = L; h->kv.H = H; h->kv.ctx = ctx_stride; h->kv.lim = max_ctx;
    if ((rc = dalloc(h, &h->kv.k, nkv * 64))) return rc;
    if ((rc = dalloc(h, &h->kv.kmask, nkv))) return rc;
    if ((rc = dalloc(h, &h->kv.kexp, nkv))) return rc;
    if ((rc = dalloc(h, &h->kv.v, nkv * 64))) return rc;
    if ((h->flags & B2_ARRIVAL_FLOAT) && (rc = dalloc(h, &h->kv.kraw, nkv * 64))) return rc;
    if ((rc = dalloc(h, &h->row_or, (size_t)4 * L * FUSED_ROWS))) return rc;
    CK(cudaMemset(h->row_or, 0, sizeof(uint64_t) * 4 * L * FUSED_ROWS));
    if ((rc = dalloc(h, &h->wq_acc, (size_t)2 * 4 * L * FUSED_ROWS))) return rc;
    if ((rc = dalloc(h, &h->wq_nsat, (size_t)4 * L * FUSED_ROWS))) return rc;
    if ((rc = dalloc(h, &h->wq_ctr, (size_t)4 * L * 2))) return rc;
    h->race_ld = 4 * ((c.vocab + 127) / 128);
    if ((rc = dalloc(h, &h->race_v, (size_t)FUSED_ROWS * h->race_ld))) return rc;
    if ((rc = dalloc(h, &h->race_i, (size_t)FUSED_ROWS * h->race_ld))) return rc;
    if ((rc = dalloc(h, &h->G2, (size_t)FUSED_ROWS * d))) return rc;
    {
        const size_t V = (size_t)c.vocab;
        if ((rc = dalloc(h, &h->fr_C, TOPFR_ROWS * V)) || (rc = dalloc(h, &h->fr_HIS, TOPFR_ROWS * V)) ||
            (rc = dalloc(h, &h->fr_p5v, (size_t)TOPFR_ROWS * FR_PARTS * 5)) ||
            (rc = dalloc(h, &h->fr_p5i, (size_t)TOPFR_ROWS * FR_PARTS * 5)) || (rc = dalloc(h, &h->fr_list, TOPFR_ROWS * V)) ||
            (rc = dalloc(h, &h->fr_cnt, TOPFR_ROWS)) || (rc = dalloc(h, &h->fr_sv, (size_t)TOPFR_ROWS * FR_FIN)) ||
            (rc = dalloc(h, &h->fr_si, (size_t)TOPFR_ROWS * FR_FIN)))
            return rc;
    }
    CK(cudaMemset(h->wq_acc, 0, sizeof(int64_t) * 2 * 4 * L * FUSED_ROWS));
    CK(cudaMemset(h->wq_nsat, 0, sizeof(int32_t) * 4 * L * FUSED_ROWS));
    CK(cudaMemset(h->wq_ctr, 0, sizeof(unsigned long long) * 4 * L * 2));
    if ((rc = dalloc(h, &h->slot_len, n_streams))) return rc;
    if ((rc = dalloc(h, &h->gen_base, n_streams))) return rc;
    if ((rc = dalloc(h, &h->gen_desc, 1))) return rc;
    CK(cudaMemset(h->gen_desc, 0, sizeof(GenDesc)));
    if ((rc = dalloc(h, &h->slot_tok, n_streams))) return rc;
    CK(cudaMemset(h->slot_len, 0, sizeof(int32_t) * n_streams));
    CK(cudaMemset(h->slot_tok, 0, sizeof(int32_t) * n_streams));
    int mr = n_streams > 2048 ? n_streams : 2048;   // rows per pass (prompt passes are chunked to this)
    h->max_rows = mr;
    if ((rc = dalloc(h, &h->row_slot, mr)) || (rc = dalloc(h, &h->row_pos, mr)) || (rc = dalloc(h, &h->row_tok, mr))) return rc;
    if ((rc = dalloc(h, &h->pf_blocks, mr))) return rc;
    h->pf_qb = prefill_smem(16, max_ctx) <= PF_SMEM_MAX ? 16 : (prefill_smem(8, max_ctx) <= PF_SMEM_MAX ? 8 : 0);
    if ((rc = dalloc(h, &h->R, (size_t)mr * d)) || (rc = dalloc(h, &h->QKV, (size_t)mr * 3 * d)) ||
        (rc = dalloc(h, &h->ATT, (size_t)mr * d)) || (rc = dalloc(h, &h->HID, (size_t)mr * F)))
        return rc;
    if ((rc = dalloc(h, &h->x16, (size_t)mr * (F > d ? F : d))) || (rc = dalloc(h, &h->ex, mr)) ||
        (rc = dalloc(h, &h->LS, mr)) || (rc = dalloc(h, &h->q16, (size_t)mr * d)) || (rc = dalloc(h, &h->qexp, (size_t)mr * H)))
        return rc;
    if ((h->flags & B2_GAUGE_FLOAT) && (rc = dalloc(h, &h->sigf, mr))) return rc;
    if ((h->flags & B2_ARRIVAL_FLOAT) && (rc = dalloc(h, &h->qraw, (size_t)mr * d))) return rc;
    if ((rc = dalloc(h, &h->head_rows, 2 * (size_t)mr)) || (rc = dalloc(h, &h->race_out, n_streams)) ||
        (rc = dalloc(h, &h->logits, (size_t)n_streams * c.vocab)))
        return rc;
    if (h->tc_min_rows < (1 << 30)) {
        rc = tc_rows_alloc(h->tcr, mr, F > d ? F : d, h->d_err);
        if (rc) return fail(h, B2_ERR_NOMEM, "tensor-core row buffers: %s", cudaGetErrorString((cudaError_t)rc));
    }
    h->n_slots = n_streams;
    h->max_ctx = max_ctx;
    h->primed = false;
    // the decode arrival at the full stream count runs one CTA per (row, head) unless few rows with long contexts
    // split it over clusters (run_attend's rule); then qkv goes unsplit, so that arrival's CTAs find SMs while it runs
    h->qkv_unsplit = !h->qkv_pair && !(n_streams * h->cfg.n_head < 2 * h->sms && max_ctx >= 256);
    if (h->entry && !h->entry_w && h->use_tc && h->tc_min_rows < (1 << 30))
        return build_entry(h);
    return B2_OK;
}

int b2_prefill(b2_handle* h, const int32_t* ids, const int32_t* lens, int32_t n_streams, int32_t* next_tok,
               int64_t* logits, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    if (!ids || !lens || !next_tok || n_streams < 1 || n_streams > h->n_slots)
        return fail(h, B2_ERR_ARG, "b2_prefill: bad argument (n_streams %d of %d slots)", n_streams, h->n_slots);
    cudaStream_t st = (cudaStream_t)stream;
    std::vector<int32_t> hl(n_streams);
    CK(cudaMemcpyAsync(hl.data(), lens, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    size_t total = 0;
    for (int s = 0; s < n_streams; s++) {
        if (hl[s] < 1 || hl[s] > h->max_ctx) return fail(h, B2_ERR_CTX, "prompt %d has %d ids (context %d)", s, hl[s], h->max_ctx);
        total += hl[s];
    }
    // row table for all prompt rows (stream-major), then chunks of max_rows
    std::vector<int32_t> rs(total), rp(total);
    std::vector<int32_t> last_row(n_streams);
    size_t o = 0;
    for (int s = 0; s < n_streams; s++) {
        for (int p = 0; p < hl[s]; p++) { rs[o] = s; rp[o] = p; o++; }
        last_row[s] = (int32_t)(o - 1);
    }
    int32_t *d_rs = nullptr, *d_rp = nullptr;
    if ((rc = dalloc(h, &d_rs, total)) || (rc = dalloc(h, &d_rp, total))) return rc;
    int64_t* lg = logits ? logits : h->logits;
    rc = B2_OK;
    do {
        if (cudaMemcpyAsync(d_rs, rs.data(), sizeof(int32_t) * total, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_rp, rp.data(), sizeof(int32_t) * total, cudaMemcpyHostToDevice, st) != cudaSuccess) {
            rc = fail(h, B2_ERR_CUDA, "prefill row table copy");
            break;
        }
        for (size_t r0 = 0; r0 < total && !rc; r0 += h->max_rows) {
            int rows = (int)(total - r0 < (size_t)h->max_rows ? total - r0 : (size_t)h->max_rows);
            if ((rc = launch(h, B2_PROF_OTHER, "prefill_rows", k_prefill_rows, (rows + 255) / 256, 256, 0, st, (int)r0, rows,
                             d_rs, d_rp, ids, h->row_slot, h->row_pos, h->row_tok)))
                break;
            // the scored rows in this chunk: each stream's last prompt position
            std::vector<int32_t> hr, hm;
            for (int s = 0; s < n_streams; s++)
                if ((size_t)last_row[s] >= r0 && (size_t)last_row[s] < r0 + rows) { hr.push_back(last_row[s] - (int)r0); hm.push_back(s); }
            int nh = (int)hr.size();
            if (nh) {
                std::vector<int32_t> both(hr);
                both.insert(both.end(), hm.begin(), hm.end());
                if (cudaMemcpyAsync(h->head_rows, both.data(), sizeof(int32_t) * both.size(), cudaMemcpyHostToDevice, st) != cudaSuccess) {
                    rc = fail(h, B2_ERR_CUDA, "prefill head rows copy");
                    break;
                }
                // head rows must stay valid until the chunk's kernels have read them
            }
            // the arrival's query blocks: runs of up to pf_qb consecutive positions of one stream
            int nblocks = 0;
            if (h->pf_qb) {
                std::vector<PrefillBlock> bl;
                for (int i = 0; i < rows;) {
                    const size_t g = r0 + i;
                    int n = 1;
                    while (n < h->pf_qb && i + n < rows && rs[g + n] == rs[g] && rp[g + n] == rp[g] + n) n++;
                    bl.push_back(PrefillBlock{i, n, rs[g], rp[g]});
                    i += n;
                }
                nblocks = (int)bl.size();
                if (cudaMemcpyAsync(h->pf_blocks, bl.data(), sizeof(PrefillBlock) * bl.size(), cudaMemcpyHostToDevice, st) !=
                    cudaSuccess) {
                    rc = fail(h, B2_ERR_CUDA, "prefill block table copy");
                    break;
                }
            }
            rc = stamp_open(h, st);
            if (!rc) rc = run_rows(h, rows, h->head_rows, h->head_rows + nh, nh, lg, h->race_out, st, nblocks);
            if (!rc) rc = stamp_close(h, st);
            if (!rc && cudaStreamSynchronize(st) != cudaSuccess) rc = fail(h, B2_ERR_CUDA, "prefill chunk sync");
        }
    } while (0);
    cudaStreamSynchronize(st);
    dfree(h, d_rs);
    dfree(h, d_rp);
    if (rc) return rc;
    // stream state: length = prompt length, last word = the race's word
    CK(cudaMemcpyAsync(h->slot_len, lens, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToDevice, st));
    CK(cudaMemcpyAsync(h->slot_tok, h->race_out, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToDevice, st));
    CK(cudaMemcpyAsync(next_tok, h->race_out, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToDevice, st));
    CK(cudaStreamSynchronize(st));
    h->primed = true;
    return read_device_error(h);
}

namespace {
// one decode step for slots 0..n-1 (row r = slot r); words into the call's GenDesc, words by slot into race_out
int step_body(b2_handle* h, int n, cudaStream_t st) {
    if (wq_ok(h, n) || wq_pythia_ok(h, n)) {
        int rc = h->cfg.kind == B2_PYTHIA ? run_decode_wq_pythia(h, n, st) : run_decode_wq(h, n, st);
        if (rc) return rc;
        return launch(h, B2_PROF_OTHER, "decode_commit", k_decode_commit, (n + 127) / 128, 128, 0, st, n, h->race_out,
                      h->slot_len, h->slot_tok, h->gen_desc, h->gen_base);
    }
    int rc = launch(h, B2_PROF_OTHER, "decode_rows", k_decode_rows, (n + 127) / 128, 128, 0, st, n, (const int32_t*)nullptr,
                    h->slot_len, h->slot_tok, h->row_slot, h->row_pos, h->row_tok);
    if (rc) return rc;
    if ((rc = run_rows(h, n, nullptr, nullptr, n, h->logits, h->race_out, st))) return rc;
    return launch(h, B2_PROF_OTHER, "decode_commit", k_decode_commit, (n + 127) / 128, 128, 0, st, n, h->race_out,
                  h->slot_len, h->slot_tok, h->gen_desc, h->gen_base);
}
int step_core(b2_handle* h, int n, cudaStream_t st) {
    h->split_idx = 0;
    int rc = stamp_open(h, st);
    if (!rc) rc = step_body(h, n, st);
    if (!rc) rc = stamp_close(h, st);
    return rc;
}

// the step captured once per stream count (on an internal stream), then replayed
int step_graph(b2_handle* h, int n, cudaStream_t st) {
    if (h->graph.exec && (h->graph.n != n || h->graph.want_logits != h->want_logits)) drop_graph(h);
    if (!h->graph.exec) {
        if (!h->cap_stream) CK(cudaStreamCreateWithFlags(&h->cap_stream, cudaStreamNonBlocking));
        CK(cudaStreamSynchronize(st));
        int64_t before[B2_PROF_N], l0 = h->prof.launches;
        for (int c = 0; c < B2_PROF_N; c++) before[c] = h->prof.cnt[c];
        CK(cudaStreamBeginCapture(h->cap_stream, cudaStreamCaptureModeThreadLocal));
        int rc = step_core(h, n, h->cap_stream);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(h->cap_stream, &g);
        for (int c = 0; c < B2_PROF_N; c++) { h->graph.cnt[c] = h->prof.cnt[c] - before[c]; h->prof.cnt[c] = before[c]; }
        h->prof.launches = l0;
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        if (e != cudaSuccess) return fail(h, B2_ERR_CUDA, "step capture: %s", cudaGetErrorString(e));
        e = cudaGraphInstantiate(&h->graph.exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { h->graph.exec = nullptr; return fail(h, B2_ERR_CUDA, "step graph: %s", cudaGetErrorString(e)); }
        h->graph.n = n;
        h->graph.want_logits = h->want_logits;
    }
    CK(cudaGraphLaunch(h->graph.exec, st));
    for (int c = 0; c < B2_PROF_N; c++) { h->prof.cnt[c] += h->graph.cnt[c]; h->prof.launches += h->graph.cnt[c]; }
    return B2_OK;
}

// n_steps decode steps; the words of step t go to out[s * ld + t] (out may be NULL); logits of the last step copied out
int run_steps(b2_handle* h, int n, int n_steps, int32_t* out, int ld, int64_t* logits, cudaStream_t st) {
    h->want_logits = logits != nullptr;
    int rc = launch(h, B2_PROF_OTHER, "gen_begin", k_gen_begin, (n + 127) / 128, 128, 0, st, n, h->slot_len, h->gen_base,
                    h->gen_desc, out, ld);
    if (rc) return rc;
    for (int t = 0; t < n_steps; t++) {
        rc = (h->use_graph && h->prof.timing != 1) ? step_graph(h, n, st) : step_core(h, n, st);
        if (rc) return rc;
    }
    if (logits) CK(cudaMemcpyAsync(logits, h->logits, sizeof(int64_t) * n * h->cfg.vocab, cudaMemcpyDeviceToDevice, st));
    return B2_OK;
}
}  // namespace

int b2_step(b2_handle* h, const int32_t* tok_in, int32_t n_streams, int32_t* tok_out, int64_t* logits, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    if (n_streams < 1 || n_streams > h->n_slots || !tok_out) return fail(h, B2_ERR_ARG, "b2_step: bad argument");
    if (!tok_in && !h->primed) return fail(h, B2_ERR_STATE, "b2_step without tok_in before any b2_prefill");
    cudaStream_t st = (cudaStream_t)stream;
    if (tok_in) CK(cudaMemcpyAsync(h->slot_tok, tok_in, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToDevice, st));
    return run_steps(h, n_streams, 1, tok_out, 1, logits, st);
}

int b2_generate(b2_handle* h, int32_t n_streams, int32_t n_steps, int32_t* tokens_out, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    if (n_streams < 1 || n_streams > h->n_slots || n_steps < 0 || !tokens_out) return fail(h, B2_ERR_ARG, "b2_generate: bad argument");
    if (!h->primed) return fail(h, B2_ERR_STATE, "b2_generate before b2_prefill");
    return run_steps(h, n_streams, n_steps, tokens_out, n_steps, nullptr, (cudaStream_t)stream);
}

int b2_step_host(b2_handle* h, const int32_t* tok_in, int32_t n_streams, int32_t* tok_out) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    if (!tok_in || !tok_out || n_streams < 1 || n_streams > h->n_slots) return fail(h, B2_ERR_ARG, "b2_step_host: bad argument");
    cudaStream_t st = 0;
    // the words go in as each stream's last word; the race's answer comes back from race_out
    CK(cudaMemcpyAsync(h->slot_tok, tok_in, sizeof(int32_t) * n_streams, cudaMemcpyHostToDevice, st));
    if ((rc = run_steps(h, n_streams, 1, nullptr, 1, nullptr, st))) return rc;
    CK(cudaMemcpyAsync(tok_out, h->race_out, sizeof(int32_t) * n_streams, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return read_device_error(h);
}

int b2_bank(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, int32_t mode, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    int bi = bank_index(h, name);
    if (bi < 0 || !X || !out || rows < 1 || rows > h->max_rows || mode < 0 || mode > 3)
        return fail(h, B2_ERR_ARG, "b2_bank: bad argument");
    if (h->cfg.kind == B2_PYTHIA && mode < 2)
        return fail(h, B2_ERR_ARG, "b2_bank: Pythia's banks are plain (modes 2 and 3); its norm is b2_gauge");
    cudaStream_t st = (cudaStream_t)stream;
    const DevBank& bk = h->banks[bi];
    if ((rc = run_quant(h, X, bk.nin, nullptr, rows, mode < 2, st))) return rc;
    const int epi[4] = {EPI_GAUGED, EPI_GAUGED_EDGE, EPI_PLAIN_OUT, EPI_PLAIN_EDGE};
    return run_bank(h, bi, epi[mode], rows, out, bk.nout, nullptr, st);
}

int b2_gauge(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    const char* part = nullptr;
    char full[64];
    snprintf(full, sizeof full, "%s.g", name ? name : "");
    const int ni = name ? norm_index(h, full, &part) : -1;
    if (ni < 0 || !X || !out || rows < 1 || rows > h->max_rows)
        return fail(h, B2_ERR_ARG, "b2_gauge: bad argument (a Pythia norm name: ln1.<l>, ln2.<l> or lnf)");
    return run_gauge(h, X, nullptr, rows, ni, out, (cudaStream_t)stream);
}

// ---- b2_bank_noalloc: b2_bank for callers that cannot let the library allocate device memory ----------------------
// The quantised rows (x16, ex, LS) that b2_bank keeps in buffers from b2_alloc_streams go instead to this fixed area
// of the library's own device image, one per device, shared by every handle on that device. Its address is looked up
// once per device (first call, device current) and cached.
}  // extern "C"

namespace {
constexpr size_t NOALLOC_BYTES = 4u << 20;   // B2_NOALLOC_SCRATCH_BYTES in base2.h
constexpr int NOALLOC_MAX_DEVICES = 64;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }
}  // namespace

extern "C" {

int b2_bank_noalloc(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, int32_t mode,
                    void* stream) {
    if (!h) return B2_ERR_ARG;
    if (!h->finalized) return fail(h, B2_ERR_STATE, "b2_bank_noalloc: b2_finalize has not been called");
    const int bi = name ? bank_index(h, name) : -1;
    if (bi < 0 || !X || !out || rows < 1 || mode < 0 || mode > 3)
        return fail(h, B2_ERR_ARG, "b2_bank_noalloc: bad argument");
    if (h->cfg.kind == B2_PYTHIA && mode < 2)
        return fail(h, B2_ERR_ARG, "b2_bank_noalloc: Pythia's banks are plain (modes 2 and 3)");
    if (h->flags) return fail(h, B2_ERR_ARG, "b2_bank_noalloc: integer stages only (the handle has float switches)");
    if (h->device < 0 || h->device >= NOALLOC_MAX_DEVICES)
        return fail(h, B2_ERR_ARG, "b2_bank_noalloc: device %d past the %d this entry point serves", h->device,
                    NOALLOC_MAX_DEVICES);
    const DevBank& bk = h->banks[bi];
    // x16 [rows][nin] int32, ex [rows] int32, LS [rows] int64, each at a 256-byte boundary
    const size_t o_ex = align256((size_t)rows * bk.nin * sizeof(int32_t));
    const size_t o_ls = o_ex + align256((size_t)rows * sizeof(int32_t));
    const size_t need = o_ls + (size_t)rows * sizeof(int64_t);
    if (need > NOALLOC_BYTES)
        return fail(h, B2_ERR_ARG, "b2_bank_noalloc: %d rows of %d inputs need %zu bytes of scratch, the fixed area holds "
                    "%zu (use b2_bank for larger calls)", rows, bk.nin, need, NOALLOC_BYTES);
    CK(cudaSetDevice(h->device));
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[h->device]) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return fail(h, B2_ERR_CUDA, "b2_bank_noalloc: scratch address on device %d: %s", h->device,
                            cudaGetErrorString(e));
            g_noalloc_ptr[h->device] = p;
        }
        base = (unsigned char*)g_noalloc_ptr[h->device];
    }
    // nothing here has to start at zero: every scratch entry a kernel reads was written earlier in the same call
    int32_t* x16 = (int32_t*)base;
    int32_t* ex = (int32_t*)(base + o_ex);
    int64_t* LS = (int64_t*)(base + o_ls);
    cudaStream_t st = (cudaStream_t)stream;
    const int gauge = mode < 2;
    if (bk.nin > 1024)
        k_quant<512><<<rows, 512, 0, st>>>(X, bk.nin, nullptr, rows, x16, ex, LS, gauge, h->LOG2, h->log768, h->eps40,
                                           PlaneOut{});
    else
        k_quant<256><<<rows, 256, 0, st>>>(X, bk.nin, nullptr, rows, x16, ex, LS, gauge, h->LOG2, h->log768, h->eps40,
                                           PlaneOut{});
    if (int rc = check_launch(h, "b2_bank_noalloc quant")) return rc;
    BankArgs a{x16, bk.w, bk.nin, bk.nout, rows, {ex, LS, bk.e, bk.b, out, bk.nout, nullptr, h->EXP2, h->PHI}};
    constexpr int RT = 8;
    const dim3 grid((bk.nout + 255) / 256, (rows + RT - 1) / RT);
    switch (mode) {
        case 0: k_bank_simt<EPI_GAUGED, RT><<<grid, 256, 0, st>>>(a); break;
        case 1: k_bank_simt<EPI_GAUGED_EDGE, RT><<<grid, 256, 0, st>>>(a); break;
        case 2: k_bank_simt<EPI_PLAIN_OUT, RT><<<grid, 256, 0, st>>>(a); break;
        default: k_bank_simt<EPI_PLAIN_EDGE, RT><<<grid, 256, 0, st>>>(a); break;
    }
    return check_launch(h, "b2_bank_noalloc bank");
}

int b2_rewind(b2_handle* h, int32_t n_streams, const int32_t* lens, const int32_t* last_tok, void* stream) {
    int rc = ensure_ready(h);
    if (rc) return rc;
    if (n_streams < 1 || n_streams > h->n_slots || !lens || !last_tok) return fail(h, B2_ERR_ARG, "b2_rewind: bad argument");
    cudaStream_t st = (cudaStream_t)stream;
    return launch(h, B2_PROF_OTHER, "rewind", k_rewind, (n_streams + 127) / 128, 128, 0, st, n_streams, lens, last_tok,
                  h->cfg.vocab, h->slot_len, h->slot_tok, h->d_err);
}

int b2_profile(b2_handle* h, int timing) {
    if (!h) return B2_ERR_ARG;
    CK(cudaSetDevice(h->device));
    CK(cudaDeviceSynchronize());
    for (int c = 0; c < B2_PROF_N; c++) {
        for (auto& p : h->prof.ev[c]) { h->prof.pool.push_back(p.first); h->prof.pool.push_back(p.second); }
        h->prof.ev[c].clear();
        h->prof.cnt[c] = 0;
    }
    h->prof.launches = 0;
    if (timing < 0 || timing > 2) return fail(h, B2_ERR_ARG, "b2_profile: mode %d (0 counts, 1 events, 2 stamps)", timing);
    if (timing == 2) {
        int rc;
        if (!h->stamp_slots && (rc = dalloc(h, &h->stamp_slots, (size_t)B2_PROF_N * STAMP_PER_CLASS))) return rc;
        if (!h->stamp_tot && (rc = dalloc(h, &h->stamp_tot, (size_t)2 * B2_PROF_N))) return rc;
        CK(cudaMemset(h->stamp_tot, 0, sizeof(uint64_t) * 2 * B2_PROF_N));
    }
    if ((timing == 2) != (h->prof.timing == 2)) drop_graph(h);   // a captured step holds (or lacks) the stamp kernels
    h->prof.timing = timing;
    return B2_OK;
}

int b2_profile_read(b2_handle* h, int64_t* launches, int64_t* counts, double* ms) {
    if (!h) return B2_ERR_ARG;
    CK(cudaSetDevice(h->device));
    CK(cudaDeviceSynchronize());
    if (launches) *launches = h->prof.launches;
    if (h->prof.timing == 2) {   // stamps: ms = the summed durations of the stamped launches of each class
        uint64_t tot[2 * B2_PROF_N];
        CK(cudaMemcpy(tot, h->stamp_tot, sizeof tot, cudaMemcpyDeviceToHost));
        for (int c = 0; c < B2_PROF_N; c++) {
            if (counts) counts[c] = h->prof.cnt[c];
            if (ms) ms[c] = (double)tot[2 * c] * 1e-6;
        }
        return B2_OK;
    }
    for (int c = 0; c < B2_PROF_N; c++) {
        if (counts) counts[c] = h->prof.cnt[c];
        double t = 0;
        for (auto& p : h->prof.ev[c]) {
            float f = 0;
            if (cudaEventElapsedTime(&f, p.first, p.second) == cudaSuccess) t += f;
        }
        if (ms) ms[c] = t;
    }
    return B2_OK;
}

int b2_check_wait(b2_handle* h, void* stream) {
    if (!h) return B2_ERR_ARG;
    CK(cudaSetDevice(h->device));
    cudaStream_t st = (cudaStream_t)stream;
    int rc = launch(h, B2_PROF_OTHER, "wait_check", k_wait_check, 1, 32, 0, st, h->d_err);
    if (rc) return rc;
    CK(cudaStreamSynchronize(st));
    return read_device_error(h);
}

int b2_sync(b2_handle* h) {
    if (!h) return B2_ERR_ARG;
    CK(cudaSetDevice(h->device));
    CK(cudaDeviceSynchronize());
    return read_device_error(h);
}

void b2_destroy(b2_handle* h) {
    if (!h) return;
    cudaSetDevice(h->device);
    cudaDeviceSynchronize();
    drop_graph(h);
    if (h->cap_stream) cudaStreamDestroy(h->cap_stream);
    if (h->split_trace) {
        const size_t n = (size_t)SPLIT_TRACE_LAUNCHES * SPLIT_TRACE_SLOT;
        std::vector<uint64_t> t(n);
        if (cudaMemcpy(t.data(), h->split_trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost) == cudaSuccess) {
            if (FILE* f = fopen(h->split_trace_path.c_str(), "wb")) {
                fwrite(t.data(), sizeof(uint64_t), n, f);
                fclose(f);
            }
        }
        cudaFree(h->split_trace);
    }
    if (h->att_trace) {
        const size_t n = (size_t)h->cfg.n_layer * 64 * h->cfg.n_head * 8;
        std::vector<uint64_t> t(n);
        if (cudaMemcpy(t.data(), h->att_trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost) == cudaSuccess) {
            if (FILE* f = fopen(h->att_trace_path.c_str(), "wb")) {
                fwrite(t.data(), sizeof(uint64_t), n, f);
                fclose(f);
            }
        }
        cudaFree(h->att_trace);
    }
    for (auto& bk : h->banks) tc_bank_free(bk.tc);
    tc_rows_free(h->tcr);
    for (int c = 0; c < B2_PROF_N; c++)
        for (auto& p : h->prof.ev[c]) { cudaEventDestroy(p.first); cudaEventDestroy(p.second); }
    for (auto e : h->prof.pool) cudaEventDestroy(e);
    for (void* p : h->allocs) cudaFree(p);
    delete h;
}

}  // extern "C"
