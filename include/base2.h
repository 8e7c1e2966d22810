/*
 * base2.h -- C ABI of libbase2cuda.so, the B200 (sm_100a) engine for streaming-machine's integer-only GPT-2 and
 * its Pythia variant (foundation0/pythia_base2.py).
 *
 * The reference has no FFI: its "API" is base2.py's module namespace (forward, gauged_bank, plain_bank, attention,
 * edge, race, ...; base2.py:18-114), the converter's npz keys (base2_convert.py:31-61) and the Metal engine's prompt
 * pass + per-token loop (base2_stream.swift:264-281). Each entry point below names the piece it replaces.
 *
 * Conventions
 *   - plain pointers and sizes; no torch types. Model arrays passed to b2_set_* are HOST pointers (copied).
 *   - ids/tokens/logits of b2_prefill/b2_step/b2_generate are DEVICE pointers, work is queued on `stream`
 *     (a cudaStream_t, NULL = the legacy default stream). b2_step_host takes HOST pointers and synchronises.
 *   - every call returns a b2_status; b2_last_error() gives the message. No exception crosses the ABI.
 *   - one handle per (process, GPU); calls on a handle must not overlap.
 */
#ifndef BASE2_H
#define BASE2_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_ABI_VERSION 1

typedef struct b2_handle b2_handle;

typedef enum {
    B2_OK = 0,
    B2_ERR_ARG = 1,      /* bad argument, shape or name */
    B2_ERR_CUDA = 2,     /* a CUDA runtime call failed */
    B2_ERR_NOMEM = 3,    /* device allocation failed */
    B2_ERR_CTX = 4,      /* a position passed the allocated context (or the model's n_ctx) */
    B2_ERR_VALUE = 5,    /* a value did not fit the device layout (e.g. a V-cache entry beyond int32) */
    B2_ERR_STATE = 6,    /* call out of order (e.g. b2_step before b2_prefill) */
    B2_ERR_DEVICE = 7    /* a device-side check failed (token id out of range, ...) */
} b2_status;

typedef enum { B2_GPT2 = 0, B2_PYTHIA = 1 } b2_kind;

/* stage switches (base2.py:10-11 gauge=/edge=/arrival=; pythia_base2.py:20 adds turn=): a set bit puts that stage
 * back to float64, in the reference's order of operations (base2.py:66-69, 79-80, 89-92, 110-113; pythia_base2.py:
 * 102-104, 118-120, 130-133, 144-146). The gauge and the turn give the reference's integers exactly; the bends and
 * the arrival use the device's tanh/pow/erf/exp, which can differ from the C library's in the last place and so,
 * rarely, move an integer by one. A handle with any switch set runs the CUDA-core bank kernel. */
enum { B2_GAUGE_FLOAT = 1, B2_EDGE_FLOAT = 2, B2_ARRIVAL_FLOAT = 4, B2_TURN_FLOAT = 8 /* Pythia only */ };

typedef struct {
    int32_t kind;       /* b2_kind */
    int32_t n_layer;    /* 12 */
    int32_t d_model;    /* 768 */
    int32_t n_head;     /* 12 (head size d_model / n_head = 64) */
    int32_t d_ff;       /* 3072 */
    int32_t vocab;      /* 50257 (GPT-2), 50304 (Pythia-160M) */
    int32_t n_ctx;      /* 1024: rows of the position table (GPT-2); 2048: rows of the turn tables (Pythia) */
} b2_config;

/* Create a handle on `device` (replaces base2.py's module import, base2.py:10-16). flags: B2_*_FLOAT bits. */
int b2_create(const b2_config* cfg, int device, int flags, b2_handle** out);

/* One weight bank in the converter's layout (base2_convert.py:40-45, base2_gpu.py:9-14): name "qkv.L", "proj.L",
 * "fc.L", "mproj.L" or "head"; w [nin][nout] int16, e [nout] per-column power of two, b [nout] bias (stream scale;
 * NULL = no bias, Pythia's head, pythia_base2.py:56). Pythia's qkv columns are per head q, k, v (pythia_base2.py:126). */
int b2_set_bank(b2_handle* h, const char* name, const int16_t* w, const int64_t* e, const int64_t* b,
                int32_t nin, int32_t nout);

/* A bank's tensor-core layout computed ahead of time (streaming_machine_b200/layout.py writes it to disk beside the
 * reference's device files, base2_gpu.py:9-17): wh = w >> 8 and wl = (w & 255) - 128 as int8 [nout_pad][nin]
 * (K-major, nout_pad = nout rounded up to 128, padded outputs w = 0), colcorr [nout_pad] = 128 sum_i w[i][j] - 16384 nin,
 * colcorr_kb [nin / 128][nout_pad] the same per 128-input block (0 on padded outputs). Given after that bank's
 * b2_set_bank and before b2_finalize, finalize uploads it instead of building it on the device. No reference
 * counterpart: the reference's device layout is the [nin][nout] int16 bank itself. */
int b2_set_bank_layout(b2_handle* h, const char* name, const int8_t* wh, const int8_t* wl, const int64_t* colcorr,
                       const int64_t* colcorr_kb);

/* Copy a finalized bank's tensor-core layout (as above) to host buffers: to check or save a layout file. */
int b2_get_bank_layout(b2_handle* h, const char* name, int8_t* wh, int8_t* wl, int64_t* colcorr, int64_t* colcorr_kb);

/* A table or embedding by its npz key (base2_convert.py:46-59): "wte" [vocab][d], "wpe" [n_ctx][d], "phi" [65536],
 * "arrival" [n], "log2" [65536], "exp2" [65536]. Pythia (pythia_convert.py's keys, `plates=finished`): "embed.w"
 * [vocab][d] and "embed.e" [vocab] (each word's row and its power of two), "cos"/"sin" [n_ctx][rot/2] at 2^-30, and
 * each norm's gain and offset "ln1.<l>.g", "ln1.<l>.b", "ln2.<l>.g", "ln2.<l>.b", "lnf.g", "lnf.b" [d]. */
int b2_set_array(b2_handle* h, const char* name, const int64_t* data, int64_t n);

/* A scalar by its npz key: "log2_768", "eps40" (base2_convert.py:60-61); Pythia: "eps40", "half_log2_hs", "rot"
 * (16) and each norm's gain exponent "ln1.<l>.ge", "ln2.<l>.ge", "lnf.ge". One engine setting besides: "wait_ns",
 * how long a device-side wait (a TMA or bulk-copy completion, a counter other CTAs raise) may take before the
 * kernel gives up, flags the call and returns (default 0 = 0.5 s); it may be set at any time. And "top_read" (the
 * reference's top=plain / top=fr switch, base2_stream_fr2.swift:23-38): 0 (default) scores every word then races;
 * 1 races decode steps of up to 4 streams that store no scores by the exact collapsing read (every word's coarse score
 * from the high byte plane, bounds from the input's positive and negative sums, only the words that can still win read
 * their low bytes): the same words. "entry_tables" (GPT-2; the reference's stored layer-0 entry, base2_entry.py,
 * base2_layer0.py, base2_stream_fr2.swift:407-428): 1 makes every decode step take layer 0's qkv piles from two stored
 * rows, wte . W and wpe . W of the qkv.0 bank (built as exact int64 piles at the next b2_alloc_streams, 0.95 GB for
 * GPT-2 124M), instead of the bank product: the same bits, refused (B2_ERR_ARG) when an embedded value can reach 2^15,
 * where to16 would round the row; 0 (default) drops them. */
int b2_set_scalar(b2_handle* h, const char* name, int64_t v);

/* All arrays given: build the device layouts. */
int b2_finalize(b2_handle* h);

/* Reserve `n_streams` independent stream slots with a key/value store of `max_ctx` positions each
 * (the Metal engine's per-layer KV buffers, base2_stream.swift:205-208, here per stream). */
int b2_alloc_streams(b2_handle* h, int32_t n_streams, int32_t max_ctx);

/* Prompt pass for streams 0..n_streams-1 (base2_stream.swift:274-275; base2.py:102-114 on the prompt).
 * ids: the prompts concatenated, lens[s] ids for stream s (device pointers). Resets those streams.
 * next_tok [n_streams]: the race's word at each prompt's last position. logits (optional, may be NULL):
 * [n_streams][vocab] int64, the scores raced on. */
int b2_prefill(b2_handle* h, const int32_t* ids, const int32_t* lens, int32_t n_streams,
               int32_t* next_tok, int64_t* logits, void* stream);

/* One new position for each of streams 0..n_streams-1 (base2_stream.swift:276-280; base2.py:123 with the prefix
 * kept). tok_in [n_streams] (NULL: each stream's last word, fed back on the device like `nextin`,
 * base2_stream.swift:143-146). tok_out [n_streams]; logits optional [n_streams][vocab]. */
int b2_step(b2_handle* h, const int32_t* tok_in, int32_t n_streams, int32_t* tok_out, int64_t* logits,
            void* stream);

/* n_steps greedy steps with the words fed back on the device; tokens_out [n_streams][n_steps] (device). */
int b2_generate(b2_handle* h, int32_t n_streams, int32_t n_steps, int32_t* tokens_out, void* stream);

/* b2_step with HOST buffers: copies tok_in in, runs the step, copies tok_out back, synchronises. */
int b2_step_host(b2_handle* h, const int32_t* tok_in, int32_t n_streams, int32_t* tok_out);

/* One bank on given rows, for unit parity (base2.py:62-76): mode 0 = gauged_bank, 1 = gauged_bank then edge,
 * 2 = plain_bank, 3 = plain_bank then edge (Pythia's fc, pythia_base2.py:166; Pythia takes modes 2 and 3 only).
 * X [rows][nin] int64, out [rows][nout] int64 (device pointers). */
int b2_bank(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, int32_t mode, void* stream);

/* Pythia's layer norm on given rows (pythia_base2.py:100-110, gauge(R, name)): name "ln1.<l>", "ln2.<l>" or "lnf";
 * X, out [rows][d] int64 (device pointers). */
int b2_gauge(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, void* stream);

/* b2_bank (modes 0-3, same results) for callers that cannot let the library allocate device memory: a host whose
 * own allocator owns the GPU's memory, or code that must not pay cudaMalloc/cudaFree's implicit device-wide
 * synchronisation. This call allocates nothing and needs only b2_finalize (not b2_alloc_streams). The quantised rows
 * go to a fixed scratch area of B2_NOALLOC_SCRATCH_BYTES inside the library's device image, one per device:
 * rows x (4 nin + 12) bytes plus alignment must fit (about 1,360 rows of a 768-input bank, 340 of a 3,072-input
 * bank); larger calls return B2_ERR_ARG and should use b2_bank. The area is shared by every handle on the device, so
 * calls on one device must not overlap: two calls in flight at once (other threads or other streams) race on it and
 * give wrong results. Nothing in it needs to start at zero. X, out device pointers; work queued on `stream` (the
 * CUDA-core bank kernel). No reference counterpart (the reference allocates per call, base2.py:62-76). */
#define B2_NOALLOC_SCRATCH_BYTES (4u << 20)
int b2_bank_noalloc(b2_handle* h, const char* name, const int64_t* X, int32_t rows, int64_t* out, int32_t mode,
                    void* stream);

/* Truncate streams 0..n_streams-1 back to lens[s] positions with last_tok[s] as the word to feed next (device
 * pointers). Keys/values below lens[s] are kept. A truncation past a stream's current length is a device-checked
 * error (B2_ERR_CTX). The reference has no counterpart: its machine recomputes every prefix (base2.py:123). */
int b2_rewind(b2_handle* h, int32_t n_streams, const int32_t* lens, const int32_t* last_tok, void* stream);

/* Profiling. B2_PROF_* kernel classes; b2_profile(h, mode) resets the counters. mode 1 brackets every launch with
 * CUDA events on its stream (launches then run without programmatic overlap and outside the step graph); mode 2
 * leaves launches, step graph and overlap as they are and has each bank, arrival, quantisation and heads kernel
 * stamp the start of its dependent work (%globaltimer, first CTA); a kernel's duration is then its start to the next
 * stamped start, so unstamped kernels count towards the stamped one before them. b2_profile_read fills launches
 * (total kernel launches since the reset) and, per class, the launch count and the summed time in ms (arrays of
 * B2_PROF_N). No reference counterpart beyond the Metal engine's bench modes (base2_stream_fr2.swift:1060-1149). */
enum { B2_PROF_BANK = 0, B2_PROF_ATTEND = 1, B2_PROF_QUANT = 2, B2_PROF_HEADS = 3, B2_PROF_RACE = 4, B2_PROF_OTHER = 5,
       B2_PROF_N = 6 };
int b2_profile(b2_handle* h, int timing);
int b2_profile_read(b2_handle* h, int64_t* launches, int64_t* counts, double* ms);

/* Wait for queued work and report any device-side check that failed since the last call. */
int b2_sync(b2_handle* h);

/* Self-check of failure detection: one kernel waits, through the engine's bounded wait, for a copy that never comes.
 * After the "wait_ns" limit it gives up; the call returns B2_ERR_DEVICE ("bounded wait gave up") and the handle
 * stays usable. No reference counterpart (the reference's machine has no device waits, base2.py:102-114). */
int b2_check_wait(b2_handle* h, void* stream);

const char* b2_last_error(const b2_handle* h);
void b2_destroy(b2_handle* h);
int b2_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif
