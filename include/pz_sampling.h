/*
 * pz_sampling.h — C ABI of the B200 token sampler (logits -> token id).
 *
 * Two layers:
 *
 *  1. The six legacy entry points of Project Zero's sampler, with the same
 *     names, signatures and semantics.  They take HOST pointers, exactly like
 *     the CPU code they replace; the library stages the row to the GPU, runs
 *     the sm_100a kernels and copies the result back.  Defining
 *     PZ_NO_LEGACY_NAMES before including this header hides the unprefixed
 *     names; the pz_-prefixed aliases are always exported.
 *
 *       reference include/sampling/sampling.h:12  int   sample_argmax(const float*, int)
 *       reference include/sampling/sampling.h:23  void  apply_temperature(float*, int, float)
 *       reference include/sampling/sampling.h:36  int   sample_top_p(float*, int, float, unsigned long long*)
 *       reference include/sampling/sampling.h:49  int   sample_top_k(float*, int, int, unsigned long long*)
 *       reference include/sampling/rng.h:14       void  rng_seed(unsigned long long*, unsigned long long)
 *       reference include/sampling/rng.h:21       float rng_float(unsigned long long*)
 *
 *  2. A batched, stream-ordered API on DEVICE pointers (device-resident
 *     hand-off from the LM head: no host round trip).  One call samples B
 *     rows, each with its own pz_sampler_config, penalty history and RNG
 *     state.  It replaces the per-step sampling block of the reference's
 *     generate loop (reference src/transformer/generate.c:146-170) for a
 *     whole batch, with the penalty / top-k -> top-p composition defined in
 *     the pipeline contract below.
 *
 * Pipeline contract per row (what pz_sample_batch computes):
 *   x      = logits row, widened to fp32 (bf16 -> fp32 is exact: bits << 16)
 *   A8     for each distinct id t in the row's history with count c (ids
 *          outside [0,V) ignored):
 *            if (rep != 1) x[t] = x[t] > 0 ? x[t] / rep : x[t] * rep;
 *            x[t] = x[t] - (c * freq + presence)     (float ops, in that order)
 *   A7     if (T <= 0 || T < 1e-6f): token = argmax(x) (first index of the
 *          maximum, NaN never wins unless at [0]); no RNG draw.
 *   A3     x *= 1.0f / T     (reference src/sampling/temperature.c:11-20;
 *                             PZ_CFG_TEMP_DIVIDE selects x /= T, :22-23)
 *   A9     k_eff = (k <= 0 || k >= V) ? 0 : min(k, 1024)
 *          k_eff == 0:  0 < p < 1 -> sample_top_p over the whole row
 *                                    (reference src/sampling/top_p.c:30-108)
 *                       otherwise -> softmax + CDF walk in index order
 *                                    (reference src/transformer/generate.c:157-168)
 *          k_eff >= 1:  the top-k selection of reference
 *                       src/sampling/top_k.c:27-48 (value desc, lowest index
 *                       among ties, entries > -1e30 only, padded with
 *                       (-1e30, -1)); then
 *                       0 < p < 1 -> the sample_top_p steps run over that
 *                                    sorted list (top_p.c:37-105)
 *                       otherwise -> the top-k softmax and draw (top_k.c:50-72)
 *   A1     every non-greedy row consumes exactly one xorshift64* draw from
 *          its RNG state (reference src/sampling/rng.c:8-17).
 * With no history, k = 0 and fp32 input this IS the reference call sequence
 * of generate.c:151-170.
 */
#ifndef PZ_SAMPLING_H
#define PZ_SAMPLING_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status codes.  Modelled on TernaryError (reference include/core/error.h:4-31):
 * zero is success, every failure has its own code and a string. */
typedef enum pz_status {
  PZ_OK = 0,
  PZ_ERR_INVALID_ARGS = 1,   /* null pointer, bad size, bad dtype ...        */
  PZ_ERR_CUDA = 2,           /* a CUDA runtime call failed                   */
  PZ_ERR_OOM = 3,            /* device or host allocation failed             */
  PZ_ERR_NCCL = 4,           /* NCCL unavailable or a collective failed      */
  PZ_ERR_TIMEOUT = 5,        /* a bounded wait ran out                       */
  PZ_ERR_UNSUPPORTED = 6,    /* request outside the library's limits         */
  PZ_ERR_NO_DEVICE = 7,      /* no CUDA device visible                       */
  PZ_ERR_COUNT
} pz_status;

const char *pz_status_str(pz_status s);

/* Per-row status written by the kernels (optional output array). */
enum {
  PZ_ROW_OK = 0,
  PZ_ROW_HISTORY_TOO_LONG = 1, /* row history longer than the ctx's max_history */
  PZ_ROW_HINT_VIOLATED = 2,    /* row needs a full-vocabulary pass the hints excluded */
  PZ_ROW_TIMEOUT = 3           /* a bounded wait inside the kernel ran out */
};

typedef enum pz_dtype { PZ_DTYPE_F32 = 0, PZ_DTYPE_BF16 = 1 } pz_dtype;

/* Per-row sampler settings, 32 bytes, read by the kernels from device memory. */
typedef struct pz_sampler_config {
  float temperature;         /* <= 0 or < 1e-6: greedy (A7)                */
  int32_t top_k;             /* 0 or >= V: off; clamped to 1024 (A9)       */
  float top_p;               /* nucleus when 0 < top_p < 1 (A5)            */
  float repetition_penalty;  /* 1: off (A8)                                */
  float frequency_penalty;   /* 0: off (A8)                                */
  float presence_penalty;    /* 0: off (A8)                                */
  uint32_t flags;            /* PZ_CFG_* bits                              */
  uint32_t reserved;         /* must be 0                                  */
} pz_sampler_config;

/* Temperature as `x /= T` (the reference's non-AVX-512 build,
 * temperature.c:22-23) instead of `x *= 1/T` (its AVX-512 build, :11-20). */
#define PZ_CFG_TEMP_DIVIDE 0x1u

/* Top-k list cap (reference src/sampling/top_k.c:6 TOP_K_MAX). */
#define PZ_TOP_K_MAX 1024
/* sample_top_p falls back to argmax above this vocabulary size
 * (reference src/sampling/top_p.c:26,33-34). */
#define PZ_TOP_P_MAX_VOCAB 200000

/* ------------------------------------------------------------------------ */
/* Layer 1: the reference's six calls (host pointers, one row).             */

/* reference src/sampling/argmax.c:3-13 */
int pz_sample_argmax(const float *logits, int vocab_size);
/* reference src/sampling/temperature.c:8-25 (multiply-by-reciprocal variant) */
void pz_apply_temperature(float *logits, int vocab_size, float temperature);
/* reference src/sampling/top_p.c:30-108; logits are read, not modified */
int pz_sample_top_p(float *logits, int vocab_size, float top_p,
                    unsigned long long *rng_state);
/* reference src/sampling/top_k.c:8-73; logits are read, not modified */
int pz_sample_top_k(float *logits, int vocab_size, int k,
                    unsigned long long *rng_state);
/* reference src/sampling/rng.c:3-6 */
void pz_rng_seed(unsigned long long *state, unsigned long long seed);
/* reference src/sampling/rng.c:8-17 */
float pz_rng_float(unsigned long long *state);

/* Full-softmax draw of the reference's generate loop
 * (src/transformer/generate.c:157-168): softmax over the whole row, then the
 * CDF walk in index order; fallback V-1.  `logits` is read, not modified
 * (the reference's tn_softmax leaves the probabilities in the buffer; no
 * caller reads them after the draw). */
int pz_sample_softmax(float *logits, int vocab_size,
                      unsigned long long *rng_state);

#ifndef PZ_NO_LEGACY_NAMES
int sample_argmax(const float *logits, int vocab_size);
void apply_temperature(float *logits, int vocab_size, float temperature);
int sample_top_p(float *logits, int vocab_size, float top_p,
                 unsigned long long *rng_state);
int sample_top_k(float *logits, int vocab_size, int k,
                 unsigned long long *rng_state);
void rng_seed(unsigned long long *state, unsigned long long seed);
float rng_float(unsigned long long *state);
#endif

/* Status of the most recent legacy call on this thread (the legacy
 * signatures have no status return; a failed call returns -1 / leaves the
 * data unchanged and records the reason here). */
pz_status pz_last_error(void);
/* Text of the CUDA error behind the last PZ_ERR_CUDA on this thread ("" if none). */
const char *pz_last_error_detail(void);

/* ------------------------------------------------------------------------ */
/* Layer 2: batched device API.                                              */

typedef struct pz_sampler_ctx pz_sampler_ctx;

/* Capacity of a context.  Scratch memory is sized from these at creation;
 * pz_sample_batch rejects calls beyond them with PZ_ERR_UNSUPPORTED. */
typedef struct pz_ctx_limits {
  int32_t max_batch;     /* rows per call                                  */
  int32_t max_vocab;     /* V per call (vocab slice length when sharded)   */
  int32_t max_top_k;     /* largest top_k any row will use (<= 1024)       */
  int32_t max_history;   /* longest penalty history of any row             */
} pz_ctx_limits;

/* Creates a context on `device` (the caller's current device is restored on
 * return).  All scratch is allocated here; sampling calls allocate nothing. */
pz_status pz_ctx_create(pz_sampler_ctx **ctx, int device,
                        const pz_ctx_limits *limits);
pz_status pz_ctx_destroy(pz_sampler_ctx *ctx);
/* Bytes of device scratch the context holds. */
size_t pz_ctx_scratch_bytes(const pz_sampler_ctx *ctx);

/* Hints that let a call skip work.  Passing NULL means "no promises".
 *   max_top_k / max_history: upper bounds over the rows of this call
 *       (0 = use the context limit);
 *   no_full_vocab: 1 promises that no row needs a full-vocabulary pass
 *       (every non-greedy row has 1 <= top_k < V).  A row that breaks the
 *       promise gets token -1 and PZ_ROW_HINT_VIOLATED. */
typedef struct pz_batch_hints {
  int32_t max_top_k;
  int32_t max_history;
  int32_t no_full_vocab;
  int32_t reserved;
} pz_batch_hints;

/* Optional per-row outputs; any pointer may be NULL.
 *   cand_ids / cand_probs: [B x cand_stride]; for rows with k_eff >= 1 the
 *       sorted top-k list (ids) and the probabilities the sampler computed
 *       for it (A5 steps: e*inv in list order, 0 for entries the max-20
 *       filter dropped; A4: e/sum); other rows get -1 / 0.
 *   n_cand: [B] number of list entries written (k_eff, or 0).
 *   row_status: [B] PZ_ROW_* codes.
 *   token_logprob: [B] OpenAI-style log-probability of the sampled id: its
 *       value minus the log-sum-exp of the whole row, over the penalised,
 *       tempered values (greedy rows: penalised, untempered) — the
 *       distribution before top-k / top-p truncation; NaN for a row with no
 *       token.  No counterpart in the reference.
 *   cand_logprobs: [B x cand_stride] the same for the list entries (the
 *       row's most likely ids, in order: OpenAI's top_logprobs), -inf past
 *       n_cand.  Asking for either costs one more read of each row; fp32
 *       accuracy (~1e-5).  Not available from the vocab-sharded call. */
typedef struct pz_batch_outputs {
  int32_t *cand_ids;
  float *cand_probs;
  int32_t *n_cand;
  int32_t *row_status;
  int32_t cand_stride;
  int32_t reserved;
  float *token_logprob;
  float *cand_logprobs;
} pz_batch_outputs;

/* Samples B rows.  All pointers are DEVICE pointers on the ctx's device.
 *   logits:      B rows of V elements, row r at logits + r*ld (elements).
 *   cfg:         B configs, one per row.
 *   hist, hist_off: CSR penalty history: the ids of row r are
 *                hist[hist_off[r] .. hist_off[r+1]); both may be NULL (no
 *                history).
 *   rng_state:   B xorshift64* states, advanced in place (one draw per
 *                non-greedy row).
 *   out_tokens:  B sampled ids.
 * Stream-ordered and asynchronous on `stream` (a cudaStream_t; NULL = the
 * legacy default stream).  Calls that share a context must be ordered (one
 * stream, or explicit events): they share the context's scratch. */
pz_status pz_sample_batch(pz_sampler_ctx *ctx, const void *logits,
                          pz_dtype dtype, int B, int V, int64_t ld,
                          const pz_sampler_config *cfg, const int32_t *hist,
                          const int32_t *hist_off,
                          unsigned long long *rng_state, int32_t *out_tokens,
                          const pz_batch_hints *hints,
                          const pz_batch_outputs *outputs, void *stream);

/* Context-free, allocation-free form of pz_sample_batch.  No counterpart in
 * the reference (whose sampler is a single-row CPU routine with no scratch):
 * it exists for callers that may not allocate device memory at sampling
 * time.  Its scratch is one fixed device array per device (about 2.1 MiB)
 * sized for the limits below.
 *   - Runs on the caller's CURRENT device.  The first call on a device does
 *     the set-up (looks up the array's address and sets kernel attributes);
 *     make that first call before any stream capture.  Later calls allocate
 *     nothing and only launch kernels.
 *   - B > PZ_STATIC_MAX_BATCH or V > PZ_STATIC_MAX_VOCAB: PZ_ERR_UNSUPPORTED
 *     with the reason in pz_last_error_detail().  Rows whose top_k is 0 or
 *     above PZ_STATIC_MAX_TOP_K (they would need a full-vocabulary pass or a
 *     longer list) get token -1 and PZ_ROW_HINT_VIOLATED; rows with more
 *     than PZ_STATIC_MAX_HISTORY history ids get PZ_ROW_HISTORY_TOO_LONG.
 *   - outputs->cand_stride, when candidates are asked for, is at least
 *     PZ_STATIC_MAX_TOP_K.
 *   - Every call on a device shares the one array: calls that overlap in
 *     time (two streams, two host threads without ordering) race and give
 *     wrong tokens.  Order them on one stream or with events.
 * Results are identical to pz_sample_batch's for the rows it accepts. */
#define PZ_STATIC_MAX_BATCH 1024
#define PZ_STATIC_MAX_VOCAB 1048576
#define PZ_STATIC_MAX_TOP_K 64
#define PZ_STATIC_MAX_HISTORY 1024
pz_status pz_sample_batch_static(const void *logits, pz_dtype dtype, int B,
                                 int V, int64_t ld,
                                 const pz_sampler_config *cfg,
                                 const int32_t *hist, const int32_t *hist_off,
                                 unsigned long long *rng_state,
                                 int32_t *out_tokens,
                                 const pz_batch_outputs *outputs,
                                 void *stream);

/* Kernel timing for performance work.  pz_ctx_profile(ctx, n) creates n
 * slots of CUDA events (n = 0 turns timing off); while on, each of the next
 * n sampling calls on the context records events around its kernels on the
 * call's stream.  pz_ctx_profile_read waits for the recorded calls and
 * returns the summed milliseconds of the streaming kernels (slice_kernel,
 * which also decides the rows, and in large batches with lists longer
 * than 64 the slice_long_kernel launch after it) and of the rest of each call (the
 * full-vocabulary pass, when a row needs one), the number of calls timed
 * and the number of kernels they launched; it then starts a new count. */
pz_status pz_ctx_profile(pz_sampler_ctx *ctx, int n_calls);
pz_status pz_ctx_profile_read(pz_sampler_ctx *ctx, double *slice_ms,
                              double *rest_ms, int *calls, int *kernels);
/* The same timing split by phase: phase_ms[0] the slice kernels, [1] the
 * full-vocabulary pass (full_kernel), [2] the vocab-sharded allgather,
 * [3] merge_kernel; summed over the timed calls.  Starts a new count. */
pz_status pz_ctx_profile_phases(pz_sampler_ctx *ctx, double phase_ms[4],
                                int *calls, int *kernels);

/* Seeds B RNG states on the device: state[r] = seed_base + r (0 -> 1, as
 * rng_seed does), or state[r] = seeds[r] when `seeds` (device) is non-NULL. */
pz_status pz_rng_seed_batch(unsigned long long *rng_state, int B,
                            unsigned long long seed_base,
                            const unsigned long long *seeds, void *stream);

/* ------------------------------------------------------------------------ */
/* The generate loop on the device.                                          */

/* Appends each row's sampled id to its history window: tokens[r] goes to
 * hist_ring[r * W + (*counter % W)], then *counter advances by one (all on
 * `stream`, device pointers).  Penalties count the ids of a row's window, so
 * the ring order does not matter; slots holding -1 (or any id outside
 * [0, V)) are ignored, so a window starts as -1s or the prompt's last ids.
 * The window is passed to pz_sample_batch as hist = hist_ring, hist_off[r] =
 * r * W.  (The reference keeps no history: its loop only draws, generate.c
 * :137-170.) */
pz_status pz_history_append(int32_t *hist_ring, int B, int W, const int32_t *tokens,
                            int32_t *counter, void *stream);

/* The hand-off from the LM head.  pz_lm_head_logits is the classifier of
 * reference src/transformer/forward.c:102-165 in its bf16 form
 * (parallel_matmul_bf16): logits[b][v] = sum_d hidden[b][d] * w_cls[v][d],
 * hidden fp32 [B x dim], w_cls bf16 bits [V x dim] (row v = token v's
 * classifier row), logits fp32 rows of stride ld, all device pointers, on
 * `stream` (dim a multiple of 8, hidden and w_cls 16-byte aligned).
 * pz_sample_from_hidden runs it and pz_sample_batch on that buffer back to
 * back on the stream: the logits never leave the device.  (fp32 sums in an
 * order of its own: the LM head is outside the sampler's parity contract.) */
pz_status pz_lm_head_logits(pz_sampler_ctx *ctx, const float *hidden, int B, int dim,
                            const uint16_t *w_cls, int V, float *logits, int64_t ld,
                            void *stream);
pz_status pz_sample_from_hidden(pz_sampler_ctx *ctx, const float *hidden, int B, int dim,
                                const uint16_t *w_cls, int V, float *logits, int64_t ld,
                                const pz_sampler_config *cfg, const int32_t *hist,
                                const int32_t *hist_off, unsigned long long *rng_state,
                                int32_t *out_tokens, const pz_batch_hints *hints,
                                const pz_batch_outputs *outputs, void *stream);

/* One sampling step of the generate loop (reference
 * src/transformer/generate.c:137-170) recorded once as a CUDA graph and
 * replayed every step: sample the B rows of the fixed logits buffer the LM
 * head writes (as RunState.logits is rewritten each step in the reference,
 * forward.c:221), advance the rows' RNG states in place, and append the
 * sampled ids to the history window (hist_ring of W slots per row, or NULL
 * and W = 0 for no penalty window).  Device pointers, fixed for the step's
 * life.  Seed the states once with pz_rng_seed_batch (for instance from
 * pz_sampling_params.seed: the reference parses --seed but seeds with
 * time(NULL), generate.c:126).  Creation captures on a private stream and
 * allocates; launches allocate nothing. */
typedef struct pz_decode_step pz_decode_step;
pz_status pz_decode_step_create(pz_sampler_ctx *ctx, const void *logits, pz_dtype dtype,
                                int B, int V, int64_t ld,
                                const pz_sampler_config *cfg, int32_t *hist_ring,
                                int W, unsigned long long *rng_state,
                                int32_t *out_tokens, const pz_batch_hints *hints,
                                pz_decode_step **step);
pz_status pz_decode_step_launch(pz_decode_step *step, void *stream);
/* Steps launched so far (synchronous read of the device counter). */
pz_status pz_decode_step_count(const pz_decode_step *step, int32_t *steps);
pz_status pz_decode_step_destroy(pz_decode_step *step);

/* ------------------------------------------------------------------------ */
/* Multi-GPU.                                                                */

/* Row sharding: the contiguous row range [*begin, *begin + *count) that rank
 * `rank` of `world` owns in a batch of B rows (no communication). */
void pz_row_shard(int B, int world, int rank, int *begin, int *count);

/* Vocab sharding: each rank holds the columns [v_offset, v_offset + V_local)
 * of every row.  The rank computes its local top-k candidates, all ranks
 * exchange them with ONE NCCL allgather, and every rank merges the G*k
 * candidates into the exact global top-k (value desc, global id asc) and
 * draws with the row's RNG state.  Every rank returns the same tokens and
 * advances the same RNG states.  Penalty history is given in GLOBAL ids;
 * each rank applies the ids that fall in its slice (no extra collective).
 * Requires every non-greedy row to have 1 <= top_k < V_global — other rows
 * get token -1 and PZ_ROW_HINT_VIOLATED.  Greedy rows take the global
 * argmax. */
pz_status pz_nccl_get_unique_id(void *id_out, size_t id_bytes);
/* Joins the context to a communicator of `world` ranks.  The communicator
 * is non-blocking: its set-up and every allgather are polled against a
 * deadline of timeout_ms (60 s for pz_ctx_init_nccl).  A rank that never
 * joins, or an NCCL error, makes the call abort the communicator and return
 * PZ_ERR_TIMEOUT / PZ_ERR_NCCL instead of waiting for ever; later sharded
 * calls on the context then fail with PZ_ERR_NCCL. */
pz_status pz_ctx_init_nccl(pz_sampler_ctx *ctx, int world, int rank,
                           const void *unique_id, size_t id_bytes);
pz_status pz_ctx_init_nccl_timeout(pz_sampler_ctx *ctx, int world, int rank,
                                   const void *unique_id, size_t id_bytes,
                                   int timeout_ms);
/* Waits at most timeout_ms for the work queued on `stream` (a sharded
 * call's allgather included).  Polls the communicator's asynchronous error
 * meanwhile: an NCCL error gives PZ_ERR_NCCL, and the deadline
 * PZ_ERR_TIMEOUT; either way the communicator is aborted, which ends its
 * collectives still in flight.  PZ_OK once the stream is idle. */
pz_status pz_ctx_wait(pz_sampler_ctx *ctx, void *stream, int timeout_ms);
/* Aborts the context's communicator (for a caller that learned from
 * elsewhere, e.g. a heartbeat, that a peer has gone). */
pz_status pz_ctx_abort_nccl(pz_sampler_ctx *ctx);
pz_status pz_sample_batch_vocab_sharded(
    pz_sampler_ctx *ctx, const void *logits_slice, pz_dtype dtype, int B,
    int V_local, int64_t ld, int64_t v_offset, int V_global,
    const pz_sampler_config *cfg, const int32_t *hist,
    const int32_t *hist_off, unsigned long long *rng_state,
    int32_t *out_tokens, const pz_batch_outputs *outputs, void *stream);

/* ------------------------------------------------------------------------ */
/* Several GPUs driven by one host thread.  The reference samples one row on
 * the CPU of a single process (src/transformer/generate.c:143-170); a server
 * that owns all of a node's GPUs in one process shards the batch over them
 * with these two calls instead of one process per GPU. */

/* One device's part of a multi-device call: a context on that device, the
 * stream to queue on (a stream of that device) and DEVICE pointers on it. */
typedef struct pz_shard {
  pz_sampler_ctx *ctx;
  const void *logits;      /* rows (row mode) or column slice (vocab mode)    */
  int64_t ld;              /* elements between rows                           */
  int32_t B;               /* rows held here (vocab mode: the same on all)    */
  int32_t V;               /* columns held here                               */
  int64_t v_offset;        /* vocab mode: global id of column 0; row mode: 0  */
  const pz_sampler_config *cfg;
  const int32_t *hist;     /* CSR history in GLOBAL ids, or NULL              */
  const int32_t *hist_off;
  unsigned long long *rng_state;
  int32_t *out_tokens;
  const pz_batch_outputs *outputs;  /* may be NULL                           */
  void *stream;
} pz_shard;

#define PZ_SHARD_ROWS 0
#define PZ_SHARD_VOCAB 1

/* Joins n contexts, on n distinct devices of this process, to one
 * communicator: ctxs[i] becomes rank i of n.  Non-blocking and bound by
 * timeout_ms, as pz_ctx_init_nccl_timeout. */
pz_status pz_multi_init_nccl(pz_sampler_ctx *const *ctxs, int n, int timeout_ms);

/* Samples a batch spread over n devices, from one host thread.
 *   PZ_SHARD_ROWS: shard i holds its own rows (pz_row_shard gives the even
 *     split); each is sampled exactly as pz_sample_batch(shard.ctx, ...)
 *     with `hints`; no communication.  Every shard has V == V_global and
 *     v_offset == 0.
 *   PZ_SHARD_VOCAB: every shard holds the same B rows, columns
 *     [v_offset, v_offset + V) of V_global, and its context was joined as
 *     rank i by pz_multi_init_nccl.  The local passes, ONE grouped
 *     allgather of the candidate lists and the merges run as in
 *     pz_sample_batch_vocab_sharded (same requirements; `hints` unused):
 *     every shard's out_tokens and rng_state receive the same values.
 * Asynchronous: returns once every device's work is queued on its stream
 * (pz_ctx_wait on each shard's context and stream waits for it). */
pz_status pz_sample_batch_multi(int mode, int n, const pz_shard *shards,
                                pz_dtype dtype, int V_global,
                                const pz_batch_hints *hints);

/* ------------------------------------------------------------------------ */
/* Settings from the front ends of the generate loop.                       */

/* One request's sampler settings as the front ends give them: the config a
 * row of pz_sample_batch takes, the RNG seed (-1: none given; the caller
 * picks one, as the reference does with time(NULL) at generate.c:126) and
 * the OpenAI-style logprob request. */
#define PZ_TOP_LOGPROBS_MAX 20
typedef struct pz_sampling_params {
  pz_sampler_config cfg;
  int64_t seed;
  int32_t logprobs;      /* 1: the sampled id's log-probability is wanted   */
  int32_t top_logprobs;  /* 0..PZ_TOP_LOGPROBS_MAX most likely ids as well   */
} pz_sampling_params;

/* Defaults of the command line (reference src/cli/args.c:82-89: T 0.7,
 * top-p 0.9, seed -1) and of an API request (src/api/json_parse.c:299-300:
 * T 1.0, top-p 1.0); no top-k, no penalties. */
void pz_params_init_cli(pz_sampling_params *p);
void pz_params_init_api(pz_sampling_params *p);
/* Command-line flags over the CLI defaults: the reference's --temperature,
 * --top-p (args.c:117-120) and --seed (args.c:125-126, which the reference
 * parses but never uses), plus --top-k, --repeat-penalty,
 * --frequency-penalty, --presence-penalty, --logprobs and --top-logprobs N.
 * Other flags are left to the caller's own parser. */
pz_status pz_params_from_args(pz_sampling_params *p, int argc, char **argv);
/* A chat-completions JSON body over the API defaults: "temperature" and
 * "top_p" (json_parse.c:344-347), plus "top_k", "repetition_penalty",
 * "frequency_penalty", "presence_penalty", "seed", "logprobs" and
 * "top_logprobs"; other keys are skipped.  Then the API's clamps
 * (http_server.c:415-417: T to [0, 2], top-p outside [0, 1] -> 1) and the
 * OpenAI ranges of the added fields (penalties to [-2, 2], top_logprobs to
 * [0, 20]).  PZ_ERR_INVALID_ARGS for a body that is not a JSON object. */
pz_status pz_params_from_json(pz_sampling_params *p, const char *json);

/* Library version string. */
const char *pz_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PZ_SAMPLING_H */
