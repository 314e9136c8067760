/*
 * pz_oracle.h — CPU restatement of Project Zero's sampler, TEST
 * INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this code, and only as the checker.  The product (libpz_sampling.so) never
 * links or calls it.
 *
 * Every function restates one reference function (file:line given at each
 * definition) in plain C99, built with -ffp-contract=off so that each float
 * operation rounds exactly where the reference's does.  The pipeline
 * (pzo_sample_row) adds the stages the reference lacks (penalties, the
 * top-k -> top-p composition, bf16 widening) per the contract written in
 * include/pz_sampling.h.
 *
 * Pinning: the restatement is checked bit-for-bit against the reference's
 * own sources compiled into oracle/_ref (see oracle/Makefile) and against
 * the committed golden vectors in tests/golden/.
 */
#ifndef PZ_ORACLE_H
#define PZ_ORACLE_H

#include <stdint.h>

#include "../include/pz_sampling.h"

#ifdef __cplusplus
extern "C" {
#endif

void pzo_rng_seed(uint64_t *state, uint64_t seed);
float pzo_rng_float(uint64_t *state);
int pzo_sample_argmax(const float *logits, int V);
/* divide = 0: x *= 1/T (AVX-512 build); divide = 1: x /= T (scalar build) */
void pzo_apply_temperature(float *logits, int V, float T, int divide);
int pzo_sample_top_k(const float *logits, int V, int k, uint64_t *rng);
int pzo_sample_top_p(const float *logits, int V, float p, uint64_t *rng);
/* softmax in place + CDF walk in index order (generate.c:157-168) */
int pzo_sample_softmax(float *x, int V, uint64_t *rng);

/* One pipeline row.  `x` is the fp32 row (already widened) and is used as
 * working storage (overwritten).  cand_ids/cand_probs (may be NULL) receive
 * the top-k list and its probabilities for rows with k_eff >= 1 (at most
 * 1024 entries); *n_cand gets their count (0 for other rows). */
int pzo_sample_row(float *x, int V, const pz_sampler_config *cfg,
                   const int32_t *hist, int H, uint64_t *rng,
                   int32_t *cand_ids, float *cand_probs, int32_t *n_cand);

/* B rows; logits fp32 (dtype 0) or bf16 bits (dtype 1), row r at
 * logits + r*ld elements.  hist/hist_off may be NULL.  cand arrays are
 * [B x cand_stride] and may be NULL.  Returns 0, or -1 on bad arguments. */
int pzo_sample_batch(const void *logits, int dtype, int B, int V, int64_t ld,
                     const pz_sampler_config *cfg, const int32_t *hist,
                     const int32_t *hist_off, uint64_t *rng, int32_t *out,
                     int32_t *cand_ids, float *cand_probs, int32_t *n_cand,
                     int cand_stride);

/* The draw of one pipeline row, traced: walk order, running CDF, the draw
 * as compared, and the fallback id (see pz_oracle.c).  x_in is not
 * modified; `rng` is the row's state before the call. */
int pzo_row_trace(const float *x_in, int V, const pz_sampler_config *cfg,
                  const int32_t *hist, int H, uint64_t rng, float *r_out,
                  int32_t *order, float *cdf, int *n_walk, int32_t *fallback);

/* Penalty stage alone (A8), exposed for tests: applies the contract to x. */
void pzo_apply_penalties(float *x, int V, const int32_t *hist, int H,
                         float rep, float freq, float pres);

#ifdef __cplusplus
}
#endif

#endif /* PZ_ORACLE_H */
