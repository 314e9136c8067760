/*
 * ref_pipeline.c — drives the REFERENCE's own compiled sampler through the
 * pipeline contract (TEST INFRASTRUCTURE ONLY).
 *
 * Built by oracle/Makefile together with the reference's unmodified sources
 * (src/sampling/{rng,argmax,temperature,top_k,top_p}.c and
 * src/math/softmax*.c, compiled where they lie with the reference's release
 * flags -std=c99 -O3 -march=native) into oracle/_ref/libpzref.so.  Nothing
 * from the reference is copied into this repository.
 *
 * Stage by stage:
 *   A8 penalties            contract code (pz_contract.h) — no reference code
 *   A7 greedy               sample_argmax            (argmax.c:3-13)
 *   A3 temperature          apply_temperature        (temperature.c:8-25)
 *   k_eff = 0, 0 < p < 1    sample_top_p on the row  (top_p.c:30-108)
 *   k_eff = 0, otherwise    tn_softmax's kernel + the CDF walk of
 *                           generate.c:158-168 (the walk is restated: it is
 *                           inline in the reference's generate loop)
 *   k_eff >= 1, p off       sample_top_k on the row  (top_k.c:8-73)
 *   k_eff >= 1, 0 < p < 1   the selection loop of top_k.c:27-48 (restated in
 *                           pz_contract.h: the reference fuses it with its
 *                           draw), then sample_top_p on the sorted list.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "core/platform.h"
#include "math/softmax.h"
#include "sampling/rng.h"
#include "sampling/sampling.h"

#include "../include/pz_sampling.h"
#include "pz_contract.h"

#if TN_HAS_AVX512
extern void softmax_avx512(float *x, int size);
#define PZR_SOFTMAX softmax_avx512
#define PZR_SOFTMAX_NAME "softmax_avx512"
#elif TN_HAS_AVX2
extern void softmax_avx2(float *x, int size);
#define PZR_SOFTMAX softmax_avx2
#define PZR_SOFTMAX_NAME "softmax_avx2"
#else
#define PZR_SOFTMAX softmax
#define PZR_SOFTMAX_NAME "softmax"
#endif

/* Which reference branches this build compiled: bit 0 = TN_HAS_AVX512
 * (apply_temperature multiplies by 1/T when set, divides when clear). */
int pzr_build_info(void) { return TN_HAS_AVX512 ? 1 : 0; }
const char *pzr_softmax_kernel(void) { return PZR_SOFTMAX_NAME; }

/* Direct access to the six reference calls, for the golden-vector script. */
int pzr_sample_argmax(const float *x, int V) { return sample_argmax(x, V); }
void pzr_apply_temperature(float *x, int V, float T) {
  apply_temperature(x, V, T);
}
int pzr_sample_top_p(float *x, int V, float p, unsigned long long *rng) {
  return sample_top_p(x, V, p, rng);
}
int pzr_sample_top_k(float *x, int V, int k, unsigned long long *rng) {
  return sample_top_k(x, V, k, rng);
}
void pzr_rng_seed(unsigned long long *s, unsigned long long seed) {
  rng_seed(s, seed);
}
float pzr_rng_float(unsigned long long *s) { return rng_float(s); }

/* generate.c:157-168 with the dispatched softmax kernel. */
int pzr_sample_softmax(float *x, int V, unsigned long long *rng) {
  PZR_SOFTMAX(x, V);
  float r = rng_float(rng);
  float cdf = 0.0f;
  int next = V - 1;
  for (int i = 0; i < V; i++) {
    cdf += x[i];
    if (r < cdf) {
      next = i;
      break;
    }
  }
  return next;
}

static int ref_row(float *x, int V, const pz_sampler_config *cfg,
                   const int32_t *hist, int H, unsigned long long *rng) {
  const float rep = cfg->repetition_penalty;
  const float freq = cfg->frequency_penalty;
  const float pres = cfg->presence_penalty;
  if (H > 0 && (rep != 1.0f || freq != 0.0f || pres != 0.0f))
    pzc_apply_penalties(x, V, hist, H, rep, freq, pres);
  const float T = cfg->temperature;
  if (T <= 0.0f || T < 1e-6f) return sample_argmax(x, V);
  apply_temperature(x, V, T);
  const int keff = pzc_k_eff(cfg->top_k, V);
  const float p = cfg->top_p;
  const int p_on = (p < 1.0f && p > 0.0f);
  if (keff == 0) {
    if (p_on) return sample_top_p(x, V, p, rng);
    return pzr_sample_softmax(x, V, rng);
  }
  if (!p_on) return sample_top_k(x, V, keff, rng);
  float vals[1024];
  int32_t indices[1024];
  pzc_select_top_k(x, V, keff, vals, indices);
  const int pos = sample_top_p(vals, keff, p, rng);
  return indices[pos];
}

/* Same contract and signature as pzo_sample_batch (without the candidate
 * outputs, which the reference cannot produce). */
int pzr_sample_batch(const void *logits, int dtype, int B, int V, int64_t ld,
                     const pz_sampler_config *cfg, const int32_t *hist,
                     const int32_t *hist_off, unsigned long long *rng,
                     int32_t *out) {
  if (B < 0 || V <= 0 || ld < V || !logits || !cfg || !rng || !out) return -1;
  if (dtype != 0 && dtype != 1) return -1;
  float *x = (float *)malloc((size_t)V * sizeof(float));
  if (!x) return -1;
  for (int r = 0; r < B; r++) {
    if (dtype == 0) {
      memcpy(x, (const float *)logits + (size_t)r * (size_t)ld,
             (size_t)V * sizeof(float));
    } else {
      const uint16_t *src = (const uint16_t *)logits + (size_t)r * (size_t)ld;
      for (int i = 0; i < V; i++) x[i] = pzc_bf16_to_f32(src[i]);
    }
    const int32_t *h = NULL;
    int H = 0;
    if (hist && hist_off) {
      h = hist + hist_off[r];
      H = hist_off[r + 1] - hist_off[r];
    }
    out[r] = ref_row(x, V, &cfg[r], h, H, &rng[r]);
  }
  free(x);
  return 0;
}
