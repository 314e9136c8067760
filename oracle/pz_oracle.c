/*
 * pz_oracle.c — CPU restatement of Project Zero's sampler (TEST
 * INFRASTRUCTURE ONLY; see pz_oracle.h).  Build: oracle/Makefile, with
 * -std=c99 -O2 -ffp-contract=off.  libm expf and the reference's float
 * operation order are used throughout so the results are the reference's
 * bits.
 */
#include "pz_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "pz_contract.h"

/* reference src/sampling/rng.c:3-6 */
void pzo_rng_seed(uint64_t *state, uint64_t seed) {
  *state = (seed == 0) ? 1 : seed;
}

/* reference src/sampling/rng.c:8-17: xorshift64* (12/25/27), the top 31
 * bits of s * 0x2545F4914F6CDD1D converted to float (round to nearest) and
 * divided by 2^31.  The result can be exactly 1.0f. */
float pzo_rng_float(uint64_t *state) {
  uint64_t s = *state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  *state = s;
  return (float)((s * 0x2545F4914F6CDD1DULL) >> 33) / (float)(1u << 31);
}

/* reference src/sampling/argmax.c:3-13 */
int pzo_sample_argmax(const float *logits, int V) {
  int best_idx = 0;
  float best_val = logits[0];
  for (int i = 1; i < V; i++) {
    if (logits[i] > best_val) {
      best_val = logits[i];
      best_idx = i;
    }
  }
  return best_idx;
}

/* reference src/sampling/temperature.c:8-25.  divide=0 is the AVX-512 build
 * (x *= 1/T, :11-20), divide=1 the scalar build (x /= T, :22-23). */
void pzo_apply_temperature(float *logits, int V, float T, int divide) {
  if (T < 1e-6f) T = 1e-6f;
  if (!divide) {
    const float inv = 1.0f / T;
    for (int i = 0; i < V; i++) logits[i] *= inv;
  } else {
    for (int i = 0; i < V; i++) logits[i] /= T;
  }
}

/* Softmax and draw over a sorted top-k list: reference
 * src/sampling/top_k.c:50-72 (division by the sum, fallback entry 0). */
static int list_softmax_draw(float *vals, const int32_t *indices, int k,
                             uint64_t *rng) {
  const float max_val = vals[0];
  float sum = 0.0f;
  for (int i = 0; i < k; i++) {
    vals[i] = expf(vals[i] - max_val);
    sum += vals[i];
  }
  for (int i = 0; i < k; i++) vals[i] /= sum;
  const float r = pzo_rng_float(rng);
  float cdf = 0.0f;
  for (int i = 0; i < k; i++) {
    cdf += vals[i];
    if (r < cdf) return indices[i];
  }
  return indices[0];
}

/* reference src/sampling/top_k.c:8-73 */
int pzo_sample_top_k(const float *logits, int V, int k, uint64_t *rng) {
  if (k > V) k = V;
  if (k <= 0) k = 1;
  if (k > 1024) k = 1024;
  float vals[1024];
  int32_t indices[1024];
  pzc_select_top_k(logits, V, k, vals, indices);
  return list_softmax_draw(vals, indices, k, rng);
}

typedef struct {
  float prob;
  int index;
} prob_index;

/* Stable sort by prob descending: glibc 2.39's qsort (used by reference
 * src/sampling/top_p.c:77 with compare_prob_desc, :12-20) is a stable
 * mergesort, so equal probabilities keep index order.  This is a bottom-up
 * mergesort with the same comparison. */
static void stable_sort_desc(prob_index *a, int n, prob_index *tmp) {
  for (int width = 1; width < n; width *= 2) {
    for (int lo = 0; lo < n; lo += 2 * width) {
      int mid = lo + width < n ? lo + width : n;
      int hi = lo + 2 * width < n ? lo + 2 * width : n;
      int i = lo, j = mid, o = lo;
      while (i < mid && j < hi) {
        /* take from the right run only if strictly greater */
        if (a[j].prob > a[i].prob)
          tmp[o++] = a[j++];
        else
          tmp[o++] = a[i++];
      }
      while (i < mid) tmp[o++] = a[i++];
      while (j < hi) tmp[o++] = a[j++];
    }
    memcpy(a, tmp, (size_t)n * sizeof *a);
  }
}

/* The steps of reference src/sampling/top_p.c:37-105 over an array of n
 * values (the whole row, or a sorted top-k list).  Returns a position in
 * that array.  probs_out (may be NULL) receives each position's normalised
 * probability (0 where the max-20 filter dropped it). */
static int top_p_steps(const float *logits, int V, float top_p, uint64_t *rng,
                       float *probs_out) {
  /* :37-41 */
  float max_val = logits[0];
  for (int i = 1; i < V; i++)
    if (logits[i] > max_val) max_val = logits[i];
  /* :53-65 */
  const float log_threshold = max_val - 20.0f;
  prob_index *c = (prob_index *)malloc((size_t)(V > 0 ? V : 1) * sizeof *c);
  prob_index *tmp = (prob_index *)malloc((size_t)(V > 0 ? V : 1) * sizeof *tmp);
  if (!c || !tmp) abort();
  int n = 0;
  float sum = 0.0f;
  for (int i = 0; i < V; i++) {
    if (logits[i] >= log_threshold) {
      const float e = expf(logits[i] - max_val);
      c[n].prob = e;
      c[n].index = i;
      sum += e;
      n++;
    }
  }
  if (probs_out)
    for (int i = 0; i < V; i++) probs_out[i] = 0.0f;
  /* :68-69 */
  if (n == 0) {
    free(c);
    free(tmp);
    return pzo_sample_argmax(logits, V);
  }
  /* :72-74 */
  const float inv_sum = 1.0f / sum;
  for (int i = 0; i < n; i++) c[i].prob *= inv_sum;
  if (probs_out)
    for (int i = 0; i < n; i++) probs_out[c[i].index] = c[i].prob;
  /* :77 */
  stable_sort_desc(c, n, tmp);
  /* :80-88 */
  float cumulative = 0.0f;
  int cutoff = n;
  for (int i = 0; i < n; i++) {
    cumulative += c[i].prob;
    if (cumulative >= top_p) {
      cutoff = i + 1;
      break;
    }
  }
  /* :91-93 */
  float trunc_sum = 0.0f;
  for (int i = 0; i < cutoff; i++) trunc_sum += c[i].prob;
  /* :96-105 */
  const float r = pzo_rng_float(rng) * trunc_sum;
  float cdf = 0.0f;
  int result = c[0].index;
  for (int i = 0; i < cutoff; i++) {
    cdf += c[i].prob;
    if (r < cdf) {
      result = c[i].index;
      break;
    }
  }
  free(c);
  free(tmp);
  return result;
}

/* reference src/sampling/top_p.c:30-108 */
int pzo_sample_top_p(const float *logits, int V, float p, uint64_t *rng) {
  if (V > 200000) return pzo_sample_argmax(logits, V); /* :33-34 */
  return top_p_steps(logits, V, p, rng, NULL);
}

/* reference src/math/softmax.c:4-23 followed by the CDF walk of
 * src/transformer/generate.c:158-168 (fallback V-1). */
int pzo_sample_softmax(float *x, int V, uint64_t *rng) {
  float max_val = x[0];
  for (int i = 1; i < V; i++)
    if (x[i] > max_val) max_val = x[i];
  float sum = 0.0f;
  for (int i = 0; i < V; i++) {
    x[i] = expf(x[i] - max_val);
    sum += x[i];
  }
  const float inv_sum = 1.0f / sum;
  for (int i = 0; i < V; i++) x[i] *= inv_sum;
  const float r = pzo_rng_float(rng);
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

void pzo_apply_penalties(float *x, int V, const int32_t *hist, int H,
                         float rep, float freq, float pres) {
  pzc_apply_penalties(x, V, hist, H, rep, freq, pres);
}

/* One pipeline row: the contract of include/pz_sampling.h. */
int pzo_sample_row(float *x, int V, const pz_sampler_config *cfg,
                   const int32_t *hist, int H, uint64_t *rng,
                   int32_t *cand_ids, float *cand_probs, int32_t *n_cand) {
  if (n_cand) *n_cand = 0;
  const float rep = cfg->repetition_penalty;
  const float freq = cfg->frequency_penalty;
  const float pres = cfg->presence_penalty;
  if (H > 0 && (rep != 1.0f || freq != 0.0f || pres != 0.0f))
    pzc_apply_penalties(x, V, hist, H, rep, freq, pres);
  /* generate.c:151-152 */
  const float T = cfg->temperature;
  if (T <= 0.0f || T < 1e-6f) return pzo_sample_argmax(x, V);
  /* generate.c:154 */
  pzo_apply_temperature(x, V, T, (cfg->flags & PZ_CFG_TEMP_DIVIDE) != 0);
  const int keff = pzc_k_eff(cfg->top_k, V);
  const float p = cfg->top_p;
  const int p_on = (p < 1.0f && p > 0.0f); /* generate.c:155 */
  if (keff == 0)
    return p_on ? pzo_sample_top_p(x, V, p, rng) : pzo_sample_softmax(x, V, rng);

  float vals[1024];
  int32_t indices[1024];
  pzc_select_top_k(x, V, keff, vals, indices);
  if (n_cand) *n_cand = keff;
  if (cand_ids)
    for (int i = 0; i < keff; i++) cand_ids[i] = indices[i];
  if (p_on) {
    float probs[1024];
    const int pos = top_p_steps(vals, keff, p, rng, probs);
    if (cand_probs)
      for (int i = 0; i < keff; i++) cand_probs[i] = probs[i];
    return indices[pos];
  }
  /* list softmax of top_k.c:50-72, probabilities kept for the output */
  {
    const float max_val = vals[0];
    float sum = 0.0f;
    for (int i = 0; i < keff; i++) {
      vals[i] = expf(vals[i] - max_val);
      sum += vals[i];
    }
    for (int i = 0; i < keff; i++) vals[i] /= sum;
    if (cand_probs)
      for (int i = 0; i < keff; i++) cand_probs[i] = vals[i];
    const float r = pzo_rng_float(rng);
    float cdf = 0.0f;
    for (int i = 0; i < keff; i++) {
      cdf += vals[i];
      if (r < cdf) return indices[i];
    }
    return indices[0];
  }
}

int pzo_sample_batch(const void *logits, int dtype, int B, int V, int64_t ld,
                     const pz_sampler_config *cfg, const int32_t *hist,
                     const int32_t *hist_off, uint64_t *rng, int32_t *out,
                     int32_t *cand_ids, float *cand_probs, int32_t *n_cand,
                     int cand_stride) {
  if (B < 0 || V <= 0 || ld < V || !logits || !cfg || !rng || !out) return -1;
  if ((dtype != 0 && dtype != 1)) return -1;
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
    out[r] = pzo_sample_row(
        x, V, &cfg[r], h, H, &rng[r],
        cand_ids ? cand_ids + (size_t)r * (size_t)cand_stride : NULL,
        cand_probs ? cand_probs + (size_t)r * (size_t)cand_stride : NULL,
        n_cand ? n_cand + r : NULL);
  }
  free(x);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Draw trace of one pipeline row (test support for boundary cases).
 *
 * Runs the same steps as pzo_sample_row and records the walk the draw makes:
 * order[j] is the id at walk position j, cdf[j] the running float sum the
 * reference compares the draw with at that position (top_p.c:96-105,
 * top_k.c:62-70, generate.c:159-167), r the draw as compared (u * trunc_sum
 * for top-p, u otherwise), and *fallback the id taken when r reaches past
 * the last position.  *n_walk is the number of positions (0: no draw, the
 * token comes from argmax).  order and cdf hold at least V entries.
 * Returns the sampled id. */
static int walk_list(const float *probs, const int32_t *ids, int n, float r,
                     int32_t *order, float *cdf, int *n_walk) {
  float c = 0.0f;
  int res = -1;
  for (int i = 0; i < n; i++) {
    c += probs[i];
    order[i] = ids[i];
    cdf[i] = c;
    if (res < 0 && r < c) res = ids[i];
  }
  *n_walk = n;
  return res;
}

int pzo_row_trace(const float *x_in, int V, const pz_sampler_config *cfg,
                  const int32_t *hist, int H, uint64_t rng, float *r_out,
                  int32_t *order, float *cdf, int *n_walk, int32_t *fallback) {
  float *x = (float *)malloc((size_t)V * sizeof(float));
  if (!x) abort();
  memcpy(x, x_in, (size_t)V * sizeof(float));
  *n_walk = 0;
  *r_out = 0.0f;
  *fallback = -1;
  int tok = -1;
  const float rep = cfg->repetition_penalty, freq = cfg->frequency_penalty,
              pres = cfg->presence_penalty;
  if (H > 0 && (rep != 1.0f || freq != 0.0f || pres != 0.0f))
    pzc_apply_penalties(x, V, hist, H, rep, freq, pres);
  const float T = cfg->temperature;
  if (T <= 0.0f || T < 1e-6f) {
    tok = pzo_sample_argmax(x, V);
    free(x);
    return tok;
  }
  pzo_apply_temperature(x, V, T, (cfg->flags & PZ_CFG_TEMP_DIVIDE) != 0);
  const int keff = pzc_k_eff(cfg->top_k, V);
  const float p = cfg->top_p;
  const int p_on = (p < 1.0f && p > 0.0f);
  float *vals = x; /* the array the top-p steps run over */
  int n_vals = V;
  int32_t *ids = (int32_t *)malloc((size_t)V * sizeof(int32_t));
  float *lv = (float *)malloc((size_t)V * sizeof(float));
  prob_index *c = (prob_index *)malloc((size_t)V * sizeof *c);
  prob_index *tmp = (prob_index *)malloc((size_t)V * sizeof *tmp);
  float *pr = (float *)malloc((size_t)V * sizeof(float));
  if (!ids || !lv || !c || !tmp || !pr) abort();
  if (keff > 0) {
    pzc_select_top_k(x, V, keff, lv, ids);
    vals = lv;
    n_vals = keff;
  } else {
    for (int i = 0; i < V; i++) ids[i] = i;
  }
  if (keff == 0 && !p_on) {
    /* softmax over the row, CDF walk in index order, fallback V-1 */
    float mx = x[0];
    for (int i = 1; i < V; i++)
      if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < V; i++) {
      x[i] = expf(x[i] - mx);
      sum += x[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < V; i++) x[i] *= inv;
    const float r = pzo_rng_float(&rng);
    *r_out = r;
    *fallback = V - 1;
    tok = walk_list(x, ids, V, r, order, cdf, n_walk);
    if (tok < 0) tok = V - 1;
  } else if (keff > 0 && !p_on) {
    /* top_k.c:50-72 over the list, fallback indices[0] */
    const float mx = vals[0];
    float sum = 0.0f;
    for (int i = 0; i < keff; i++) {
      vals[i] = expf(vals[i] - mx);
      sum += vals[i];
    }
    for (int i = 0; i < keff; i++) vals[i] /= sum;
    const float r = pzo_rng_float(&rng);
    *r_out = r;
    *fallback = ids[0];
    tok = walk_list(vals, ids, keff, r, order, cdf, n_walk);
    if (tok < 0) tok = ids[0];
  } else if (keff == 0 && V > 200000) {
    tok = pzo_sample_argmax(x, V); /* top_p.c:33-34 */
  } else {
    /* top_p.c:37-105 over vals[0..n_vals) */
    float mx = vals[0];
    for (int i = 1; i < n_vals; i++)
      if (vals[i] > mx) mx = vals[i];
    const float thr = mx - 20.0f;
    int n = 0;
    float sum = 0.0f;
    for (int i = 0; i < n_vals; i++) {
      if (vals[i] >= thr) {
        const float e = expf(vals[i] - mx);
        c[n].prob = e;
        c[n].index = ids[i];
        sum += e;
        n++;
      }
    }
    if (n == 0) {
      tok = ids[pzo_sample_argmax(vals, n_vals)];
    } else {
      const float inv = 1.0f / sum;
      for (int i = 0; i < n; i++) c[i].prob *= inv;
      stable_sort_desc(c, n, tmp);
      float cum = 0.0f;
      int cutoff = n;
      for (int i = 0; i < n; i++) {
        cum += c[i].prob;
        if (cum >= p) {
          cutoff = i + 1;
          break;
        }
      }
      float trunc = 0.0f;
      for (int i = 0; i < cutoff; i++) trunc += c[i].prob;
      const float r = pzo_rng_float(&rng) * trunc;
      *r_out = r;
      *fallback = c[0].index;
      for (int i = 0; i < cutoff; i++) {
        pr[i] = c[i].prob;
        ids[i] = c[i].index;
      }
      tok = walk_list(pr, ids, cutoff, r, order, cdf, n_walk);
      if (tok < 0) tok = c[0].index;
    }
  }
  free(x);
  free(ids);
  free(lv);
  free(c);
  free(tmp);
  free(pr);
  return tok;
}
