/*
 * pz_contract.h — the pipeline stages the reference does not have, written
 * once and shared by the CPU restatement (pz_oracle.c) and the driver that
 * runs the reference's own compiled sampler (ref_pipeline.c).  TEST
 * INFRASTRUCTURE ONLY.
 *
 *   - A8 penalties over a history window (project contract; parity is
 *     pinned against this code, not against the reference);
 *   - the top-k selection loop that the composition top-k -> top-p needs as
 *     a separate step.  It is the insertion selection of reference
 *     src/sampling/top_k.c:27-48 (the reference only exposes it fused with
 *     its own softmax and draw).
 *
 * Compile with -ffp-contract=off: every float operation below rounds on its
 * own, in the order written.
 */
#ifndef PZ_CONTRACT_H
#define PZ_CONTRACT_H

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static int pzc_cmp_i32(const void *a, const void *b) {
  int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
  return (x > y) - (x < y);
}

/* A8: for each distinct id t in hist[0..H) with count c, ids outside [0,V)
 * ignored:
 *   if (rep != 1) x[t] = x[t] > 0 ? x[t] / rep : x[t] * rep;
 *   pen = (float)c * freq;  pen = pen + pres;  x[t] = x[t] - pen; */
static void pzc_apply_penalties(float *x, int V, const int32_t *hist, int H,
                                float rep, float freq, float pres) {
  if (H <= 0 || hist == NULL) return;
  int32_t *ids = (int32_t *)malloc((size_t)H * sizeof(int32_t));
  if (!ids) abort();
  int n = 0;
  for (int j = 0; j < H; j++)
    if (hist[j] >= 0 && hist[j] < V) ids[n++] = hist[j];
  qsort(ids, (size_t)n, sizeof(int32_t), pzc_cmp_i32);
  for (int i = 0; i < n;) {
    int j = i;
    while (j < n && ids[j] == ids[i]) j++;
    const int32_t t = ids[i];
    const int c = j - i;
    float v = x[t];
    if (rep != 1.0f) v = (v > 0.0f) ? v / rep : v * rep;
    float pen = (float)c * freq;
    pen = pen + pres;
    v = v - pen;
    x[t] = v;
    i = j;
  }
  free(ids);
}

/* Top-k selection of reference src/sampling/top_k.c:27-48 with k already
 * clamped to [1, 1024]: vals/indices sorted by value descending, the lower
 * index first among equal values, only entries > -1e30 admitted, unused
 * slots left as (-1e30, -1). */
static void pzc_select_top_k(const float *x, int V, int k, float *vals,
                             int32_t *indices) {
  for (int i = 0; i < k; i++) {
    indices[i] = -1;
    vals[i] = -1e30f;
  }
  for (int i = 0; i < V; i++) {
    if (x[i] > vals[k - 1]) {
      int j = k - 1;
      while (j > 0 && x[i] > vals[j - 1]) {
        vals[j] = vals[j - 1];
        indices[j] = indices[j - 1];
        j--;
      }
      vals[j] = x[i];
      indices[j] = i;
    }
  }
}

/* k_eff of the pipeline: 0 disables top-k (k <= 0 or k >= V), else k
 * clamped to 1024 (top_k.c:17-18). */
static int pzc_k_eff(int k, int V) {
  if (k <= 0 || k >= V) return 0;
  return k > 1024 ? 1024 : k;
}

/* bf16 bits -> fp32, exact. */
static float pzc_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

#endif /* PZ_CONTRACT_H */
