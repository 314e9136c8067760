// pz_listmath.cuh — the reference's list arithmetic (softmax normaliser,
// cumulative probabilities, cutoff and CDF draw) over a short sorted list,
// computed by one warp: element-wise steps in parallel, each float sum in
// the reference's sequential order.
#pragma once

#include <climits>

#include "pz_seqsum.cuh"
#include "pz_warpsel.cuh"

namespace pz {

// Sorts lk[0..n) (distinct keys, n <= 64) descending in place, one warp:
// each key's position is the number of keys above it.
__device__ __forceinline__ void warp_rank_sort_desc(unsigned long long *lk, int n) {
  const int lane = static_cast<int>(lane_id());
  const unsigned long long k0 = lane < n ? lk[lane] : 0ull;
  const unsigned long long k1 = lane + 32 < n ? lk[lane + 32] : 0ull;
  int r0 = 0, r1 = 0;
  for (int j = 0; j < n; j++) {
    const unsigned long long o = lk[j];
    r0 += o > k0 ? 1 : 0;
    r1 += o > k1 ? 1 : 0;
  }
  __syncwarp();
  if (lane < n) lk[r0] = k0;
  if (lane + 32 < n) lk[r1] = k1;
  __syncwarp();
}

// The reference's list sampling over a sorted list of keff <= 64 entries
// (lk[0..n_sel) keys, the rest the reference's empty slots (-1e30, -1)),
// one warp: element-wise steps in parallel, each sequential float sum on
// lane 0 in the reference's order, searches by ballot.  p_on: reference
// src/sampling/top_p.c:37-105 on the list; else: src/sampling/top_k.c:50-72.
// `rs` advances by one draw unless the nucleus is empty.  e, c: shared
// scratch of 64 floats each.  Writes the list's probabilities to
// pr_out[0..keff) when pr_out is not null.  Returns INT_MIN if the
// probabilities are not in list order (the caller then uses the general
// path with its stable sort).
__device__ __noinline__ int warp_sample_small(const unsigned long long *lk, int n_sel, const RowPlan P,
                                              unsigned long long &rs, float *e, float *c,
                                              float *pr_out) {
  const int lane = static_cast<int>(lane_id());
  const int keff = P.keff;
  const int i0 = lane, i1 = lane + 32;
  const float v0 = i0 < n_sel ? key_val(lk[i0]) : -1e30f;
  const float v1 = i1 < n_sel ? key_val(lk[i1]) : -1e30f;
  const float mx = __shfl_sync(0xFFFFFFFFu, v0, 0);
  auto idv = [&](int i) -> int { return i < n_sel ? key_idx(lk[i]) : -1; };
  // lane 0's sequential sum of x[0..n) (unrolled so the loads run ahead)
  auto seq_sum = [&](const float *x, int n) -> float {
    float s = 0.0f;
    if (lane == 0) {
      int j = 0;
      for (; j + 4 <= n; j += 4) {
        const float a = x[j], b = x[j + 1], d = x[j + 2], f = x[j + 3];
        s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, a), b), d), f);
      }
      for (; j < n; j++) s = __fadd_rn(s, x[j]);
    }
    return __shfl_sync(0xFFFFFFFFu, s, 0);
  };
  // lane 0's running sums of x[0..n) into out[]; returns the first j with
  // out[j] >= stop (or n)
  // (four at a time, the loads ahead of the sums: the addends are not
  // negative, so the sums only grow and a block whose last sum is below
  // `stop` has no hit; sums past the hit are scratch)
  auto seq_cum = [&](const float *x, int n, float *out, float stop) -> int {
    int hit = n;
    if (lane == 0) {
      float s = 0.0f;
      int j = 0;
      for (; j + 4 <= n; j += 4) {
        const float a = x[j], b = x[j + 1], d = x[j + 2], f = x[j + 3];
        const float s1 = __fadd_rn(s, a), s2 = __fadd_rn(s1, b), s3 = __fadd_rn(s2, d), s4 = __fadd_rn(s3, f);
        out[j] = s1;
        out[j + 1] = s2;
        out[j + 2] = s3;
        out[j + 3] = s4;
        if (s4 >= stop) {
          hit = s1 >= stop ? j : s2 >= stop ? j + 1 : s3 >= stop ? j + 2 : j + 3;
          break;
        }
        s = s4;
      }
      if (hit == n) {
        for (; j < n; j++) {
          s = __fadd_rn(s, x[j]);
          out[j] = s;
          if (s >= stop) {
            hit = j;
            break;
          }
        }
      }
    }
    __syncwarp();
    return __shfl_sync(0xFFFFFFFFu, hit, 0);
  };
  // first j < n with r < cdf[j], or -1
  auto first_below = [&](const float *cdf, int n, float r) -> int {
    for (int base = 0; base < n; base += 32) {
      const int j = base + lane;
      const uint32_t b = __ballot_sync(0xFFFFFFFFu, j < n && r < cdf[j]);
      if (b) return base + __ffs(b) - 1;
    }
    return -1;
  };
  int tok;
  if (P.p_on) {
    const float thr = __fsub_rn(mx, 20.0f);                             // top_p.c:53
    const bool c0 = i0 < keff && v0 >= thr, c1 = i1 < keff && v1 >= thr;
    if (c0) e[i0] = cr_expf(__fsub_rn(v0, mx));                         // :58-59
    if (c1) e[i1] = cr_expf(__fsub_rn(v1, mx));
    // the list is sorted, so the kept entries are a prefix
    const uint32_t k0 = __ballot_sync(0xFFFFFFFFu, c0), k1 = __ballot_sync(0xFFFFFFFFu, c1);
    const int n = (~k0 != 0u) ? __ffs(~k0) - 1 : 32 + ((~k1 != 0u) ? __ffs(~k1) - 1 : 32);
    const int nk = n < keff ? n : keff;
    if (nk == 0) {                                                      // :68-69
      if (pr_out)
        for (int i = lane; i < keff; i += 32) pr_out[i] = 0.0f;
      return idv(0);
    }
    __syncwarp();
    const float sum = seq_sum(e, nk);                                   // :62
    const float inv = __fdiv_rn(1.0f, sum);                             // :72
    const float p0 = i0 < nk ? __fmul_rn(e[i0], inv) : 0.0f;            // :73-74
    const float p1 = i1 < nk ? __fmul_rn(e[i1], inv) : 0.0f;
    // stable sort by probability (:77) is the identity when they descend
    const float nx0 = __shfl_down_sync(0xFFFFFFFFu, p0, 1);
    const float nx1 = __shfl_down_sync(0xFFFFFFFFu, p1, 1);
    const float p1first = __shfl_sync(0xFFFFFFFFu, p1, 0);
    const bool up0 = i0 + 1 < nk && (lane < 31 ? nx0 : p1first) > p0;
    const bool up1 = i1 + 1 < nk && lane < 31 && nx1 > p1;
    if (__any_sync(0xFFFFFFFFu, up0 || up1)) return INT_MIN;
    __syncwarp();
    if (i0 < nk) e[i0] = p0;  // e now holds the probabilities
    if (i1 < nk) e[i1] = p1;
    __syncwarp();
    const int hit = seq_cum(e, nk, c, P.p);                             // :80-88
    const int cutoff = hit < nk ? hit + 1 : nk;
    const float trunc = c[cutoff - 1];                                  // :91-93
    const float r = __fmul_rn(rng_next(rs), trunc);                     // :96
    const int w = first_below(c, cutoff, r);                            // :98-105
    tok = idv(w >= 0 ? w : 0);
    if (pr_out) {
      if (i0 < keff) pr_out[i0] = p0;
      if (i1 < keff) pr_out[i1] = p1;
    }
  } else {
    if (i0 < keff) e[i0] = cr_expf(__fsub_rn(v0, mx));                  // top_k.c:54
    if (i1 < keff) e[i1] = cr_expf(__fsub_rn(v1, mx));
    __syncwarp();
    const float sum = seq_sum(e, keff);                                 // :55
    const float p0 = i0 < keff ? __fdiv_rn(e[i0], sum) : 0.0f;          // :57-59
    const float p1 = i1 < keff ? __fdiv_rn(e[i1], sum) : 0.0f;
    __syncwarp();
    if (i0 < keff) e[i0] = p0;
    if (i1 < keff) e[i1] = p1;
    __syncwarp();
    seq_cum(e, keff, c, INFINITY);
    const float r = rng_next(rs);                                       // :62
    const int w = first_below(c, keff, r);                              // :63-70
    tok = idv(w >= 0 ? w : 0);                                          // :72
    if (pr_out) {
      if (i0 < keff) pr_out[i0] = p0;
      if (i1 < keff) pr_out[i1] = p1;
    }
  }
  return tok;
}

// The same steps as sample_list (top_p.c:37-105 on the list, or
// top_k.c:50-72) for lists of any length up to PZ_TOP_K_MAX, one warp:
// element-wise steps lane-strided, each sequential float sum on lane 0 in
// the reference's order, eight terms at a time with the next eight loaded
// while the current ones are added, and the CDF searches by ballot.  e, c:
// shared scratch of keff floats each.  Returns INT_MIN, with rs untouched,
// if the probabilities are not in list order (the caller then runs
// sample_list, whose stable sort handles that case).
__device__ __noinline__ int warp_sample_long(const unsigned long long *lk, int n_sel, const RowPlan P,
                                             unsigned long long &rs, float *e, float *c, float *pr_out) {
  const int lane = static_cast<int>(lane_id());
  const int keff = P.keff;
  auto val = [&](int i) -> float { return i < n_sel ? key_val(lk[i]) : -1e30f; };
  auto idv = [&](int i) -> int { return i < n_sel ? key_idx(lk[i]) : -1; };
  const float mx = val(0);
  // lane 0's running sums of x[0..n), written to out[] when out is not
  // null; stops after the eight-term block holding the first sum >= stop
  // and returns that sum's index (n if none; sums past it are scratch), and
  // the last sum formed in *last
  auto seq_run = [&](const float *x, int n, float *out, float stop, float *last) -> int {
    int hit = n;
    float s = 0.0f;
    if (lane == 0) {
      float t[8];
      int j = 0;
      if (n >= 8) {
#pragma unroll
        for (int q = 0; q < 8; q++) t[q] = x[q];
      }
      for (; j + 8 <= n; j += 8) {
        float u[8];
        const bool more = j + 16 <= n;
        if (more) {
#pragma unroll
          for (int q = 0; q < 8; q++) u[q] = x[j + 8 + q];
        }
        float ss[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
          s = __fadd_rn(s, t[q]);
          ss[q] = s;
        }
        if (out != nullptr) {
#pragma unroll
          for (int q = 0; q < 8; q++) out[j + q] = ss[q];
        }
        if (ss[7] >= stop) {
          // the sums only grow (the terms are not negative): the first hit is in this block
          int h = j + 7;
#pragma unroll
          for (int q = 6; q >= 0; q--)
            if (ss[q] >= stop) h = j + q;
          hit = h;
          break;
        }
        if (more) {
#pragma unroll
          for (int q = 0; q < 8; q++) t[q] = u[q];
        }
      }
      if (hit == n) {
        for (; j < n; j++) {
          s = __fadd_rn(s, x[j]);
          if (out != nullptr) out[j] = s;
          if (s >= stop) {
            hit = j;
            break;
          }
        }
      }
    }
    __syncwarp();
    *last = __shfl_sync(0xFFFFFFFFu, s, 0);
    return __shfl_sync(0xFFFFFFFFu, hit, 0);
  };
  // first j < n with r < cdf[j], or -1
  auto first_below = [&](const float *cdf, int n, float r) -> int {
    for (int base = 0; base < n; base += 32) {
      const int j = base + lane;
      const uint32_t b = __ballot_sync(0xFFFFFFFFu, j < n && r < cdf[j]);
      if (b) return base + __ffs(b) - 1;
    }
    return -1;
  };
  int tok;
  float s_last;
  if (P.p_on) {
    const float thr = __fsub_rn(mx, 20.0f);                             // top_p.c:53
    for (int i = lane; i < keff; i += 32) {
      const float v = val(i);
      e[i] = (v >= thr) ? cr_expf(__fsub_rn(v, mx)) : -1.0f;            // :58-59
    }
    __syncwarp();
    // the entries the filter keeps lead the list (it is sorted by value)
    int n = keff;
    for (int base = 0; base < keff; base += 32) {
      const int i = base + lane;
      const uint32_t b = __ballot_sync(0xFFFFFFFFu, i < keff && !(e[i] >= 0.0f));
      if (b) {
        n = base + __ffs(b) - 1;
        break;
      }
    }
    if (n == 0) {                                                       // :68-69
      if (pr_out)
        for (int i = lane; i < keff; i += 32) pr_out[i] = 0.0f;
      return idv(0);
    }
    seq_run(e, n, nullptr, INFINITY, &s_last);                          // :62
    const float inv = __fdiv_rn(1.0f, s_last);                          // :72
    // stable sort by probability (:77) is the identity when they descend
    bool up = false;
    for (int i = lane; i < n; i += 32)
      if (i > 0 && __fmul_rn(e[i], inv) > __fmul_rn(e[i - 1], inv)) up = true;
    if (__any_sync(0xFFFFFFFFu, up)) return INT_MIN;
    __syncwarp();
    for (int i = lane; i < n; i += 32) e[i] = __fmul_rn(e[i], inv);     // :73-74
    __syncwarp();
    const int hit = seq_run(e, n, c, P.p, &s_last);                     // :80-88
    const int cutoff = hit < n ? hit + 1 : n;
    const float trunc = c[cutoff - 1];                                  // :91-93
    const float r = __fmul_rn(rng_next(rs), trunc);                     // :96
    const int w = first_below(c, cutoff, r);                            // :98-105
    tok = idv(w >= 0 ? w : 0);
    if (pr_out)
      for (int i = lane; i < keff; i += 32) pr_out[i] = i < n ? e[i] : 0.0f;
  } else {
    for (int i = lane; i < keff; i += 32) e[i] = cr_expf(__fsub_rn(val(i), mx));  // top_k.c:54
    __syncwarp();
    seq_run(e, keff, nullptr, INFINITY, &s_last);                       // :55
    const float sum = s_last;
    const float r = rng_next(rs);                                       // :62
    for (int i = lane; i < keff; i += 32) e[i] = __fdiv_rn(e[i], sum);  // :57-59
    __syncwarp();
    seq_run(e, keff, c, INFINITY, &s_last);
    const int w = first_below(c, keff, r);                              // :63-70
    tok = idv(w >= 0 ? w : 0);                                          // :72
    if (pr_out)
      for (int i = lane; i < keff; i += 32) pr_out[i] = e[i];
  }
  return tok;
}

}  // namespace pz
