// pz_listmath.cuh — the reference's list arithmetic (softmax normaliser,
// cumulative probabilities, cutoff and CDF draw) over a short sorted list,
// computed by one warp in parallel but rounding exactly like the
// reference's sequential float loops (warp-level form of pz_seqsum.cuh).
//
// Element j of the list lives in lane j / R, slot j % R.
#pragma once

#include <climits>

#include "pz_seqsum.cuh"
#include "pz_warpsel.cuh"

namespace pz {

__device__ __forceinline__ SeqMap warp_exscan_map(SeqMap v) {
  const int lane = static_cast<int>(lane_id());
  SeqMap incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    SeqMap w;
    w.e = __shfl_up_sync(0xFFFFFFFFu, incl.e, o);
    w.o = __shfl_up_sync(0xFFFFFFFFu, incl.o, o);
    if (lane >= o) incl = seq_compose(w, incl);
  }
  SeqMap ex;
  ex.e = __shfl_up_sync(0xFFFFFFFFu, incl.e, 1);
  ex.o = __shfl_up_sync(0xFFFFFFFFu, incl.o, 1);
  if (lane == 0) ex = seq_identity();
  return ex;
}

// pref[r] = s_j where s_j = fl(s_{j-1} + x_j), s_{-1} = 0, for j < n.
template <int R>
__device__ void warp_seq_prefix(const float (&x)[R], int n, float (&pref)[R]) {
  const int lane = static_cast<int>(lane_id());
  float s = 0.0f;
  int start = 0;
  for (int guard = 0; guard < 32 * R + 1; guard++) {
    const int eu = seq_grid_exp(s);
    const unsigned long long N0 = seq_N(s);
    SeqMap f[R];
    SeqMap F = seq_identity();
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int j = lane * R + r;
      f[r] = (j >= start && j < n) ? seq_elem(x[r], eu) : seq_identity();
      F = seq_compose(F, f[r]);
    }
    const SeqMap P = warp_exscan_map(F);
    unsigned long long N = seq_apply(P, N0);
    int cross = INT_MAX;
    unsigned long long Nc = 0;
    float xc = 0.0f;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int j = lane * R + r;
      if (j >= start && j < n && cross == INT_MAX) {
        const unsigned long long Nn = seq_apply(f[r], N);
        if (Nn >= kSeqLimit) {
          cross = j;
          Nc = N;
          xc = x[r];
        } else {
          pref[r] = seq_float(Nn, eu);
        }
        N = Nn;
      }
    }
    int cmin = cross;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cmin = min(cmin, __shfl_xor_sync(0xFFFFFFFFu, cmin, o));
    if (cmin == INT_MAX) return;
    // the element that leaves the binade: a real addition, then restart
    float sn = 0.0f;
    if (cross == cmin) {
      sn = __fadd_rn(seq_float(Nc, eu), xc);
#pragma unroll
      for (int r = 0; r < R; r++)
        if (lane * R + r == cmin) pref[r] = sn;
    }
    s = __shfl_sync(0xFFFFFFFFu, sn, cmin / R);
    start = cmin + 1;
  }
}

// First list position j < n (in list order) whose flag is set, or -1.
template <int R>
__device__ __forceinline__ int warp_first(const bool (&flag)[R], int n) {
  const int lane = static_cast<int>(lane_id());
  int mine = INT_MAX;
#pragma unroll
  for (int r = R - 1; r >= 0; r--)
    if (flag[r] && lane * R + r < n) mine = lane * R + r;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine = min(mine, __shfl_xor_sync(0xFFFFFFFFu, mine, o));
  return mine == INT_MAX ? -1 : mine;
}

template <int R>
__device__ __forceinline__ float warp_get(const float (&v)[R], int j) {
  float x = v[0];
#pragma unroll
  for (int r = 1; r < R; r++) x = (j % R == r) ? v[r] : x;
  return __shfl_sync(0xFFFFFFFFu, x, j / R);
}

// The list sampling of the reference over a sorted list of keff <= 32*R
// entries (lk[0..n_sel) keys, the rest the reference's empty slots
// (-1e30, -1)).  p_on: reference src/sampling/top_p.c:37-105 on the list;
// else: reference src/sampling/top_k.c:50-72.  Returns the token; `rs`
// advances by one draw unless the nucleus has no candidate.  Writes the
// list's probabilities to pr_out[0..keff) (shared or global, may be null).
// Returns INT_MIN if the probabilities are not in list order (then the
// caller uses the general path).
template <int R>
__device__ int warp_sample_list(const unsigned long long *lk, int n_sel, const RowPlan &P,
                                unsigned long long &rs, float *pr_out) {
  const int lane = static_cast<int>(lane_id());
  const int keff = P.keff;
  float val[R];
  int idv[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int j = lane * R + r;
    val[r] = j < n_sel ? key_val(lk[j]) : -1e30f;
    idv[r] = j < n_sel ? key_idx(lk[j]) : -1;
  }
  const float mx = __shfl_sync(0xFFFFFFFFu, val[0], 0);
  auto id_at = [&](int j) -> int {
    int x = idv[0];
#pragma unroll
    for (int r = 1; r < R; r++) x = (j % R == r) ? idv[r] : x;
    return __shfl_sync(0xFFFFFFFFu, x, j / R);
  };
  float e[R], pr[R], cum[R];
  if (P.p_on) {
    const float thr = __fsub_rn(mx, 20.0f);                             // top_p.c:53
    bool out_f[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int j = lane * R + r;
      const bool c = j < keff && val[r] >= thr;
      e[r] = c ? cr_expf(__fsub_rn(val[r], mx)) : 0.0f;                 // :58-59
      out_f[r] = j < keff && !c;
    }
    // the list is sorted, so the kept entries are a prefix
    int n = warp_first<R>(out_f, keff);
    if (n < 0) n = keff;
    if (n == 0) {                                                       // :68-69
      if (pr_out)
        for (int j = lane; j < keff; j += 32) pr_out[j] = 0.0f;
      return id_at(0);
    }
    warp_seq_prefix<R>(e, n, cum);                                      // :62
    const float sum = warp_get<R>(cum, n - 1);
    const float inv = __fdiv_rn(1.0f, sum);                             // :72
    bool unsorted[R];
#pragma unroll
    for (int r = 0; r < R; r++) pr[r] = (lane * R + r < n) ? __fmul_rn(e[r], inv) : 0.0f;  // :73-74
    // stable sort by probability (:77) is the identity when they descend
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int j = lane * R + r;
      const float nxt = (r + 1 < R) ? pr[(r + 1) % R] : __shfl_down_sync(0xFFFFFFFFu, pr[0], 1);
      unsorted[r] = j + 1 < n && nxt > pr[r];
    }
    if (warp_first<R>(unsorted, n) >= 0) return INT_MIN;
    warp_seq_prefix<R>(pr, n, cum);                                     // :80-88
    bool ge[R];
#pragma unroll
    for (int r = 0; r < R; r++) ge[r] = cum[r] >= P.p;
    const int hit = warp_first<R>(ge, n);
    const int cutoff = hit >= 0 ? hit + 1 : n;
    const float trunc = warp_get<R>(cum, cutoff - 1);                   // :91-93
    const float rr = __fmul_rn(rng_next(rs), trunc);                    // :96
    bool lt[R];
#pragma unroll
    for (int r = 0; r < R; r++) lt[r] = rr < cum[r];
    const int w = warp_first<R>(lt, cutoff);                            // :98-105
    if (pr_out)
#pragma unroll
      for (int r = 0; r < R; r++)
        if (lane * R + r < keff) pr_out[lane * R + r] = pr[r];
    return id_at(w >= 0 ? w : 0);
  } else {
#pragma unroll
    for (int r = 0; r < R; r++)
      e[r] = (lane * R + r < keff) ? cr_expf(__fsub_rn(val[r], mx)) : 0.0f;  // top_k.c:54
    warp_seq_prefix<R>(e, keff, cum);                                   // :55
    const float sum = warp_get<R>(cum, keff - 1);
#pragma unroll
    for (int r = 0; r < R; r++)
      pr[r] = (lane * R + r < keff) ? __fdiv_rn(e[r], sum) : 0.0f;       // :57-59
    warp_seq_prefix<R>(pr, keff, cum);
    const float rr = rng_next(rs);                                      // :62
    bool lt[R];
#pragma unroll
    for (int r = 0; r < R; r++) lt[r] = rr < cum[r];
    const int w = warp_first<R>(lt, keff);
    if (pr_out)
#pragma unroll
      for (int r = 0; r < R; r++)
        if (lane * R + r < keff) pr_out[lane * R + r] = pr[r];
    return id_at(w >= 0 ? w : 0);                                       // :72
  }
}

}  // namespace pz

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

}  // namespace pz
