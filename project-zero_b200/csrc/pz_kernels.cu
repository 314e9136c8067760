// pz_kernels.cu — sm_100a kernels of the token sampler.
//
//   slice_kernel  one streaming pass over every row, split into S slices of
//                 L columns (one CTA each): 128-bit loads, penalties
//                 (shared-memory history bitmap + sorted id counts),
//                 temperature, and the slice's top-k (or argmax) as 64-bit
//                 ordered keys.  The last CTA of a row to finish (counted
//                 with an atomic, no waiting) merges the S lists into the
//                 exact top-k and runs the reference's list arithmetic
//                 (top_p.c:37-105 or top_k.c:50-72) to draw the token.
//   full_kernel   rows with no top-k list (k = 0): the exact sequential
//                 replay (pz_seqsum.cuh) of sample_top_p's normaliser,
//                 stable sort and CDF (top_p.c:53-105), or of the softmax
//                 and CDF walk of generate.c:158-167.
//   merge_kernel  vocab sharding: merges the G gathered per-rank lists and
//                 draws.
#include <climits>

#include "pz_device.cuh"
#include "pz_kernels.cuh"
#include "pz_select.cuh"
#include "pz_seqsum.cuh"

namespace pz {

// ---------------------------------------------------------------------------
// small block helpers
// ---------------------------------------------------------------------------
template <int NT>
__device__ unsigned long long block_max_u64(unsigned long long v,
                                            unsigned long long *red) {
  v = warp_max_u64(v);
  if (lane_id() == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long w = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0ull;
    w = warp_max_u64(w);
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  const unsigned long long r = red[0];
  __syncthreads();
  return r;
}

template <int NT>
__device__ int block_exscan_int(int v, int &total, int *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int incl = warp_incl_scan(v);
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int t = lane < NT / 32 ? red[lane] : 0;
    t = warp_incl_scan(t);
    if (lane < NT / 32) red[lane] = t;
  }
  __syncthreads();
  total = red[NT / 32 - 1];
  const int r = (warp ? red[warp - 1] : 0) + incl - v;
  __syncthreads();
  return r;
}

// Ascending bitonic sort of n2 (power of two) ints in shared memory.
template <int NT>
__device__ void block_sort_asc_i32(int32_t *a, int n2) {
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < (n2 >> 1); i += NT) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool asc = ((lo & size) == 0);
        const int32_t x = a[lo], y = a[hi];
        if (asc ? (x > y) : (x < y)) {
          a[lo] = y;
          a[hi] = x;
        }
      }
    }
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ float load_scalar(const T *p, int i);
template <>
__device__ __forceinline__ float load_scalar<float>(const float *p, int i) {
  return __ldg(p + i);
}
template <>
__device__ __forceinline__ float load_scalar<uint16_t>(const uint16_t *p, int i) {
  return bf16_to_f32(__ldg(p + i));
}

// 16 bytes of a row as VEC floats.
template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void load(const float *p, int vi, float *x) {
    const float4 q = __ldg(reinterpret_cast<const float4 *>(p) + vi);
    x[0] = q.x;
    x[1] = q.y;
    x[2] = q.z;
    x[3] = q.w;
  }
};
template <>
struct Vec16<uint16_t> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void load(const uint16_t *p, int vi, float *x) {
    const uint4 q = __ldg(reinterpret_cast<const uint4 *>(p) + vi);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      x[2 * j] = __uint_as_float(w[j] << 16);
      x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
};

// Count of id t in a sorted id array a[0..n) (history counts).
__device__ __forceinline__ int sorted_count(const int32_t *a, int n, int t) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < t) lo = mid + 1; else hi = mid;
  }
  int lo2 = lo, hi2 = n;
  while (lo2 < hi2) {
    const int mid = (lo2 + hi2) >> 1;
    if (a[mid] <= t) lo2 = mid + 1; else hi2 = mid;
  }
  return lo2 - lo;
}

// ---------------------------------------------------------------------------
// Sampling over a sorted top-k list (one row, one block).
//   lk[0..n_sel) keys sorted descending; entries n_sel..keff-1 are the
//   reference's unfilled slots (-1e30, -1).
// p_on:  the steps of reference src/sampling/top_p.c:37-105 over the list;
// else:  the softmax and draw of reference src/sampling/top_k.c:50-72.
// Thread 0 runs the sequential float accumulations in the reference's order.
// ---------------------------------------------------------------------------
template <int NT>
__device__ int sample_list(const unsigned long long *lk, int n_sel,
                           const RowPlan &P, unsigned long long &rs, float *e,
                           float *pr, int *order, int *s_tok, int32_t *cids,
                           float *cprobs) {
  const int keff = P.keff;
  const int tid = threadIdx.x;
  auto val = [&](int i) -> float { return i < n_sel ? key_val(lk[i]) : -1e30f; };
  auto idv = [&](int i) -> int { return i < n_sel ? key_idx(lk[i]) : -1; };
  const float mx = val(0);
  if (P.p_on) {
    const float thr = __fsub_rn(mx, 20.0f);                           // :53
    for (int i = tid; i < keff; i += NT) {
      const float v = val(i);
      e[i] = (v >= thr) ? cr_expf(__fsub_rn(v, mx)) : -1.0f;           // :58-59
    }
    __syncthreads();
    if (tid == 0) {
      float sum = 0.0f;
      int n = 0;
      for (int i = 0; i < keff; i++)
        if (e[i] >= 0.0f) {
          order[n++] = i;
          sum = __fadd_rn(sum, e[i]);                                   // :62
        }
      int tok;
      if (n == 0) {
        for (int i = 0; i < keff; i++) pr[i] = 0.0f;
        tok = idv(0);                                                   // :68-69
      } else {
        const float inv = __fdiv_rn(1.0f, sum);                         // :72
        for (int i = 0; i < keff; i++)
          pr[i] = e[i] >= 0.0f ? __fmul_rn(e[i], inv) : 0.0f;           // :73-74
        // stable sort by probability descending (:77; glibc's qsort is a
        // stable mergesort).  The list is already in value order, so this
        // insertion sort is linear unless exp rounding ties reorder it.
        for (int j = 1; j < n; j++) {
          const int o = order[j];
          const float po = pr[o];
          int q = j - 1;
          while (q >= 0 && po > pr[order[q]]) {
            order[q + 1] = order[q];
            q--;
          }
          order[q + 1] = o;
        }
        float cum = 0.0f;
        int cutoff = n;
        for (int j = 0; j < n; j++) {                                   // :80-88
          cum = __fadd_rn(cum, pr[order[j]]);
          if (cum >= P.p) {
            cutoff = j + 1;
            break;
          }
        }
        float tr = 0.0f;
        for (int j = 0; j < cutoff; j++) tr = __fadd_rn(tr, pr[order[j]]);  // :91-93
        const float r = __fmul_rn(rng_next(rs), tr);                    // :96
        float cdf = 0.0f;
        int res = order[0];
        for (int j = 0; j < cutoff; j++) {                              // :98-105
          cdf = __fadd_rn(cdf, pr[order[j]]);
          if (r < cdf) {
            res = order[j];
            break;
          }
        }
        tok = idv(res);
      }
      *s_tok = tok;
    }
  } else {
    for (int i = tid; i < keff; i += NT) e[i] = cr_expf(__fsub_rn(val(i), mx));  // top_k.c:54
    __syncthreads();
    if (tid == 0) {
      float sum = 0.0f;
      for (int i = 0; i < keff; i++) sum = __fadd_rn(sum, e[i]);        // :55
      for (int i = 0; i < keff; i++) pr[i] = __fdiv_rn(e[i], sum);      // :57-59
      const float r = rng_next(rs);                                     // :62
      float cdf = 0.0f;
      int tok = idv(0);                                                 // :72
      for (int i = 0; i < keff; i++) {
        cdf = __fadd_rn(cdf, pr[i]);
        if (r < cdf) {
          tok = idv(i);
          break;
        }
      }
      *s_tok = tok;
    }
  }
  __syncthreads();
  if (cids != nullptr)
    for (int i = tid; i < keff; i += NT) cids[i] = idv(i);
  if (cprobs != nullptr)
    for (int i = tid; i < keff; i += NT) cprobs[i] = pr[i];
  const int tok = *s_tok;
  __syncthreads();
  return tok;
}

// ---------------------------------------------------------------------------
// slice_kernel
// ---------------------------------------------------------------------------
size_t slice_smem_bytes(int kcap, int hcap, int bm_words) {
  return sizeof(unsigned long long) * static_cast<size_t>(kcap + kCapB) +
         sizeof(uint32_t) * static_cast<size_t>(bm_words) +
         sizeof(int32_t) * 2 * static_cast<size_t>(hcap) +
         (sizeof(float) * 2 + sizeof(int)) * static_cast<size_t>(kcap);
}

template <typename T>
__global__ void __launch_bounds__(kSliceThreads)
    slice_kernel(const SliceArgs A) {
  constexpr int NT = kSliceThreads;
  constexpr int VEC = Vec16<T>::N;
  constexpr int EPT = 16;
  constexpr int UV = EPT / VEC;
  constexpr int MAXPER = (PZ_TOP_K_MAX + kCapB) / NT;

  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ SelShared sh;
  __shared__ unsigned long long s_red[NT / 32];
  __shared__ int s_nh, s_last, s_x0nan, s_tok;

  const int tid = threadIdx.x;
  const int row = blockIdx.y, sl = blockIdx.x;
  const pz_sampler_config cfg = A.cfg[row];
  const RowPlan P = plan_row(cfg, A.V_global);
  const int a = sl * A.L;
  const int b = min(A.V, a + A.L);
  const int cap = A.kcap + kCapB;
  const int hwm = A.kcap + kCapB / 2;

  unsigned long long *cand = reinterpret_cast<unsigned long long *>(smem);
  uint32_t *bitmap = reinterpret_cast<uint32_t *>(cand + cap);
  int32_t *hl = reinterpret_cast<int32_t *>(bitmap + A.bm_words);
  int32_t *hc = hl + A.hcap;
  float *fe = reinterpret_cast<float *>(hc + A.hcap);
  float *fp = fe + A.kcap;
  int *ford = reinterpret_cast<int *>(fp + A.kcap);

  const T *rowp = static_cast<const T *>(A.logits) + static_cast<size_t>(row) * static_cast<size_t>(A.ld);
  const bool greedy = P.mode == kModeGreedy;
  // a list longer than this launch was sized for (hint broken): flag the row
  const bool bad_k = P.mode == kModeTopK && (P.keff > A.kmax || P.keff > A.kcap);
  const int k_sel = (P.mode == kModeTopK && !bad_k) ? P.keff : 1;
  const bool use_buf = k_sel > 1;
  const unsigned long long tau0 = (P.mode == kModeTopK) ? key_topk_floor() : 0ull;
  const uint32_t goff = static_cast<uint32_t>(A.v_offset);

  // ---- penalty history of this slice: sorted ids, counts, bitmap --------
  int H = 0;
  const int32_t *hrow = nullptr;
  if (A.hist != nullptr && A.hist_off != nullptr && P.pen_on) {
    const int h0 = A.hist_off[row];
    H = A.hist_off[row + 1] - h0;
    hrow = A.hist + h0;
  }
  const bool too_long = H > A.hcap;
  const bool hist_on = H > 0 && !too_long;
  if (tid == 0) {
    s_nh = 0;
    s_x0nan = 0;
    sh.n = 0;
    sh.tau = tau0;
  }
  if (hist_on)
    for (int w = tid; w < A.bm_words; w += NT) bitmap[w] = 0u;
  __syncthreads();
  int nh = 0;
  if (hist_on) {
    for (int j = tid; j < H; j += NT) {
      const long long t = static_cast<long long>(hrow[j]) - A.v_offset;
      if (t >= a && t < b) hl[atomicAdd(&s_nh, 1)] = static_cast<int>(t);
    }
    __syncthreads();
    nh = s_nh;
    int np2 = 1;
    while (np2 < nh) np2 <<= 1;
    for (int i = nh + tid; i < np2; i += NT) hl[i] = INT_MAX;
    block_sort_asc_i32<NT>(hl, np2);
    for (int i = tid; i < nh; i += NT) {
      const int t = hl[i];
      if (i == nh - 1 || hl[i + 1] != t) {
        int lo = 0, hi = i;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (hl[mid] < t) lo = mid + 1; else hi = mid;
        }
        hc[i] = i - lo + 1;
        const int o = t - a;
        atomicOr(&bitmap[o >> 5], 1u << (o & 31));
      } else {
        hc[i] = 0;
      }
    }
    __syncthreads();
  }

  // ---- stream the slice: 16-byte vectors, scalar head and tail ----------
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp + a);
  int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
  if (head > b - a) head = b - a;
  const int a_al = a + head;
  const int nvec = (b - a_al) / VEC;
  const int b_al = a_al + nvec * VEC;
  const int tail = b - b_al;
  const T *vbase = rowp + a_al;

  unsigned long long best = 0ull;
  for (int v0 = 0; v0 < nvec; v0 += NT * UV) {
    float xv[EPT];
    uint32_t hb[UV];
    uint32_t ok = 0;
#pragma unroll
    for (int u = 0; u < UV; u++) {
      const int vi = v0 + u * NT + tid;
      hb[u] = 0;
      if (vi < nvec) {
        Vec16<T>::load(vbase, vi, xv + u * VEC);
        ok |= ((1u << VEC) - 1u) << (u * VEC);
        if (hist_on) {
          const int o = a_al + vi * VEC - a;
          const uint32_t w0 = bitmap[o >> 5], w1 = bitmap[(o >> 5) + 1];
          hb[u] = __funnelshift_r(w0, w1, o & 31) & ((1u << VEC) - 1u);
        }
      } else {
#pragma unroll
        for (int w = 0; w < VEC; w++) xv[u * VEC + w] = 0.0f;
      }
    }
    unsigned long long keys[EPT];
    uint32_t valid = 0;
#pragma unroll
    for (int e = 0; e < EPT; e++) {
      const int u = e / VEC, w = e % VEC;
      keys[e] = 0ull;
      if ((ok >> e) & 1u) {
        if ((hb[u] >> w) & 1u) continue;
        const int li = a_al + (v0 + u * NT + tid) * VEC + w;
        const float v = greedy ? xv[e] : temper(xv[e], P);
        if (v != v) {
          if (li == 0 && goff == 0) s_x0nan = 1;
          continue;
        }
        keys[e] = mkkey(v, static_cast<uint32_t>(li) + goff);
        valid |= 1u << e;
      }
    }
    if (use_buf) {
      offer_round<NT, MAXPER, EPT>(cand, cap, hwm, k_sel, sh, keys, valid);
    } else {
#pragma unroll
      for (int e = 0; e < EPT; e++)
        if (((valid >> e) & 1u) && keys[e] > best) best = keys[e];
    }
  }

  // head, tail, and the penalised history ids, as extra rounds
  const int n_extra = head + tail + (hist_on ? nh : 0);
  for (int base = 0; base < n_extra; base += NT * EPT) {
    unsigned long long keys[EPT];
    uint32_t valid = 0;
#pragma unroll
    for (int e = 0; e < EPT; e++) {
      keys[e] = 0ull;
      const int it = base + e * NT + tid;
      if (it >= n_extra) continue;
      int li, cnt = 0;
      if (it < head) {
        li = a + it;
      } else if (it < head + tail) {
        li = b_al + (it - head);
      } else {
        const int i = it - head - tail;
        cnt = hc[i];
        if (cnt == 0) continue;
        li = hl[i];
      }
      if (cnt == 0 && hist_on) {
        const int o = li - a;
        if ((bitmap[o >> 5] >> (o & 31)) & 1u) continue;
      }
      float x = load_scalar<T>(rowp, li);
      if (cnt > 0) x = penalize(x, cnt, P);
      const float v = greedy ? x : temper(x, P);
      if (v != v) {
        if (li == 0 && goff == 0) s_x0nan = 1;
        continue;
      }
      keys[e] = mkkey(v, static_cast<uint32_t>(li) + goff);
      valid |= 1u << e;
    }
    if (use_buf) {
      offer_round<NT, MAXPER, EPT>(cand, cap, hwm, k_sel, sh, keys, valid);
    } else {
#pragma unroll
      for (int e = 0; e < EPT; e++)
        if (((valid >> e) & 1u) && keys[e] > best) best = keys[e];
    }
  }

  // ---- this slice's list -> scratch ------------------------------------
  int m;
  unsigned long long *dst =
      A.slice_keys + (static_cast<size_t>(row) * A.S + sl) * static_cast<size_t>(A.kcap);
  if (use_buf) {
    __syncthreads();
    int n = sh.n < cap ? sh.n : cap;
    __syncthreads();
    if (n > k_sel) {
      block_select<NT, MAXPER>(cand, n, k_sel, sh);
      n = k_sel;
    }
    m = n;
    for (int i = tid; i < m; i += NT) dst[i] = cand[i];
  } else {
    best = block_max_u64<NT>(best, s_red);
    m = best > tau0 ? 1 : 0;
    if (tid == 0 && m) dst[0] = best;
  }
  __syncthreads();
  if (tid == 0) {
    A.slice_cnt[static_cast<size_t>(row) * A.S + sl] = m;
    if (a == 0) A.row_flags[row] = s_x0nan ? 1u : 0u;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&A.row_arrive[row], 1u);
    s_last = (prev == static_cast<unsigned int>(A.S - 1));
  }
  __syncthreads();
  if (!s_last) return;

  // ======================= last CTA of the row ==========================
  __threadfence();
  if (tid == 0) A.row_arrive[row] = 0u;
  const int S = A.S;
  const unsigned long long *sk = A.slice_keys + static_cast<size_t>(row) * S * static_cast<size_t>(A.kcap);
  const int32_t *sc = A.slice_cnt + static_cast<size_t>(row) * S;
  int n_sel = 0;
  unsigned long long gbest = 0ull;
  if (use_buf) {
    if (tid == 0) {
      sh.n = 0;
      sh.tau = tau0;
    }
    __syncthreads();
    const int total = S * A.kcap;
    for (int base = 0; base < total; base += NT * EPT) {
      unsigned long long keys[EPT];
      uint32_t valid = 0;
#pragma unroll
      for (int e = 0; e < EPT; e++) {
        keys[e] = 0ull;
        const int it = base + e * NT + tid;
        if (it < total) {
          const int s2 = it / A.kcap, j = it - s2 * A.kcap;
          if (j < __ldcg(sc + s2)) {
            keys[e] = __ldcg(sk + it);
            valid |= 1u << e;
          }
        }
      }
      offer_round<NT, MAXPER, EPT>(cand, cap, hwm, k_sel, sh, keys, valid);
    }
    __syncthreads();
    int n = sh.n < cap ? sh.n : cap;
    __syncthreads();
    if (n > k_sel) {
      block_select<NT, MAXPER>(cand, n, k_sel, sh);
      n = k_sel;
    }
    n_sel = n;
    for (int i = n_sel + tid; i < A.kcap; i += NT) cand[i] = 0ull;
    block_sort_desc<NT>(cand, A.kcap);
  } else {
    unsigned long long bl = 0ull;
    for (int s2 = tid; s2 < S; s2 += NT)
      if (__ldcg(sc + s2) > 0) {
        const unsigned long long k = __ldcg(sk + static_cast<size_t>(s2) * A.kcap);
        bl = k > bl ? k : bl;
      }
    gbest = block_max_u64<NT>(bl, s_red);
    if (P.mode == kModeTopK) {  // k_eff == 1: the single best admitted key
      n_sel = gbest > tau0 ? 1 : 0;
      if (tid == 0) cand[0] = gbest;
      for (int i = 1 + tid; i < A.kcap; i += NT) cand[i] = 0ull;
      __syncthreads();
    }
  }
  const bool x0nan = (__ldcg(A.row_flags + row) & 1u) != 0u;

  if (A.mode_emit) {
    // vocab sharding: publish the local list; the draw happens after the
    // allgather (merge_kernel).
    unsigned long long *ek = A.emit_keys + static_cast<size_t>(row) * (A.kcap + 1);
    int cnt;
    if (use_buf) {
      cnt = n_sel;
      for (int i = tid; i < cnt; i += NT) ek[i] = cand[i];
    } else {
      cnt = gbest > tau0 ? 1 : 0;
      if (tid == 0 && cnt) ek[0] = gbest;
    }
    if (tid == 0)
      ek[A.kcap] = static_cast<unsigned long long>(cnt | (x0nan ? (1 << 30) : 0) |
                                                   (too_long ? (1 << 29) : 0) |
                                                   (bad_k ? (1 << 28) : 0));
    return;
  }

  unsigned long long rs = A.rng[row];
  int tok = -1;
  int status = too_long ? PZ_ROW_HISTORY_TOO_LONG : PZ_ROW_OK;
  bool pending = false;
  const bool want_cand = A.cand_ids != nullptr || A.cand_probs != nullptr;
  if (too_long) {
    tok = -1;                                             // penalties could not be applied
  } else if (bad_k) {
    tok = -1;
    status = PZ_ROW_HINT_VIOLATED;
  } else if (P.mode == kModeGreedy) {
    tok = x0nan ? 0 : (gbest ? key_idx(gbest) : 0);       // argmax.c:3-13
  } else if (P.mode == kModeTopK) {
    int32_t *cids = A.cand_ids ? A.cand_ids + static_cast<size_t>(row) * A.cand_stride : nullptr;
    float *cprobs = A.cand_probs ? A.cand_probs + static_cast<size_t>(row) * A.cand_stride : nullptr;
    tok = sample_list<NT>(cand, n_sel, P, rs, fe, fp, ford, &s_tok,
                          want_cand ? cids : nullptr, want_cand ? cprobs : nullptr);
  } else if (P.mode == kModeTopPFull && A.V_global > PZ_TOP_P_MAX_VOCAB) {
    tok = x0nan ? 0 : key_idx(gbest);                     // top_p.c:33-34
  } else if (P.mode == kModeTopPFull && x0nan) {
    tok = 0;                                              // NaN max: n == 0 -> argmax
  } else if (A.no_full_vocab) {
    tok = -1;
    status = PZ_ROW_HINT_VIOLATED;
  } else {
    pending = true;
    if (tid == 0) {
      A.row_best[row] = gbest;
      A.full_rows[atomicAdd(A.n_full, 1)] = row;
    }
  }
  if (tid == 0) {
    if (!pending) {
      A.out[row] = tok;
      A.rng[row] = rs;
    }
    if (A.n_cand) A.n_cand[row] = (P.mode == kModeTopK) ? P.keff : 0;
    if (A.row_status) A.row_status[row] = status;
  }
  if (want_cand && P.mode != kModeTopK) {
    for (int i = tid; i < A.cand_stride; i += NT) {
      if (A.cand_ids) A.cand_ids[static_cast<size_t>(row) * A.cand_stride + i] = -1;
      if (A.cand_probs) A.cand_probs[static_cast<size_t>(row) * A.cand_stride + i] = 0.0f;
    }
  }
}

// ---------------------------------------------------------------------------
// full_kernel: rows that need the whole row's distribution.
// ---------------------------------------------------------------------------
size_t full_smem_bytes(int V, int hcap) {
  const size_t bm_words = static_cast<size_t>(V) / 32 + 2;
  return sizeof(uint32_t) * bm_words + sizeof(int32_t) * static_cast<size_t>(hcap) +
         sizeof(uint32_t) * (kFullThreads / 32) * 256 + sizeof(uint32_t) * 256 * 2;
}

// Stable LSD radix sort of (key, value) u32 pairs ascending by key, in
// global scratch, by one block.  Each warp owns a contiguous segment; within
// a segment elements keep their order, so equal keys keep input order.
// Returns true when the result is in (k1, v1).
template <int NT>
__device__ bool block_radix_sort(uint32_t *k0, uint32_t *v0, uint32_t *k1,
                                 uint32_t *v1, int n, uint32_t *whist,
                                 uint32_t *tot, int *s_flag) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = (n + NW - 1) / NW;
  const int s0 = min(n, warp * seg), s1 = min(n, s0 + seg);
  bool in1 = false;
  for (int shift = 0; shift < 32; shift += 8) {
    uint32_t *ki = in1 ? k1 : k0, *vi = in1 ? v1 : v0;
    uint32_t *ko = in1 ? k0 : k1, *vo = in1 ? v0 : v1;
    for (int i = tid; i < NW * 256; i += NT) whist[i] = 0u;
    __syncthreads();
    for (int j = s0 + lane; j < s1; j += 32)
      atomicAdd(&whist[warp * 256 + ((__ldcg(ki + j) >> shift) & 255u)], 1u);
    __syncthreads();
    if (tid < 256) {
      uint32_t run = 0;
      for (int w = 0; w < NW; w++) {
        const uint32_t c = whist[w * 256 + tid];
        whist[w * 256 + tid] = run;
        run += c;
      }
      tot[tid] = run;
    }
    if (tid == 0) *s_flag = 0;
    __syncthreads();
    if (tid == 0) {
      uint32_t run = 0;
      for (int d = 0; d < 256; d++) {
        const uint32_t c = tot[d];
        if (static_cast<int>(c) == n) *s_flag = 1;  // one digit only: pass is the identity
        tot[d] = run;
        run += c;
      }
    }
    __syncthreads();
    if (*s_flag) {
      __syncthreads();
      continue;
    }
    if (tid < 256)
      for (int w = 0; w < NW; w++) whist[w * 256 + tid] += tot[tid];
    __syncthreads();
    for (int j0 = s0; j0 < s1; j0 += 32) {
      const int j = j0 + lane;
      const bool act = j < s1;
      const uint32_t key = act ? __ldcg(ki + j) : 0u;
      const uint32_t val = act ? __ldcg(vi + j) : 0u;
      const uint32_t d = act ? ((key >> shift) & 255u) : (256u + lane);
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      uint32_t pos = 0;
      if (act) {
        pos = whist[warp * 256 + d] + __popc(peers & lanemask_lt());
        ko[pos] = key;
        vo[pos] = val;
      }
      __syncwarp();
      if (act && lane == __ffs(peers) - 1) whist[warp * 256 + d] += __popc(peers);
      __syncwarp();
    }
    __threadfence_block();
    __syncthreads();
    in1 = !in1;
  }
  return in1;
}

template <typename T>
__global__ void __launch_bounds__(kFullThreads, 1) full_kernel(const FullArgs A) {
  constexpr int NT = kFullThreads;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ SeqShared ssh;
  __shared__ int s_red[NT / 32];
  __shared__ int s_nh, s_flag;
  const int tid = threadIdx.x;
  const int bm_words = A.V / 32 + 2;
  uint32_t *bitmap = reinterpret_cast<uint32_t *>(smem);
  int32_t *hl = reinterpret_cast<int32_t *>(bitmap + bm_words);
  uint32_t *whist = reinterpret_cast<uint32_t *>(hl + A.hcap);
  uint32_t *tot = whist + (NT / 32) * 256;
  uint32_t *k0 = A.sort_a + static_cast<size_t>(blockIdx.x) * A.sort_stride;
  uint32_t *v0 = k0 + A.sort_stride / 2;
  uint32_t *k1 = A.sort_b + static_cast<size_t>(blockIdx.x) * A.sort_stride;
  uint32_t *v1 = k1 + A.sort_stride / 2;
  const int n_full = *A.n_full;

  for (int w = blockIdx.x; w < n_full; w += gridDim.x) {
    const int row = A.full_rows[w];
    const pz_sampler_config cfg = A.cfg[row];
    const RowPlan P = plan_row(cfg, A.V);
    const T *rowp = static_cast<const T *>(A.logits) + static_cast<size_t>(row) * static_cast<size_t>(A.ld);
    const int V = A.V;

    // history over the whole row
    int H = 0;
    const int32_t *hrow = nullptr;
    if (A.hist != nullptr && A.hist_off != nullptr && P.pen_on) {
      const int h0 = A.hist_off[row];
      H = A.hist_off[row + 1] - h0;
      hrow = A.hist + h0;
    }
    const bool hist_on = H > 0 && H <= A.hcap;
    if (tid == 0) s_nh = 0;
    if (hist_on)
      for (int i = tid; i < bm_words; i += NT) bitmap[i] = 0u;
    __syncthreads();
    int nh = 0;
    if (hist_on) {
      for (int j = tid; j < H; j += NT) {
        const int t = hrow[j];
        if (t >= 0 && t < V) {
          hl[atomicAdd(&s_nh, 1)] = t;
          atomicOr(&bitmap[t >> 5], 1u << (t & 31));
        }
      }
      __syncthreads();
      nh = s_nh;
      int np2 = 1;
      while (np2 < nh) np2 <<= 1;
      for (int i = nh + tid; i < np2; i += NT) hl[i] = INT_MAX;
      block_sort_asc_i32<NT>(hl, np2);
    }
    auto vof = [&](int i) -> float {
      float x = load_scalar<T>(rowp, i);
      if (hist_on && ((bitmap[i >> 5] >> (i & 31)) & 1u))
        x = penalize(x, sorted_count(hl, nh, i), P);
      return temper(x, P);
    };
    const float mx = key_val(A.row_best[row]);
    unsigned long long rs = A.rng[row];
    int tok;
    if (P.mode == kModeSoftmaxFull) {
      // softmax.c:12-22 then generate.c:159-167
      const SeqResult s1 = seq_scan<NT, 4>(
          V, [&](int i) { return cr_expf(__fsub_rn(vof(i), mx)); }, kSeqNone, 0.0f, ssh);
      const float inv = __fdiv_rn(1.0f, s1.s);
      const float r = rng_next(rs);
      const SeqResult s2 = seq_scan<NT, 4>(
          V, [&](int i) { return __fmul_rn(cr_expf(__fsub_rn(vof(i), mx)), inv); },
          kSeqGT, r, ssh);
      tok = s2.hit >= 0 ? s2.hit : V - 1;
    } else {
      // top_p.c:53-105 over the whole row
      const float thr = __fsub_rn(mx, 20.0f);
      const SeqResult s1 = seq_scan<NT, 4>(
          V,
          [&](int i) {
            const float v = vof(i);
            return v >= thr ? cr_expf(__fsub_rn(v, mx)) : 0.0f;
          },
          kSeqNone, 0.0f, ssh);
      const float inv = __fdiv_rn(1.0f, s1.s);
      // candidates in index order: (~prob bits, index)
      int nf = 0;
      for (int c0 = 0; c0 < V; c0 += NT * 4) {
        float pv[4];
        int cnt = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int i = c0 + tid * 4 + e;
          pv[e] = -1.0f;
          if (i < V) {
            const float v = vof(i);
            if (v >= thr) {
              pv[e] = __fmul_rn(cr_expf(__fsub_rn(v, mx)), inv);
              cnt++;
            }
          }
        }
        int total;
        int pos = nf + block_exscan_int<NT>(cnt, total, s_red);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          if (pv[e] >= 0.0f) {
            k0[pos] = ~__float_as_uint(pv[e]);
            v0[pos] = static_cast<uint32_t>(c0 + tid * 4 + e);
            pos++;
          }
        }
        nf += total;
      }
      __threadfence_block();
      __syncthreads();
      const bool in1 = block_radix_sort<NT>(k0, v0, k1, v1, nf, whist, tot, &s_flag);
      const uint32_t *ks = in1 ? k1 : k0;
      const uint32_t *vs = in1 ? v1 : v0;
      // cumulative to the cutoff (:80-88), truncated sum (:91-93)
      const SeqResult s3 = seq_scan<NT, 4>(
          nf, [&](int j) { return __uint_as_float(~__ldcg(ks + j)); }, kSeqGE, P.p, ssh);
      const int cutoff = s3.hit >= 0 ? s3.hit + 1 : nf;
      const float r = __fmul_rn(rng_next(rs), s3.s);
      const SeqResult s4 = seq_scan<NT, 4>(
          cutoff, [&](int j) { return __uint_as_float(~__ldcg(ks + j)); }, kSeqGT, r, ssh);
      const int pos = s4.hit >= 0 ? s4.hit : 0;
      tok = nf > 0 ? static_cast<int>(__ldcg(vs + pos)) : key_idx(A.row_best[row]);
    }
    if (tid == 0) {
      A.out[row] = tok;
      A.rng[row] = rs;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// merge_kernel: vocab-sharded rows after the allgather (one block per row).
// ---------------------------------------------------------------------------
size_t merge_smem_bytes(int kcap) {
  return sizeof(unsigned long long) * static_cast<size_t>(kcap + kCapB) +
         (sizeof(float) * 2 + sizeof(int)) * static_cast<size_t>(kcap);
}

__global__ void __launch_bounds__(kSliceThreads) merge_kernel(const MergeArgs A) {
  constexpr int NT = kSliceThreads;
  constexpr int EPT = 16;
  constexpr int MAXPER = (PZ_TOP_K_MAX + kCapB) / NT;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ SelShared sh;
  __shared__ unsigned long long s_red[NT / 32];
  __shared__ int s_tok, s_flags;
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int cap = A.kcap + kCapB;
  const int hwm = A.kcap + kCapB / 2;
  unsigned long long *cand = reinterpret_cast<unsigned long long *>(smem);
  float *fe = reinterpret_cast<float *>(cand + cap);
  float *fp = fe + A.kcap;
  int *ford = reinterpret_cast<int *>(fp + A.kcap);
  const RowPlan P = plan_row(A.cfg[row], A.V_global);
  const bool k_fits = P.keff <= A.kcap && P.keff <= A.kmax;
  const bool use_buf = P.mode == kModeTopK && P.keff > 1 && k_fits;
  const int k_sel = (P.mode == kModeTopK && k_fits) ? P.keff : 1;
  const unsigned long long tau0 = (P.mode == kModeTopK) ? key_topk_floor() : 0ull;
  if (tid == 0) {
    sh.n = 0;
    sh.tau = tau0;
    s_flags = 0;
  }
  __syncthreads();
  const size_t stride = static_cast<size_t>(A.kcap) + 1;
  auto gcount = [&](int g) -> int {
    return static_cast<int>(A.gathered[(static_cast<size_t>(g) * A.B + row) * stride + A.kcap]);
  };
  auto gn = [&](int g) -> int { return min(gcount(g) & ((1 << 28) - 1), A.kcap); };
  if (tid < A.G) atomicOr(&s_flags, gcount(tid) & (7 << 28));
  int n_sel = 0;
  unsigned long long gbest = 0ull;
  if (use_buf) {
    const int total = A.G * A.kcap;
    for (int base = 0; base < total; base += NT * EPT) {
      unsigned long long keys[EPT];
      uint32_t valid = 0;
#pragma unroll
      for (int e = 0; e < EPT; e++) {
        keys[e] = 0ull;
        const int it = base + e * NT + tid;
        if (it < total) {
          const int g = it / A.kcap, j = it - g * A.kcap;
          const int cnt = gn(g);
          if (j < cnt) {
            keys[e] = A.gathered[(static_cast<size_t>(g) * A.B + row) * stride + j];
            valid |= 1u << e;
          }
        }
      }
      offer_round<NT, MAXPER, EPT>(cand, cap, hwm, k_sel, sh, keys, valid);
    }
    __syncthreads();
    int n = sh.n < cap ? sh.n : cap;
    __syncthreads();
    if (n > k_sel) {
      block_select<NT, MAXPER>(cand, n, k_sel, sh);
      n = k_sel;
    }
    n_sel = n;
    for (int i = n_sel + tid; i < A.kcap; i += NT) cand[i] = 0ull;
    block_sort_desc<NT>(cand, A.kcap);
  } else {
    unsigned long long bl = 0ull;
    for (int g = tid; g < A.G; g += NT) {
      const int cnt = gn(g);
      if (cnt > 0) {
        const unsigned long long k = A.gathered[(static_cast<size_t>(g) * A.B + row) * stride];
        bl = k > bl ? k : bl;
      }
    }
    gbest = block_max_u64<NT>(bl, s_red);
    if (P.mode == kModeTopK) {  // k_eff == 1: the single best admitted key
      n_sel = gbest > tau0 ? 1 : 0;
      if (tid == 0) cand[0] = gbest;
      for (int i = 1 + tid; i < A.kcap; i += NT) cand[i] = 0ull;
      __syncthreads();
    }
  }
  const bool x0nan = (s_flags >> 30) & 1;
  const bool too_long = (s_flags >> 29) & 1;
  const bool bad_k = ((s_flags >> 28) & 1) || (P.mode == kModeTopK && !k_fits);
  unsigned long long rs = A.rng[row];
  int tok = -1;
  int status = too_long ? PZ_ROW_HISTORY_TOO_LONG : PZ_ROW_OK;
  const bool want_cand = A.cand_ids != nullptr || A.cand_probs != nullptr;
  if (too_long) {
    tok = -1;
  } else if (bad_k) {
    tok = -1;
    status = PZ_ROW_HINT_VIOLATED;
  } else if (P.mode == kModeGreedy) {
    tok = x0nan ? 0 : (gbest ? key_idx(gbest) : 0);
  } else if (P.mode == kModeTopK) {
    int32_t *cids = A.cand_ids ? A.cand_ids + static_cast<size_t>(row) * A.cand_stride : nullptr;
    float *cprobs = A.cand_probs ? A.cand_probs + static_cast<size_t>(row) * A.cand_stride : nullptr;
    tok = sample_list<NT>(cand, n_sel, P, rs, fe, fp, ford, &s_tok,
                          want_cand ? cids : nullptr, want_cand ? cprobs : nullptr);
  } else {
    status = PZ_ROW_HINT_VIOLATED;
  }
  if (tid == 0) {
    A.out[row] = tok;
    A.rng[row] = rs;
    if (A.n_cand) A.n_cand[row] = P.mode == kModeTopK ? P.keff : 0;
    if (A.row_status) A.row_status[row] = status;
  }
}

// ---------------------------------------------------------------------------
// small kernels
// ---------------------------------------------------------------------------
__global__ void temperature_kernel(float *x, int n, float inv) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fmul_rn(x[i], inv);   // temperature.c:11-20
}

__global__ void rng_seed_kernel(unsigned long long *s, int B,
                                unsigned long long base,
                                const unsigned long long *seeds) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < B) {
    const unsigned long long v = seeds ? seeds[i] : base + static_cast<unsigned long long>(i);
    s[i] = v == 0ull ? 1ull : v;   // rng.c:3-6
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t set_kernel_attributes() {
  cudaError_t e;
  const int big = 227 * 1024;
  e = cudaFuncSetAttribute(slice_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(slice_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(full_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(full_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  return e;
}

cudaError_t launch_slice(const SliceArgs &a, int dtype, size_t smem, cudaStream_t st) {
  const dim3 grid(a.S, a.B);
  if (dtype == PZ_DTYPE_F32)
    slice_kernel<float><<<grid, kSliceThreads, smem, st>>>(a);
  else
    slice_kernel<uint16_t><<<grid, kSliceThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_full(const FullArgs &a, int dtype, int grid, size_t smem, cudaStream_t st) {
  if (dtype == PZ_DTYPE_F32)
    full_kernel<float><<<grid, kFullThreads, smem, st>>>(a);
  else
    full_kernel<uint16_t><<<grid, kFullThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_merge(const MergeArgs &a, size_t smem, cudaStream_t st) {
  merge_kernel<<<a.B, kSliceThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_temperature(float *x, int n, float T, cudaStream_t st) {
  if (T < 1e-6f) T = 1e-6f;                 // temperature.c:10
  const float inv = 1.0f / T;
  temperature_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, n, inv);
  return cudaGetLastError();
}

cudaError_t launch_rng_seed(unsigned long long *s, int B, unsigned long long base,
                            const unsigned long long *seeds, cudaStream_t st) {
  rng_seed_kernel<<<(B + 255) / 256, 256, 0, st>>>(s, B, base, seeds);
  return cudaGetLastError();
}

}  // namespace pz
