// pz_kernels.cu — sm_100a kernels of the token sampler.
//
//   slice_kernel  one streaming pass over every row, one CTA per row (the
//                 rows of the GPU's last, partial wave split into S slices
//                 of L columns, one CTA each): 16-byte copies, penalties
//                 (shared-memory history table and bitmap), temperature,
//                 and the top-k (or argmax) as 64-bit ordered keys.  The
//                 row's CTA, or the last of its slices to finish (counted
//                 with an atomic, no waiting, merging the S lists), runs the
//                 reference's list arithmetic (top_p.c:37-105 or
//                 top_k.c:50-72) to draw the token.
//   full_kernel   rows with no top-k list (k = 0): the exact sequential
//                 replay (pz_seqsum.cuh) of sample_top_p's normaliser,
//                 stable sort and CDF (top_p.c:53-105), or of the softmax
//                 and CDF walk of generate.c:158-167.
//   merge_kernel  vocab sharding: merges the G gathered per-rank lists and
//                 draws.
#include <cuda_bf16.h>

#include <climits>

#include "pz_device.cuh"
#include "pz_kernels.cuh"
#include "pz_select.cuh"
#include "pz_seqsum.cuh"
#include "pz_async_copy.cuh"
#include "pz_warpsel.cuh"
#include "pz_listmath.cuh"

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
__device__ __forceinline__ void grp_sync() {
  if (NT == 32)
    __syncwarp();
  else
    __syncthreads();
}

template <int NT>
__device__ __noinline__ int sample_list(const unsigned long long *lk, int n_sel,
                           const RowPlan &P, unsigned long long &rs, float *e,
                           float *pr, int *order, int *s_tok, int32_t *cids,
                           float *cprobs) {
  const int keff = P.keff;
  const int tid = static_cast<int>(threadIdx.x) & (NT - 1);
  auto val = [&](int i) -> float { return i < n_sel ? key_val(lk[i]) : -1e30f; };
  auto idv = [&](int i) -> int { return i < n_sel ? key_idx(lk[i]) : -1; };
  const float mx = val(0);
  if (P.p_on) {
    const float thr = __fsub_rn(mx, 20.0f);                           // :53
    for (int i = tid; i < keff; i += NT) {
      const float v = val(i);
      e[i] = (v >= thr) ? cr_expf(__fsub_rn(v, mx)) : -1.0f;           // :58-59
    }
    grp_sync<NT>();
    if (tid == 0) {
      // The list is sorted by value, so the entries the max-20 filter keeps
      // are a prefix, in the reference's candidate order.
      float sum = 0.0f;
      int n = 0;
      while (n < keff && e[n] >= 0.0f) sum = __fadd_rn(sum, e[n++]);   // :62
      int tok;
      if (n == 0) {
        tok = idv(0);                                                   // :68-69
      } else {
        const float inv = __fdiv_rn(1.0f, sum);                         // :72
        bool sorted = true;
        for (int i = 0; i < n; i++) {
          pr[i] = __fmul_rn(e[i], inv);                                 // :73-74
          order[i] = i;
          if (i > 0 && pr[i] > pr[i - 1]) sorted = false;
        }
        if (!sorted) {
          // stable sort by probability descending (:77; glibc's qsort is a
          // stable mergesort).  Exp is monotone, so this never runs unless
          // rounding ties reorder neighbours.
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
        }
        // cumulative to the cutoff (:80-88); the truncated sum (:91-93) and
        // the walk's CDF (:98-105) repeat exactly these additions, so the
        // prefix sums are kept (in e[], no longer needed) and reused.
        float cum = 0.0f;
        int cutoff = n;
        for (int j = 0; j < n; j++) {
          cum = __fadd_rn(cum, pr[order[j]]);
          e[j] = cum;
          if (cum >= P.p) {
            cutoff = j + 1;
            break;
          }
        }
        const float r = __fmul_rn(rng_next(rs), e[cutoff - 1]);         // :96
        int res = order[0];
        for (int j = 0; j < cutoff; j++)
          if (r < e[j]) {
            res = order[j];
            break;
          }
        tok = idv(res);
        for (int i = n; i < keff; i++) pr[i] = 0.0f;
      }
      if (n == 0)
        for (int i = 0; i < keff; i++) pr[i] = 0.0f;
      *s_tok = tok;
    }
  } else {
    for (int i = tid; i < keff; i += NT) e[i] = cr_expf(__fsub_rn(val(i), mx));  // top_k.c:54
    grp_sync<NT>();
    if (tid == 0) {
      float sum = 0.0f;
      for (int i = 0; i < keff; i++) sum = __fadd_rn(sum, e[i]);        // :55
      const float r = rng_next(rs);                                     // :62
      float cdf = 0.0f;
      int tok = idv(0);                                                 // :72
      int i = 0;
      for (; i < keff; i++) {
        pr[i] = __fdiv_rn(e[i], sum);                                   // :57-59
        cdf = __fadd_rn(cdf, pr[i]);
        if (r < cdf) {
          tok = idv(i);
          i++;
          break;
        }
      }
      for (; i < keff; i++) pr[i] = __fdiv_rn(e[i], sum);
      *s_tok = tok;
    }
  }
  grp_sync<NT>();
  if (cids != nullptr)
    for (int i = tid; i < keff; i += NT) cids[i] = idv(i);
  if (cprobs != nullptr)
    for (int i = tid; i < keff; i += NT) cprobs[i] = pr[i];
  const int tok = *s_tok;
  grp_sync<NT>();
  return tok;
}

// The decision for one row from its merged list (one warp): the draw (or
// argmax), its outputs, a full-vocabulary hand-off to full_kernel, or the
// published list (vocab sharding).  lst: sorted descending, n_sel real keys
// then zeros up to kcap (top-k rows); gbest: the best key (other rows);
// rs: the row's RNG state.  fe, fp, ford, s_tok: the warp's shared scratch
// of kcap entries each.
// full_kernel's cost class of a full-vocabulary row: its work grows with
// the temperature and with top_p (a flatter distribution keeps more values
// and a longer nucleus to sort and replay).  Measured on config 4, a row's
// time is about 390 us x T + 1100 us x p plus a constant; softmax rows (two
// whole-row replays, no sort) sit in the middle.
__device__ __forceinline__ int full_class(const RowPlan &P) {
  const float key = P.p_on ? P.T + 2.8f * P.p : P.T + 1.5f;
  const float c = (key - 1.0f) * 2.5f;
  return c >= static_cast<float>(kFullClasses - 1) ? kFullClasses - 1 : (c > 0.0f ? static_cast<int>(c) : 0);
}

template <bool LONG>
__device__ __forceinline__ void finalize_row(const SliceArgs &A, int row, const RowPlan &P, bool bad_k,
                                          bool too_long, bool row_timed_out, bool x0nan,
                                          const unsigned long long *lst, int n_sel,
                                          unsigned long long gbest, unsigned long long rs, float *fe,
                                          float *fp, int *ford, int *s_tokp) {
  const int lane = threadIdx.x & 31;
  int &s_tok = *s_tokp;
  const unsigned long long tau0 = (P.mode == kModeTopK) ? key_topk_floor() : 0ull;
  if (A.mode_emit) {
    // vocab sharding: publish the local list; the draw happens after the
    // allgather (merge_kernel).
    unsigned long long *ek = A.emit_keys + static_cast<size_t>(row) * (A.kcap + 1);
    int cnt;
    if (P.mode == kModeTopK && !bad_k) {
      cnt = n_sel;
      for (int i = lane; i < cnt; i += 32) ek[i] = lst[i];
    } else {
      cnt = gbest > tau0 ? 1 : 0;
      if (lane == 0 && cnt) ek[0] = gbest;
    }
    if (lane == 0)
      ek[A.kcap] = static_cast<unsigned long long>(cnt | (x0nan ? (1 << 30) : 0) |
                                                   (too_long ? (1 << 29) : 0) |
                                                   (bad_k ? (1 << 28) : 0) |
                                                   (row_timed_out ? (1 << 27) : 0));
    return;
  }

  int tok = -1;
  int status = too_long ? PZ_ROW_HISTORY_TOO_LONG : PZ_ROW_OK;
  bool pending = false;
  const bool want_cand = A.cand_ids != nullptr || A.cand_probs != nullptr;
  if (row_timed_out) {
    tok = -1;
    status = PZ_ROW_TIMEOUT;
  } else if (too_long) {
    tok = -1;                                             // penalties could not be applied
  } else if (bad_k) {
    tok = -1;
    status = PZ_ROW_HINT_VIOLATED;
  } else if (P.mode == kModeGreedy) {
    tok = x0nan ? 0 : (gbest ? key_idx(gbest) : 0);       // argmax.c:3-13
  } else if (P.mode == kModeTopK) {
    int32_t *cids = A.cand_ids ? A.cand_ids + static_cast<size_t>(row) * A.cand_stride : nullptr;
    float *cprobs = A.cand_probs ? A.cand_probs + static_cast<size_t>(row) * A.cand_stride : nullptr;
    int t = INT_MIN;
    if (P.keff <= 64) {
      // element-wise steps across the warp, the sequential sums on one lane
      t = warp_sample_small(lst, n_sel, P, rs, fe, fp, want_cand ? cprobs : nullptr);
      if (t != INT_MIN && want_cand && cids != nullptr)
        for (int i = lane; i < P.keff; i += 32) cids[i] = i < n_sel ? key_idx(lst[i]) : -1;
    } else if (LONG) {
      // longer lists: the same, with the sums on one lane eight terms at a time
      t = warp_sample_long(lst, n_sel, P, rs, fe, fp, want_cand ? cprobs : nullptr);
      if (t != INT_MIN && want_cand && cids != nullptr)
        for (int i = lane; i < P.keff; i += 32) cids[i] = i < n_sel ? key_idx(lst[i]) : -1;
    }
    if (t == INT_MIN)
      t = sample_list<32>(lst, n_sel, P, rs, fe, fp, ford, &s_tok,
                          want_cand ? cids : nullptr, want_cand ? cprobs : nullptr);
    tok = t;
  } else if (P.mode == kModeTopPFull && A.V_global > PZ_TOP_P_MAX_VOCAB) {
    tok = x0nan ? 0 : key_idx(gbest);                     // top_p.c:33-34
  } else if (P.mode == kModeTopPFull && x0nan) {
    tok = 0;                                              // NaN max: n == 0 -> argmax
  } else if (A.no_full_vocab) {
    tok = -1;
    status = PZ_ROW_HINT_VIOLATED;
  } else {
    pending = true;
    if (lane == 0) {
      A.row_best[row] = gbest;
      const int c = full_class(P);
      A.full_rows[c * A.full_stride + atomicAdd(A.n_full + c, 1)] = row;
    }
  }
  if (lane == 0) {
    if (!pending) {
      A.out[row] = tok;
      A.rng[row] = rs;
    }
    if (A.n_cand) A.n_cand[row] = (P.mode == kModeTopK && !bad_k && !too_long && !row_timed_out) ? P.keff : 0;
    if (A.row_status) A.row_status[row] = status;
  }
  if (want_cand && (P.mode != kModeTopK || bad_k || too_long || row_timed_out)) {
    for (int i = lane; i < A.cand_stride; i += 32) {
      if (A.cand_ids) A.cand_ids[static_cast<size_t>(row) * A.cand_stride + i] = -1;
      if (A.cand_probs) A.cand_probs[static_cast<size_t>(row) * A.cand_stride + i] = 0.0f;
    }
  }
}

// ---------------------------------------------------------------------------
// slice_kernel
// ---------------------------------------------------------------------------
constexpr int kChunkBytes = 2048;    // a warp's chunk of the slice (16 bytes per lane x 4)
constexpr int kSlots = 2;            // ring slots per warp (copies in flight per warp)
constexpr int kSliceWarps = kSliceThreads / 32;
constexpr int kLaneVecs = kChunkBytes / 16 / 32;  // 16-byte vectors per lane per chunk
constexpr uint32_t kHashEmpty = 0xFFFFFFFFu;
constexpr uint32_t kOrdNegInf = 0x007FFFFFu;      // f2ord(-inf)
static_assert(kLaneVecs == 2 || kLaneVecs == 4, "two or four vectors per lane per chunk");

template <int R>
__device__ __forceinline__ float max_of(const float (&v)[R]) {
  float m = v[0];
#pragma unroll
  for (int r = 1; r < R; r++) m = fmaxf(m, v[r]);
  return m;
}

// Open-addressing table of the slice's history ids with their counts.  The
// table has at least twice as many slots as ids, so probes end.
__device__ __forceinline__ void hash_insert(uint32_t *hk, uint32_t *hn, uint32_t mask,
                                            uint32_t shift, uint32_t t) {
  uint32_t h = (t * 0x9E3779B1u) >> shift;
  for (uint32_t i = 0; i <= mask; i++) {
    const uint32_t prev = atomicCAS(&hk[h], kHashEmpty, t);
    if (prev == kHashEmpty || prev == t) {
      atomicAdd(&hn[h], 1u);
      return;
    }
    h = (h + 1) & mask;
  }
}

__device__ __forceinline__ int hash_count(const uint32_t *hk, const uint32_t *hn, uint32_t mask,
                                          uint32_t shift, uint32_t t) {
  uint32_t h = (t * 0x9E3779B1u) >> shift;
  for (uint32_t i = 0; i <= mask; i++) {
    const uint32_t k = hk[h];
    if (k == t) return static_cast<int>(hn[h]);
    if (k == kHashEmpty) return 0;
    h = (h + 1) & mask;
  }
  return 0;
}

// 16 bytes of a staged chunk (shared memory) as VEC floats.
template <typename T>
struct Vec16S;
template <>
struct Vec16S<float> {
  __device__ __forceinline__ static void load(const unsigned char *s, int vi, float *x) {
    const float4 q = reinterpret_cast<const float4 *>(s)[vi];
    x[0] = q.x;
    x[1] = q.y;
    x[2] = q.z;
    x[3] = q.w;
  }
};
template <>
struct Vec16S<uint16_t> {
  __device__ __forceinline__ static void load(const unsigned char *s, int vi, float *x) {
    const uint4 q = reinterpret_cast<const uint4 *>(s)[vi];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      x[2 * j] = __uint_as_float(w[j] << 16);
      x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
};

// A lane's 16-byte vector of a chunk held in registers: its largest value
// (NaN ignored, as fmaxf does) and element w.  `nan` fills the vectors past
// the end of a short chunk.
template <typename T>
struct LaneVec;
template <>
struct LaneVec<float> {
  static constexpr int N = 4;
  static constexpr uint32_t nan = 0x7FC00000u;
  __device__ __forceinline__ static float vmax(const uint4 &q) {
    return fmaxf(fmaxf(__uint_as_float(q.x), __uint_as_float(q.y)),
                 fmaxf(__uint_as_float(q.z), __uint_as_float(q.w)));
  }
  __device__ __forceinline__ static float elem(const uint4 &q, int w) {
    return __uint_as_float(w == 0 ? q.x : w == 1 ? q.y : w == 2 ? q.z : q.w);
  }
  __device__ __forceinline__ static float smem(const unsigned char *s, int i) {
    return reinterpret_cast<const float *>(s)[i];
  }
};
template <>
struct LaneVec<uint16_t> {
  static constexpr int N = 8;
  static constexpr uint32_t nan = 0x7FC07FC0u;
  __device__ __forceinline__ static __nv_bfloat162 as2(uint32_t u) {
    __nv_bfloat162 r;
    memcpy(&r, &u, sizeof r);
    return r;
  }
  __device__ __forceinline__ static float vmax(const uint4 &q) {
    const __nv_bfloat162 m2 = __hmax2(__hmax2(as2(q.x), as2(q.y)), __hmax2(as2(q.z), as2(q.w)));
    uint32_t m;
    memcpy(&m, &m2, sizeof m);
    return fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
  }
  __device__ __forceinline__ static float elem(const uint4 &q, int w) {
    const uint32_t u = (w >> 1) == 0 ? q.x : (w >> 1) == 1 ? q.y : (w >> 1) == 2 ? q.z : q.w;
    return __uint_as_float((w & 1) ? (u & 0xFFFF0000u) : (u << 16));
  }
  __device__ __forceinline__ static float smem(const unsigned char *s, int i) {
    return bf16_to_f32(reinterpret_cast<const uint16_t *>(s)[i]);
  }
};

__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// The float just below x (x > -inf).
__device__ __forceinline__ float prev_float(float x) {
  if (x == 0.0f) return __int_as_float(static_cast<int>(0x80000001u));
  const int b = __float_as_int(x);
  return __int_as_float(x > 0.0f ? b - 1 : b + 1);
}

// A raw value r such that every x < r tempers below t (temperature is
// monotone): start near the preimage t*T and step down until the float
// below r tempers below t.  -inf when t is -inf (or on the way out).
__device__ __noinline__ float raw_floor(float t, const RowPlan P) {
  if (!(t > -INFINITY)) return -INFINITY;
  float r = __fmul_rn(t, P.T);
  for (int it = 0; it < 6 && r > -INFINITY; it++) {
    const float pr = prev_float(r);
    if (temper(pr, P) < t) return r;
    r = pr;
  }
  return -INFINITY;
}


// The sketch of a list row's stream: for every chunk, the largest raw value
// of each group of kSkGroupLanes lanes' vectors (64 f32 or 128 bf16
// elements), kept as the top 16 bits of its ordered value (0: no value);
// and one bit per group that holds a history id.  After the stream the
// k-th largest sketch value bounds the list from below, and only the groups
// whose maximum can reach the bound are read again.
constexpr int kSkGroupLanes = 4;
constexpr int kSkPerChunk = 32 / kSkGroupLanes;
constexpr int kGCap = 1024;     // candidate groups
constexpr int kInsertAt = 2;    // list rows: chunk at which a warp files the first history ids
constexpr int kCCap = 2048;     // candidate keys
// Lists longer than kTQK (up to PZ_TOP_K_MAX, launched as slice_long_kernel):
// a finer sketch, one entry per lane and 16 elements of a chunk (four f32 or
// two bf16 vectors), so that the k-th largest entry is a tight bound for
// k up to 1024 (about k entries are read again, 16 elements each).
constexpr int kFineElems = 16;
constexpr int kGCapFine = 4096;  // candidate entries of a long list
__host__ __device__ inline int fine_per_chunk(int elem_bytes) {
  return kChunkBytes / (elem_bytes * kFineElems);
}
__host__ __device__ inline int slice_sketch_entries(int V, int elem_bytes, int kcap) {
  if (kcap <= 1) return 0;
  const long long nchunks = (static_cast<long long>(V) * elem_bytes + kChunkBytes - 1) / kChunkBytes + 1;
  const long long per = kcap > kTQK ? fine_per_chunk(elem_bytes) : kSkPerChunk;
  return static_cast<int>((nchunks * per + 31) / 32 * 32);
}
__device__ __forceinline__ uint32_t sk16(float m) { return m == m ? f2ord(m) >> 16 : 0u; }

// The smallest sketch value whose 16-bit bucket's largest raw value
// tempers to tb or above (1 when every nonzero value's does), by
// bisection.  b16: the bound's sketch value (its bucket qualifies, since
// tb is the temper of its smallest raw value), or 0 for no bound (tb =
// -inf).  Nonzero sketch values are at least f2ord(-inf) >> 16, and from
// there the test is monotone in the value (temperature is monotone).
__device__ __forceinline__ uint32_t sketch_vmin(uint32_t b16, float tb, const RowPlan &P) {
  constexpr uint32_t kSkMin = kOrdNegInf >> 16;
  const uint32_t ord_inf = f2ord(INFINITY);
  auto qual = [&](uint32_t v) { return !(temper(ord2f(min((v << 16) | 0xFFFFu, ord_inf)), P) < tb); };
  if (b16 <= kSkMin || qual(kSkMin)) return 1u;
  uint32_t lo = kSkMin, hi = b16;  // qual(lo) false, qual(hi) true
  while (hi - lo > 1u) {
    const uint32_t mid = lo + (hi - lo) / 2u;
    if (qual(mid))
      hi = mid;
    else
      lo = mid;
  }
  return hi;
}

// A 32-bit global load issued where it stands (volatile asm keeps it ahead
// of the stream's copies), for a value first used after the stream.
__device__ __forceinline__ int ld_early(const int32_t *p) {
  int v;
  asm volatile("ld.global.nc.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// One warp: the bin of `bins` (256 counts; bin j holds the j-th smallest
// value range) that holds the need-th largest counted value, and how many
// of that bin's values are still needed; bin -1 if the bins hold fewer
// than `need` values.
__device__ __noinline__ void radix_pick(const uint32_t *bins, int need, int *bin_out, int *rem_out) {
  const int lane = threadIdx.x & 31;
  uint32_t c[8], sum = 0u;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    c[j] = bins[lane * 8 + j];
    sum += c[j];
  }
  uint32_t suf = sum;  // values in this lane's bins and above
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xFFFFFFFFu, suf, o);
    if (lane + o < 32) suf += t;
  }
  const uint32_t above = suf - sum;
  const uint32_t n = static_cast<uint32_t>(need);
  const uint32_t m = __ballot_sync(0xFFFFFFFFu, above < n && suf >= n);
  if (m == 0u) {
    if (lane == 0) {
      *bin_out = -1;
      *rem_out = 0;
    }
    return;
  }
  if (lane == __ffs(m) - 1) {
    uint32_t acc = above;
    for (int j = 7; j >= 0; j--) {
      if (acc + c[j] >= n) {
        *bin_out = lane * 8 + j;
        *rem_out = static_cast<int>(n - acc);
        break;
      }
      acc += c[j];
    }
  }
}

// After the stream the ring holds the row's list work (the candidates and
// the ranked list, or a split row's merged slice lists: up to kMergeKeys
// keys) and, from kFinalizeOff on, the decision's scratch (values,
// probabilities, order: 12 bytes a key).
constexpr int kMergeKeys = 2048;
constexpr int kFinalizeOff = kMergeKeys * 8;
static_assert(kSliceWarps * kSlots * kChunkBytes >= kFinalizeOff + 12 * PZ_TOP_K_MAX + 16,
              "the ring holds the merged lists and the decision's scratch");

// A split row's S slice lists (written to scratch by its S CTAs), merged
// by one warp into `lst`: for list rows the k_sel best keys in descending
// order, zero-padded to kcap; for argmax rows and k == 1 the best key, in
// gbest (and in lst[0] for top-k rows).  A slice that timed out marks the row.
struct MergedList {
  unsigned long long gbest;
  int n_sel;
  int timed_out;
};
__device__ __forceinline__ MergedList merge_slice_lists(const SliceArgs &A, int row, bool topk, int k_sel,
                                                     unsigned long long tau0,
                                                     unsigned long long *lst) {
  const int lane = threadIdx.x & 31;
  const int S = A.S;
  const size_t s0 = static_cast<size_t>(row - A.B1) * S;
  const unsigned long long *sk = A.slice_keys + s0 * static_cast<size_t>(A.kcap);
  const int32_t *sc = A.slice_cnt + s0;
  bool to = false;
  int n_sel = 0;
  unsigned long long gbest = 0ull;
  if (topk && k_sel > 1) {
    int n = 0;
    for (int s2 = 0; s2 < S; s2++) {
      const int raw = __ldcg(sc + s2);
      to |= ((raw >> 30) & 1) != 0;
      const int c = raw & 0xFFFF;
      for (int i = lane; i < c; i += 32) lst[n + i] = __ldcg(sk + static_cast<size_t>(s2) * A.kcap + i);
      n += c;
    }
    __syncwarp();
    if (n > k_sel) {
      const unsigned long long kth = warp_kth(lst, n, k_sel);
      n = warp_compact_ge(lst, n, kth);
    }
    n_sel = n;
    if (A.kcap <= 64) {
      warp_rank_sort_desc(lst, n_sel);
      for (int i = n_sel + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      __syncwarp();
    } else {
      for (int i = n_sel + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      warp_sort_desc(lst, A.kcap);
    }
  } else {
    unsigned long long bl = 0ull;
    bool lto = false;
    for (int s2 = lane; s2 < S; s2 += 32) {
      const int raw = __ldcg(sc + s2);
      lto |= ((raw >> 30) & 1) != 0;
      if ((raw & 0xFFFF) > 0) {
        const unsigned long long k = __ldcg(sk + static_cast<size_t>(s2) * A.kcap);
        bl = k > bl ? k : bl;
      }
    }
    to |= __any_sync(0xFFFFFFFFu, lto);
    gbest = warp_max_u64(bl);
    if (topk) {  // k_eff == 1 (or a rejected list length): the single best admitted key
      n_sel = gbest > tau0 ? 1 : 0;
      if (lane == 0) lst[0] = gbest;
      for (int i = 1 + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      __syncwarp();
    }
  }
  MergedList r;
  r.gbest = gbest;
  r.n_sel = n_sel;
  r.timed_out = to ? 1 : 0;
  return r;
}

// Shared memory of slice_kernel:
//   ring   NW x nslots x kChunkBytes  (per-warp copy rings; after the
//          stream: the list work and the rare exact rescan)
//   cbuf   block buffer keys           (lists longer than kTQK only)
//   hash   2 x hts words                (history ids and counts)
//   hbm    V/128 words                  (one bit per 4 columns: a history id there;
//                                        argmax launches only)
//   sketch 16-bit group maxima of the stream, then one bit per group (list rows)
__host__ __device__ inline int slice_cbuf_keys(int kcap) {
  return kcap > kTQK ? kcap + kCapB : 0;
}

// The bitmap only where there is room for it: in launches of argmax rows
// (no sketch).  Without it a lookup goes to the table directly.
__host__ __device__ inline int slice_hbm_words(int V, int hts, int kcap) {
  return hts > 0 && kcap <= 1 ? (V + 127) >> 7 : 0;
}

size_t slice_smem_bytes(int kcap, int hts, int nslots, int V, int elem_bytes) {
  const size_t sk = static_cast<size_t>(slice_sketch_entries(V, elem_bytes, kcap));
  return static_cast<size_t>(nslots) * kSliceWarps * kChunkBytes +
         sizeof(unsigned long long) * static_cast<size_t>(slice_cbuf_keys(kcap)) +
         sizeof(uint32_t) * (2 * static_cast<size_t>(hts) + slice_hbm_words(V, hts, kcap)) +
         sizeof(uint16_t) * sk + sizeof(uint32_t) * (sk / 32);
}

// Ring slots per warp: kSlots chunks of 2 KB in flight per warp (32 KB per
// CTA; with the history table and the sketch, four CTAs fit in an SM's
// 228 KB, 128 KB of copies in flight per SM).  After the stream the ring holds the list work: the candidates
// (up to kCCap keys from 8 KB on), the merged slice lists and the
// decision's scratch (from kFinalizeOff on), or the rescan buffer.
int slice_stages(int, int) { return kSlots; }

// CTAs per SM the registers allow: slice_kernel four (64 a thread),
// slice_long_kernel (launches with lists longer than kTQK) two.
int slice_ctas_per_sm_max(int kcap) { return kcap > kTQK ? 2 : 4; }

// Arrivals of first-wave CTAs per SM (counted across launches; consecutive
// arrivals on an SM take consecutive slots modulo its CTAs in flight).
__device__ unsigned g_slot_arrivals[256];

// One CTA per row (or per slice of L columns of a split row).  The slice's
// 16-byte-aligned body is cut into chunks of kChunkBytes; warp w streams
// chunks w, w + NW, ... through its own ring, each lane copying (cp.async)
// the four 16-byte vectors it reads and refilling its part of a slot as soon
// as it has read it, so warps never wait for one another while streaming.
// Per chunk a lane takes the maximum of its vectors.  List rows (k <= 64)
// keep only that, as the group maxima of the sketch, and find their list
// after the stream; argmax and long-list rows compare the tempered maximum
// with their bound (temperature is monotone) and look at the values of the
// lanes that reach it.

// LONG: the launch's lists may be longer than kTQK (slice_long_kernel, two
// CTAs per SM): those rows keep the fine sketch.  Otherwise every list is at
// most kTQK long (slice_kernel, four CTAs per SM).
template <typename T, bool LONG>
__device__ __forceinline__ void slice_body(const SliceArgs &A) {
  constexpr int NT = kSliceThreads;
  constexpr int NW = kSliceWarps;
  constexpr int VEC = LaneVec<T>::N;          // elements per 16-byte vector
  constexpr int XPT = 16;                     // rescan items per thread per round
  constexpr int XPE = 4;                      // extra-round items per thread per round
  constexpr int MAXPER = (PZ_TOP_K_MAX + kCapB) / NT;

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ SelShared sh;
  __shared__ unsigned long long s_red[NW];
  __shared__ uint32_t s_tauv;           // ordered value: the block's admission bound
  __shared__ RowPlan s_plan;
  __shared__ unsigned long long s_rng;  // the row's RNG state at entry
  __shared__ int s_sel[4];              // radix picks of the sketch bound
  __shared__ uint32_t s_skmax;          // largest sketch value of the slice
  __shared__ int s_x0nan, s_timeout, s_cnt, s_gcnt, s_n;

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  // CTA u < B1 takes all of row u; the rows after B1 come in S slices of L
  // columns each (the last CTAs launched, filling the GPU's final wave)
  const int u = blockIdx.x;
  if (LONG && A.deferred && u >= *A.n_defer) return;  // more CTAs than deferred rows
  const bool split = u >= A.B1;
  const int row = (LONG && A.deferred) ? A.defer_rows[u] : (split ? A.B1 + (u - A.B1) / A.S : u);
  const int a = split ? (u - A.B1) % A.S * A.L : 0;
  const int b = split ? min(A.V, a + A.L) : A.V;

  constexpr int NS = kSlots;
  unsigned char *ring = smem;
  unsigned long long *cbuf =
      reinterpret_cast<unsigned long long *>(smem + static_cast<size_t>(NW) * NS * kChunkBytes);
  uint32_t *hk = reinterpret_cast<uint32_t *>(cbuf + slice_cbuf_keys(A.kcap));
  uint32_t *hn = hk + A.hts;
  uint32_t *hbm = hn + A.hts;  // one bit per 4 columns of the row (argmax launches)
  const bool has_hbm = slice_hbm_words(A.V, A.hts, A.kcap) > 0;
  uint16_t *sketch = reinterpret_cast<uint16_t *>(hbm + slice_hbm_words(A.V, A.hts, A.kcap));
  const int sk_cap = slice_sketch_entries(A.V, static_cast<int>(sizeof(T)), A.kcap);
  uint32_t *gbm = reinterpret_cast<uint32_t *>(sketch + sk_cap);  // one bit per sketch group
  const uint32_t hmask = static_cast<uint32_t>(A.hts - 1);
  const uint32_t hshift = static_cast<uint32_t>(A.hshift);
  const T *rowp = static_cast<const T *>(A.logits) + static_cast<size_t>(row) * static_cast<size_t>(A.ld);

  // ---- aligned body, cut into chunks; the first copies go out first -------
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp + a);
  int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
  if (head > b - a) head = b - a;
  const int a_al = a + head;
  const int nvec = (b - a_al) / VEC;
  const int b_al = a_al + nvec * VEC;
  const int tail = b - b_al;
  const unsigned char *body = reinterpret_cast<const unsigned char *>(rowp + a_al);
  const int body_bytes = nvec * 16;
  const int nchunks = (body_bytes + kChunkBytes - 1) / kChunkBytes;
  const int nw = nchunks > warp ? (nchunks - warp + NW - 1) / NW : 0;  // this warp's chunks
  unsigned char *wring = ring + static_cast<size_t>(warp) * NS * kChunkBytes;

  // Warp-local chunk i (global chunk warp + NW*i) into ring slot `slot`:
  // each lane copies the four vectors it will read (u*32 + lane); in the
  // slice's last, short chunk the lanes past its end store NaN instead, so
  // the readers need no bounds tests.
  const unsigned char *lsrc = body + static_cast<size_t>(warp) * kChunkBytes + lane * 16;
  unsigned char *ldst = wring + lane * 16;
  auto issue = [&](int i, int slot) {
    const int c = warp + NW * i;
    const unsigned char *src = lsrc + static_cast<size_t>(i) * (NW * kChunkBytes);
    unsigned char *dst = ldst + slot * kChunkBytes;
    if (c != nchunks - 1) {
#pragma unroll
      for (int u = 0; u < kLaneVecs; u++) cp_async16(dst + u * 512, src + u * 512);
    } else {
      const int cv = (body_bytes - c * kChunkBytes) >> 4;
#pragma unroll
      for (int u = 0; u < kLaneVecs; u++) {
        if (u * 32 + lane < cv)
          cp_async16(dst + u * 512, src + u * 512);
        else
          *reinterpret_cast<uint4 *>(dst + u * 512) =
              make_uint4(LaneVec<T>::nan, LaneVec<T>::nan, LaneVec<T>::nan, LaneVec<T>::nan);
      }
    }
  };
  // one copy group per chunk slot, empty past the end, so that "chunk i has
  // landed" is always "at most NS - 1 groups pending"
  for (int i = 0; i < NS; i++) {
    if (i < nw) issue(i, i);
    cp_async_commit();
  }

  // ---- the row's settings and history extent (loaded together) ------------
  const pz_sampler_config cfg = A.cfg[row];
  int h0 = 0, h1 = 0;
  if (A.hist != nullptr && A.hist_off != nullptr) {
    h0 = A.hist_off[row];
    h1 = A.hist_off[row + 1];
  }
  const float x0raw = (a == 0 && A.v_offset == 0 && tid == 0) ? load_scalar<T>(rowp, 0) : 0.0f;
  // the row's RNG state, needed only by the decision: fetched now, with the settings
  const unsigned long long rng0 = (tid == 0 && !A.mode_emit) ? A.rng[row] : 0ull;
  const RowPlan P0 = plan_row(cfg, A.V_global);
  const bool greedy = P0.mode == kModeGreedy;
  // a list longer than this launch was sized for (hint broken): flag the row
  const bool bad_k = P0.mode == kModeTopK && (P0.keff > A.kmax || P0.keff > A.kcap);
  if (!LONG && bad_k && A.defer_kmax > 0 && P0.keff <= A.defer_kmax) {
    // a longer list than this launch keeps: slice_long_kernel samples the
    // row in the next launch (this CTA's first copies land before it leaves)
    cp_async_wait<0>();
    if (tid == 0) A.defer_rows[atomicAdd(A.n_defer, 1)] = row;
    return;
  }
  const int k_sel = (P0.mode == kModeTopK && !bad_k) ? P0.keff : 1;
  // lists up to kTQK long: the stream keeps only the sketch, and the list
  // comes from the groups that can reach its bound; longer lists: one
  // block-wide buffer.
  const bool use_tq = k_sel > 1 && k_sel <= kTQK;
  // longer lists (LONG launches only): the fine sketch, one entry per
  // kFineElems elements (one lane's kFineVPE vectors of a chunk)
  const bool fine = LONG && k_sel > kTQK;
  const bool skp = use_tq || fine;  // the stream keeps only a sketch
  constexpr int kFineEPL = kLaneVecs * VEC / kFineElems;  // fine entries per lane per chunk
  constexpr int kFineVPE = kFineElems / VEC;               // vectors per fine entry
  constexpr int kFineEPC = 32 * kFineEPL;                  // fine entries per chunk
  const int sk_per_chunk = fine ? kFineEPC : kSkPerChunk;
  // the sketch covers a whole row (the largest slice), so this always holds
  const bool sketch_ok = nchunks * sk_per_chunk <= sk_cap;
  const unsigned long long tau0 = (P0.mode == kModeTopK) ? key_topk_floor() : 0ull;
  const float tau0_f = tau0 == 0ull ? -INFINITY : key_val(tau0);
  const uint32_t goff = static_cast<uint32_t>(A.v_offset);
  const int cap = A.kcap + kCapB;         // block list buffer
  const int hwm = A.kcap + kCapB / 2;

  const int H = P0.pen_on ? h1 - h0 : 0;
  const int32_t *hrow = A.hist + h0;
  const bool too_long = H > A.hcap;
  const bool hist_on = H > 0 && !too_long && A.hts > 0;
  // Penalties that can only lower a value (rep >= 1, freq >= 0, pres >= 0):
  // a history id whose raw value is below the bound stays below it, so list
  // rows score history ids among the read-again groups with their penalised
  // value.  Other penalties: every history id in the history round.
  const bool pen_dec = P0.rep >= 1.0f && P0.freq >= 0.0f && P0.pres >= 0.0f;
  const bool hist_stream = hist_on && skp && pen_dec;

  if (tid == 0) {
    if (skp && A.stagger_ns > 0 && blockIdx.x < static_cast<unsigned>(A.stagger_ctas)) {
      // the first wave: this CTA's slot on its SM (arrival order), and a
      // start that many stagger steps late (the first copies already fly;
      // the wait is bounded by the clock and by a step count)
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      const unsigned slot = atomicAdd(&g_slot_arrivals[smid & 255u], 1u) % static_cast<unsigned>(A.stagger_occ);
      const unsigned long long wait = static_cast<unsigned long long>(slot) * static_cast<unsigned>(A.stagger_ns);
      if (wait > 0ull) {
        unsigned long long t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        for (int it = 0; it < 20000; it++) {
          __nanosleep(500);
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (t - t0 >= wait) break;
        }
      }
    }
    s_plan = P0;
    s_rng = rng0;
    s_x0nan = 0;
    s_timeout = 0;
    s_cnt = 0;
    s_tauv = f2ord(tau0_f);
    s_skmax = 0u;
    sh.n = 0;
    sh.tau = tau0;
  }
  __syncthreads();
  // The row plan from here on is read from shared memory: its fields are
  // used now and then, and would otherwise hold registers through the stream.
  const RowPlan &P = s_plan;

  // ---- the slice's history ids and counts ---------------------------------
  // The first NT*IPT ids are loaded now, while the first copies fly.  Argmax
  // and long-list rows build the table before the stream, which consults
  // it; list rows during it (their stream keeps only the sketch, and the
  // table is first needed after it).
  constexpr int IPT = 4;
  int hid[IPT];
#pragma unroll
  for (int u = 0; u < IPT; u++) {
    const int j = u * NT + tid;
    hid[u] = hist_on && j < H ? static_cast<int>(static_cast<long long>(ld_early(hrow + j)) - A.v_offset) : -1;
  }
  auto init_hist = [&]() {
    for (int i = tid; i < A.hts; i += NT) {
      hk[i] = kHashEmpty;
      hn[i] = 0u;
    }
    for (int i = tid; i < slice_hbm_words(A.V, A.hts, A.kcap); i += NT) hbm[i] = 0u;
    if (skp)
      for (int i = tid; i < sk_cap / 32; i += NT) gbm[i] = 0u;
  };
  auto insert_ids = [&](const int (&t)[IPT]) {
#pragma unroll
    for (int u = 0; u < IPT; u++)
      if (t[u] >= a && t[u] < b) {
        hash_insert(hk, hn, hmask, hshift, static_cast<uint32_t>(t[u]));
        if (has_hbm) atomicOr(&hbm[t[u] >> 7], 1u << ((t[u] >> 2) & 31));
        if (skp && t[u] >= a_al && t[u] < b_al) {
          // the sketch group of column t: chunk, then the lane of its vector
          // (and for the fine sketch, which of the lane's entries)
          constexpr int kPerChunk = kChunkBytes / static_cast<int>(sizeof(T));
          const int off = t[u] - a_al;
          const int vi = (off % kPerChunk) / VEC;
          const int g = fine ? (off / kPerChunk) * kFineEPC + (vi & 31) * kFineEPL + (vi >> 5) / kFineVPE
                             : (off / kPerChunk) * kSkPerChunk + (vi & 31) / kSkGroupLanes;
          atomicOr(&gbm[g >> 5], 1u << (g & 31));
        }
      }
  };
  // argmax rows take the history round right after the table is built, so
  // the logits the ids name are fetched into L2 first
  const bool pre = !skp;
  auto insert_rest = [&]() {  // the ids past the first NT*IPT
    for (int base = NT * IPT; base < H; base += NT * IPT) {
      int t[IPT];
#pragma unroll
      for (int u = 0; u < IPT; u++) {
        const int j = base + u * NT + tid;
        t[u] = j < H ? static_cast<int>(static_cast<long long>(hrow[j]) - A.v_offset) : -1;
      }
      if (pre) {
#pragma unroll
        for (int u = 0; u < IPT; u++)
          if (t[u] >= a && t[u] < b) prefetch_l2(rowp + t[u]);
      }
      insert_ids(t);
    }
  };
  if (hist_on && !skp) {
    init_hist();
    if (pre) {
#pragma unroll
      for (int u = 0; u < IPT; u++)
        if (hid[u] >= a && hid[u] < b) prefetch_l2(rowp + hid[u]);
    }
    __syncthreads();  // the table is initialised
    insert_ids(hid);
    insert_rest();
    __syncthreads();
  }
  if (hist_on && skp) {
    // list rows: the table is filled during the stream (the first ids at the
    // warp's chunk kInsertAt, when their loads have landed), the rest after it
    init_hist();
    __syncthreads();
  }
  // the bitmap answers most lookups; a set bit sends the id to the table
  auto hist_count = [&](int li) -> int {
    return hist_on && (!has_hbm || ((hbm[li >> 7] >> ((li >> 2) & 31)) & 1u) != 0u)
               ? hash_count(hk, hn, hmask, hshift, static_cast<uint32_t>(li))
               : 0;
  };
  auto in_hist = [&](int li) -> bool { return hist_count(li) > 0; };

  unsigned long long best = 0ull;       // argmax path
  float best_f = -INFINITY;
  // Admission bound: a value below it cannot make the slice's list (at
  // least k_sel elements of the slice are at or above it).  Shared by the
  // warps through s_tauv.
  float tau_wf = tau0_f;
  const float nanf_ = __int_as_float(0x7FC00000);

  auto offer_key = [&](unsigned long long key) {  // argmax rows
    if (key > best) {
      best = key;
      best_f = key_val(key);
    }
  };
  // list rows: the candidates read again after the stream, and their bound
  // (long lists: in the block buffer)
  unsigned long long *ck = fine ? cbuf : reinterpret_cast<unsigned long long *>(ring + 8192);
  const int ccap = fine ? cap : kCCap;
  float tb = -INFINITY;
  auto cand_push = [&](unsigned long long key) {
    const int p = atomicAdd(&s_cnt, 1);
    if (p < ccap) ck[p] = key;
  };

  // ---- row 0's first logit (the NaN rule of argmax.c:3-13) ---------------
  // (with the table built: before the stream, or after it for list rows)
  auto x0_check = [&]() {
    if (a == 0 && goff == 0 && tid == 0) {
      float x = x0raw;
      const int c = hist_on ? hash_count(hk, hn, hmask, hshift, 0u) : 0;
      if (c > 0) x = penalize(x, c, P);
      const float v = greedy ? x : temper(x, P);
      s_x0nan = (v != v) ? 1 : 0;
    }
  };
  if (!skp) x0_check();

  // ---- head, tail and the penalised history ids: exact keys ---------------
  // Argmax rows take them before the stream (the best of them is a strong
  // first bound); list rows after it (the tight bound rejects most of them).
  // A history id in the head or tail is scored there, with its count.
  auto history_round = [&]() {
    const int n_extra = head + tail + ((hist_on && !hist_stream) ? A.hts : 0);
    for (int base = 0; base < n_extra; base += NT * XPE) {
      float xv[XPE];
      int lis[XPE], cnts[XPE];
      uint32_t have = 0;
      // the items' columns first (column a stands in for an empty item), then
      // every load at once, then the values
  #pragma unroll
      for (int e = 0; e < XPE; e++) {
        const int it = base + e * NT + tid;
        int li = a, cnt = 0;
        bool h = false;
        if (it < head) {
          li = a + it;
          cnt = hist_count(li);
          h = true;
        } else if (it < head + tail) {
          li = b_al + (it - head);
          cnt = hist_count(li);
          h = true;
        } else if (it < n_extra) {
          const int i = it - head - tail;
          const uint32_t t = hk[i];
          if (t != kHashEmpty && static_cast<int>(t) >= a_al && static_cast<int>(t) < b_al) {
            li = static_cast<int>(t);
            cnt = static_cast<int>(hn[i]);
            h = true;
          }
        }
        lis[e] = li;
        cnts[e] = cnt;
        have |= h ? (1u << e) : 0u;
      }
  #pragma unroll
      for (int e = 0; e < XPE; e++) xv[e] = load_scalar<T>(rowp, lis[e]);
  #pragma unroll
      for (int e = 0; e < XPE; e++) {
        if (!((have >> e) & 1u)) continue;
        float x = xv[e];
        if (cnts[e] > 0) x = penalize(x, cnts[e], P);
        xv[e] = greedy ? x : temper(x, P);
      }
      if (skp) {
        // after the stream the bound is tight: most values stop here
  #pragma unroll
        for (int e = 0; e < XPE; e++)
          if (((have >> e) & 1u) && xv[e] >= tb) {
            const unsigned long long key = mkkey(xv[e], static_cast<uint32_t>(lis[e]) + goff);
            if (key > tau0) cand_push(key);
          }
      } else {
  #pragma unroll
        for (int e = 0; e < XPE; e++)
          if (((have >> e) & 1u) && xv[e] >= tau_wf)
            offer_key(mkkey(xv[e], static_cast<uint32_t>(lis[e]) + goff));
      }
    }
  };
  if (!skp) {
    history_round();
    const uint32_t bo = __reduce_max_sync(0xFFFFFFFFu, best != 0ull ? f2ord(best_f) : kOrdNegInf);
    if (lane == 0) atomicMax(&s_tauv, bo);
  }

  // ---- the stream ----------------------------------------------------------
  // Temperature of the stream: a multiplication by `scale` (1 for greedy
  // rows), which is monotone, so the tempered chunk maximum is the maximum
  // of the tempered values; with PZ_CFG_TEMP_DIVIDE a division, tested
  // through a raw threshold instead.
  const bool mulT = greedy || !P.divide;
  const float scale = greedy ? 1.0f : P.inv_T;
  if (skp) {
    // List rows: the stream only records the sketch (each group's raw
    // maximum; temperature is monotone, so it orders the tempered values too).
    int slot = 0;
    uint32_t run_max = 0u;  // the warp's largest sketch value so far
    for (int i = 0; i < nw; i++) {
      cp_async_wait<NS - 1>();
      const unsigned char *lsb = ldst + slot * kChunkBytes;
      float mv[kLaneVecs];
#pragma unroll
      for (int u = 0; u < kLaneVecs; u++) mv[u] = LaneVec<T>::vmax(*reinterpret_cast<const uint4 *>(lsb + u * 512));
      float m = max_of(mv);
      // the lane's vectors of the slot are in registers (m depends on all of
      // them, and the empty asm orders m's computation before the copies):
      // refill the slot before the reductions, so that the copy is in flight
      // that much sooner
      asm volatile("" ::"f"(m));
      if (i + NS < nw) issue(i + NS, slot);
      cp_async_commit();
      if (fine) {
        // the lane's own entries (kFineVPE vectors each), stored together
        uint32_t pk = 0u;
#pragma unroll
        for (int j = 0; j < kFineEPL; j++) {
          float q = mv[j * kFineVPE];
#pragma unroll
          for (int t = 1; t < kFineVPE; t++) q = fmaxf(q, mv[j * kFineVPE + t]);
          pk |= sk16(q) << (16 * j);
        }
        if (sketch_ok) {
          const int g0 = (warp + NW * i) * kFineEPC + lane * kFineEPL;
          if (kFineEPL == 2)
            *reinterpret_cast<uint32_t *>(sketch + g0) = pk;
          else
            sketch[g0] = static_cast<uint16_t>(pk);
        }
        run_max = max(run_max, sk16(m));
      } else {
#pragma unroll
        for (int o = 1; o < kSkGroupLanes; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        const uint32_t v16 = sk16(m);
        if ((lane & (kSkGroupLanes - 1)) == 0 && sketch_ok)
          sketch[(warp + NW * i) * kSkPerChunk + lane / kSkGroupLanes] = static_cast<uint16_t>(v16);
        run_max = max(run_max, v16);
      }
      if (i == kInsertAt && hist_on) insert_ids(hid);
      slot = slot + 1 == NS ? 0 : slot + 1;
    }
    {
      const uint32_t wmax = __reduce_max_sync(0xFFFFFFFFu, run_max);
      if (lane == 0 && wmax > 0u) atomicMax(&s_skmax, wmax);
    }
    if (hist_on && nw <= kInsertAt) insert_ids(hid);  // a warp with too few chunks
  } else {
    // argmax: the threshold is the block's best value so far (warp-uniform);
    // only a lane's maximum and its ties can beat it
    uint32_t seen_tau = *reinterpret_cast<volatile uint32_t *>(&s_tauv);
    tau_wf = fmaxf(tau_wf, ord2f(seen_tau));
    float rthr = mulT ? 0.0f : raw_floor(tau_wf, P);
    int slot = 0;
    for (int i = 0; i < nw; i++) {
      cp_async_wait<NS - 1>();
      const unsigned char *sb = wring + slot * kChunkBytes;
      const unsigned char *lsb = ldst + slot * kChunkBytes;
      uint4 q[kLaneVecs];
      float mv[kLaneVecs];
#pragma unroll
      for (int u = 0; u < kLaneVecs; u++) {
        q[u] = *reinterpret_cast<const uint4 *>(lsb + u * 512);
        mv[u] = LaneVec<T>::vmax(q[u]);
      }
      const float m = max_of(mv);
      const bool hot = mulT ? !(__fmul_rn(m, scale) < tau_wf) : !(m < rthr);
      if (__any_sync(0xFFFFFFFFu, hot)) {
        const int e0 = a_al + (warp + NW * i) * (kChunkBytes / static_cast<int>(sizeof(T)));
        uint32_t pend = 0;
        if (hot) {
          // the lane's maximum and its ties; every element at or above the
          // threshold when the maximum may be a (penalised) history id
          const float te = hist_on ? (mulT ? tau_wf : rthr) : (mulT ? fmaxf(tau_wf, __fmul_rn(m, scale)) : fmaxf(rthr, m));
#pragma unroll
          for (int u = 0; u < kLaneVecs; u++) {
            if ((mulT ? __fmul_rn(mv[u], scale) : mv[u]) < te) continue;
#pragma unroll
            for (int w = 0; w < VEC; w++) {
              const float x = LaneVec<T>::elem(q[u], w);
              if ((mulT ? __fmul_rn(x, scale) : x) >= te) pend |= 1u << (u * VEC + w);
            }
          }
        }
        while (pend) {
          const int e = __ffs(pend) - 1;
          pend &= pend - 1;
          const int pos = ((e / VEC) * 32 + lane) * VEC + (e % VEC);
          const int li = e0 + pos;
          if (in_hist(li)) continue;
          const float x = LaneVec<T>::smem(sb, pos);
          const float v = greedy ? x : temper(x, P);
          const unsigned long long key = mkkey(v, static_cast<uint32_t>(li) + goff);
          if (key > best) {
            best = key;
            best_f = v;
          }
        }
        const uint32_t bo = __reduce_max_sync(0xFFFFFFFFu, best != 0ull ? f2ord(best_f) : kOrdNegInf);
        if (lane == 0 && bo > *reinterpret_cast<volatile uint32_t *>(&s_tauv)) atomicMax(&s_tauv, bo);
      }
      if (i + NS < nw) issue(i + NS, slot);
      cp_async_commit();
      const uint32_t tb = *reinterpret_cast<volatile uint32_t *>(&s_tauv);
      if (tb != seen_tau) {
        seen_tau = tb;
        const float tf = ord2f(tb);
        if (tf > tau_wf) {
          tau_wf = tf;
          if (!mulT) rthr = raw_floor(tf, P);
        }
      }
      slot = slot + 1 == NS ? 0 : slot + 1;
    }
  }
  cp_async_wait<0>();
  // The CTA that will most likely take this slot next (one wave of CTAs
  // later) finds its row's settings in L2: its setup waits on them.
  if (tid == 0 && !split && A.stagger_ctas > 0) {
    const int nu = u + A.stagger_ctas;
    if (nu < A.B1) {
      prefetch_l2(A.cfg + nu);
      if (A.hist_off != nullptr) prefetch_l2(A.hist_off + nu);
      if (A.rng != nullptr) prefetch_l2(A.rng + nu);
    }
  }

  if (skp && hist_on) insert_rest();
  __syncthreads();
  const bool timed_out = s_timeout != 0;

  // ---- this slice's list -> scratch ---------------------------------------
  unsigned long long *lst = reinterpret_cast<unsigned long long *>(ring);  // the list
  unsigned long long *rb = fine ? cbuf : lst;                              // block buffer
  if (!skp) {
    best = warp_max_u64(best);
    if (lane == 0) s_red[warp] = best;
  }
  __syncthreads();
  bool exact_rescan = false;
  int n_tq = 0;  // list length (sketch path)
  if (skp) {
    // ---- a list row's list, from the sketch ---------------------------------
    // The bound: the k-th largest sketch value, by a two-pass radix select
    // over the 16-bit values; tb, the tempered floor of that value.
    // Candidates, each with its exact key: every element at or above tb of
    // the groups whose maximum can temper to tb or above, the head and tail,
    // and (penalties that can raise a value) every history id.  Every
    // element at or above tb is a candidate, so if k of them are, the list
    // (their best k_sel, ranked) is exact.  The first pass counts every
    // group; a group maximum that is a history id can fall below tb once
    // penalised, and if fewer than k candidates remain, a second pass bounds
    // with the groups that hold no history id, whose k maxima stand.
    // Long lists (fine sketch): the same with one entry per kFineElems
    // elements as the group, and the list ranked by a block-wide select and
    // sort in the block buffer.
    const int ng = sketch_ok ? nchunks * sk_per_chunk : 0;
    const int gcap = fine ? kGCapFine : kGCap;
    uint32_t *bins = reinterpret_cast<uint32_t *>(ring);  // 2 x 256 counts
    int *glist = reinterpret_cast<int *>(ring + 2048);    // gcap groups
    unsigned long long *sorted = reinterpret_cast<unsigned long long *>(ring + 6144);
    int nc = 0, ngs = 0;
    for (int pass = 0; pass < 2; pass++) {
      const bool all = pass == 0;
      for (int i = tid; i < 512; i += NT) bins[i] = 0u;
      if (tid == 0) {
        s_cnt = 0;
        s_gcnt = 0;
      }
      __syncthreads();
      if (pass == 0) x0_check();  // the history table is complete
      auto eligible = [&](int g) -> bool {
        return all || !(hist_on && ((gbm[g >> 5] >> (g & 31)) & 1u) != 0u);
      };
      // pass 0 bounds a few places lower, so that a handful of group maxima
      // that are penalised history ids do not force the second pass
      const int kb = all && hist_on ? k_sel + 8 : k_sel;
      // usually one pass: the values within 255 of the largest, M, each in
      // its own bin; else the high byte, then the low byte
      const uint32_t M = s_skmax;
      uint32_t b16 = 0u;  // 0: fewer than k groups, no bound
      if (fine) {
        // k up to 1024 is rarely within 255 of the largest: the high byte,
        // then the low byte within its bin, each count aggregated per warp
        // (the values crowd a few bins)
        auto count = [&](int hsel, uint32_t *bn) {
          for (int g0 = 0; g0 < ng; g0 += NT) {
            const int g = g0 + tid;
            int d = -1;
            if (g < ng) {
              const uint32_t v = sketch[g];
              if (v != 0u && eligible(g)) {
                if (hsel < 0)
                  d = static_cast<int>(v >> 8);
                else if (static_cast<int>(v >> 8) == hsel)
                  d = static_cast<int>(v & 255u);
              }
            }
            const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
            if (d >= 0 && lane == __ffs(peers) - 1) atomicAdd(&bn[d], static_cast<uint32_t>(__popc(peers)));
          }
        };
        count(-1, bins);
        __syncthreads();
        if (warp == 0) radix_pick(bins, kb, &s_sel[0], &s_sel[1]);
        __syncthreads();
        const int hb = s_sel[0];
        if (hb >= 0) {
          const int need = s_sel[1];
          count(hb, bins + 256);
          __syncthreads();
          if (warp == 0) radix_pick(bins + 256, need, &s_sel[2], &s_sel[3]);
          __syncthreads();
          b16 = (static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(s_sel[2]);
        }
      } else {
      for (int g = tid; g < ng; g += NT) {
        const uint32_t v = sketch[g];
        if (v != 0u && M - v < 256u && eligible(g)) atomicAdd(&bins[255u - (M - v)], 1u);
      }
      __syncthreads();
      if (warp == 0) radix_pick(bins, kb, &s_sel[0], &s_sel[1]);
      __syncthreads();
      if (s_sel[0] >= 0) {
        b16 = M - 255u + static_cast<uint32_t>(s_sel[0]);
      } else {
        for (int i = tid; i < 256; i += NT) bins[i] = 0u;
        __syncthreads();
        for (int g = tid; g < ng; g += NT) {
          const uint32_t v = sketch[g];
          if (v != 0u && eligible(g)) atomicAdd(&bins[v >> 8], 1u);
        }
        __syncthreads();
        if (warp == 0) radix_pick(bins, kb, &s_sel[0], &s_sel[1]);
        __syncthreads();
        const int hb = s_sel[0];
        if (hb >= 0) {
          const int need = s_sel[1];
          for (int g = tid; g < ng; g += NT) {
            const uint32_t v = sketch[g];
            if (static_cast<int>(v >> 8) == hb && eligible(g)) atomicAdd(&bins[256 + (v & 255u)], 1u);
          }
          __syncthreads();
          if (warp == 0) radix_pick(bins + 256, need, &s_sel[2], &s_sel[3]);
          __syncthreads();
          b16 = (static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(s_sel[2]);
        }
      }
      }
      const uint32_t bord = b16 << 16;
      tb = bord > kOrdNegInf ? temper(ord2f(bord), P) : -INFINITY;
      // the groups to read again: a maximum below ord2f((v + 1) << 16)
      // tempers to at most that value's temper, so a group qualifies when
      // the largest raw value of its 16-bit bucket tempers to tb or above;
      // that is the groups with sketch value v >= vmin
      const uint32_t vmin = sketch_vmin(b16, tb, P);
      for (int g0 = 0; g0 < ng; g0 += NT) {
        const int g = g0 + tid;
        const bool sel = g < ng && sketch[g] >= vmin;
        const uint32_t bal = __ballot_sync(0xFFFFFFFFu, sel);
        int base = 0;
        if (lane == 0 && bal) base = atomicAdd(&s_gcnt, __popc(bal));
        base = __shfl_sync(0xFFFFFFFFu, base, 0);
        if (sel) {
          const int p = base + __popc(bal & lanemask_lt());
          if (p < gcap) glist[p] = g;
        }
      }
      __syncthreads();
      ngs = s_gcnt;
      if (ngs <= gcap) {
        // each group: kSkGroupLanes lanes x kLaneVecs vectors (fine: one
        // lane's kFineVPE vectors), read from L2 or HBM, XG at a time per
        // thread with all loads in flight together
        const int GV = fine ? kFineVPE : kSkGroupLanes * kLaneVecs;
        constexpr int XG = 4;
        constexpr int kPerChunk = kChunkBytes / static_cast<int>(sizeof(T));
        for (int base = 0; base < ngs * GV; base += NT * XG) {
          uint4 qv[XG];
          int el[XG];
          uint32_t ok = 0u, gh = 0u;  // loaded; in a group with a history id
#pragma unroll
          for (int e = 0; e < XG; e++) {
            const int it = base + e * NT + tid;
            el[e] = 0;
            if (it < ngs * GV) {
              const int g = glist[it / GV];
              const int v = it % GV;
              int c, vi;
              if (fine) {
                c = g / kFineEPC;
                const int r = g % kFineEPC;
                vi = ((r % kFineEPL) * kFineVPE + v) * 32 + r / kFineEPL;
              } else {
                c = g / kSkPerChunk;
                const int pq = g % kSkPerChunk;
                vi = (v / kSkGroupLanes) * 32 + pq * kSkGroupLanes + (v % kSkGroupLanes);
              }
              const int cv = c == nchunks - 1 ? (body_bytes - c * kChunkBytes) >> 4 : kChunkBytes / 16;
              if (vi < cv) {
                qv[e] = __ldg(reinterpret_cast<const uint4 *>(body + static_cast<size_t>(c) * kChunkBytes) + vi);
                el[e] = a_al + c * kPerChunk + vi * VEC;
                ok |= 1u << e;
                if (hist_on && ((gbm[g >> 5] >> (g & 31)) & 1u) != 0u) gh |= 1u << e;
              }
            }
          }
#pragma unroll
          for (int e = 0; e < XG; e++) {
            if (!((ok >> e) & 1u)) continue;
#pragma unroll
            for (int w = 0; w < VEC; w++) {
              const int li = el[e] + w;
              float x = LaneVec<T>::elem(qv[e], w);
              float v = temper(x, P);
              if (v >= tb) {
                // only a value that reaches the bound unpenalised is looked
                // up: a penalty that can only lower it cannot lift a value
                // below the bound, and the other penalties' ids are scored
                // in the history round
                if ((gh >> e) & 1u) {
                  const int hc = hist_count(li);
                  if (hc > 0) {
                    if (!pen_dec) continue;
                    v = temper(penalize(x, hc, P), P);
                    if (!(v >= tb)) continue;
                  }
                }
                const unsigned long long key = mkkey(v, static_cast<uint32_t>(li) + goff);
                if (key > tau0) cand_push(key);
              }
            }
          }
        }
        history_round();
      }
      __syncthreads();
      nc = s_cnt;
      if (ngs > gcap || nc > ccap) break;
      if (nc >= k_sel || !hist_on || b16 == 0u) break;
      __syncthreads();  // every thread has read s_cnt before the next pass resets it
    }
    if (ngs > gcap || nc > ccap || !sketch_ok) {
      exact_rescan = true;  // too many to keep: redo the slice below
    } else if (fine) {
      // the best k_sel candidates (block-wide radix select), then sorted
      // descending (bitonic, padded with zero keys to a power of two)
      int n = nc;
      if (n > k_sel) {
        block_select<NT, MAXPER>(cbuf, n, k_sel, sh);
        n = k_sel;
      }
      int n2 = 1;
      while (n2 < n) n2 <<= 1;
      for (int i = n + tid; i < n2; i += NT) cbuf[i] = 0ull;
      block_sort_desc<NT>(cbuf, n2);
      n_tq = n;
      lst = cbuf;
    } else {
      for (int i = tid; i < nc; i += NT) {
        const unsigned long long key = ck[i];
        int r = 0;
        for (int j = 0; j < nc; j++) r += ck[j] > key ? 1 : 0;
        if (r < k_sel) sorted[r] = key;
      }
      __syncthreads();
      n_tq = nc < k_sel ? nc : k_sel;
      lst = sorted;
    }
  }
  if (exact_rescan) {
    // rare: redo the slice exactly with a block-wide buffer (all threads)
    if (tid == 0) {
      sh.n = 0;
      sh.tau = tau0;
    }
    __syncthreads();
    for (int base = a; base < b; base += NT * XPT) {
      unsigned long long keys[XPT];
      uint32_t valid = 0;
#pragma unroll
      for (int e = 0; e < XPT; e++) {
        keys[e] = 0ull;
        const int li = base + e * NT + tid;
        if (li < b) {
          float x = load_scalar<T>(rowp, li);
          const int c = hist_on ? hash_count(hk, hn, hmask, hshift, static_cast<uint32_t>(li)) : 0;
          if (c > 0) x = penalize(x, c, P);
          const float v = temper(x, P);
          if (v == v) {
            keys[e] = mkkey(v, static_cast<uint32_t>(li) + goff);
            valid |= 1u << e;
          }
        }
      }
      offer_round<NT, MAXPER, XPT>(rb, cap, hwm, k_sel, sh, keys, valid);
    }
    __syncthreads();
    int n = sh.n < cap ? sh.n : cap;
    __syncthreads();
    if (n > k_sel) {
      block_select<NT, MAXPER>(rb, n, k_sel, sh);
      n = k_sel;
    }
    if (tid == 0) s_n = n;
    __syncthreads();
  }
  if (warp != 0) return;

  // The row's list for the decision: this CTA's own (the whole row), or,
  // for a split row, the merge of its S slice lists by whichever of its
  // CTAs finishes last.  The decision's scratch sits in the ring from
  // kFinalizeOff on, after the list work or the merged lists.
  float *fe = reinterpret_cast<float *>(ring + kFinalizeOff);
  float *fp = fe + A.kcap;
  int *ford = reinterpret_cast<int *>(fp + A.kcap);
  int *s_tokp = ford + A.kcap;
  unsigned long long *fl = lst;
  int n_sel = 0;
  unsigned long long gbest = 0ull;
  bool row_timed_out = timed_out, x0nan = s_x0nan != 0;
  if (blockIdx.x < static_cast<unsigned>(A.B1)) {
    if (exact_rescan) {
      fl = rb;
      n_sel = s_n;
      for (int i = n_sel + lane; i < A.kcap; i += 32) fl[i] = 0ull;
      __syncwarp();
      warp_sort_desc(fl, A.kcap);
    } else if (skp) {
      n_sel = n_tq;
      for (int i = n_sel + lane; i < A.kcap; i += 32) fl[i] = 0ull;
      __syncwarp();
    } else {
      const unsigned long long bl = lane < NW ? s_red[lane] : 0ull;
      gbest = warp_max_u64(bl);
      if (P.mode == kModeTopK) {  // k_eff == 1 (or a rejected list length)
        n_sel = gbest > tau0 ? 1 : 0;
        if (lane == 0) fl[0] = gbest;
        for (int i = 1 + lane; i < A.kcap; i += 32) fl[i] = 0ull;
        __syncwarp();
      }
    }
  } else {
    int m = 0;
    const size_t si = static_cast<size_t>(blockIdx.x) - A.B1;  // (row - B1) * S + slice
    unsigned long long *dst = A.slice_keys + si * static_cast<size_t>(A.kcap);
    if (exact_rescan) {
      m = s_n;
      for (int i = lane; i < m; i += 32) dst[i] = rb[i];
    } else if (skp) {
      m = n_tq;
      for (int i = lane; i < m; i += 32) dst[i] = lst[i];
    } else {
      unsigned long long bl = lane < NW ? s_red[lane] : 0ull;
      bl = warp_max_u64(bl);
      m = bl > tau0 ? 1 : 0;
      if (lane == 0 && m) dst[0] = bl;
    }
    if (lane == 0) {
      A.slice_cnt[si] = m | (timed_out ? (1 << 30) : 0);
      if (a == 0) A.row_flags[row] = s_x0nan ? 1u : 0u;
    }
    // publish the list, then take a ticket: the row's S-th arrival decides
    __threadfence();
    __syncwarp();
    unsigned last = 0u;
    if (lane == 0) {
      last = atomicAdd(A.row_arrive + row, 1u) == static_cast<unsigned>(A.S - 1) ? 1u : 0u;
      if (last) A.row_arrive[row] = 0u;  // ready for the next launch
    }
    last = __shfl_sync(0xFFFFFFFFu, last, 0);
    if (!last) return;
    __threadfence();
    fl = reinterpret_cast<unsigned long long *>(ring);
    const MergedList ml = merge_slice_lists(A, row, P.mode == kModeTopK, k_sel, tau0, fl);
    n_sel = ml.n_sel;
    gbest = ml.gbest;
    row_timed_out |= ml.timed_out != 0;
    x0nan = (__ldcg(A.row_flags + row) & 1u) != 0u;
  }
  finalize_row<LONG>(A, row, P, bad_k, too_long, row_timed_out, x0nan, fl, n_sel, gbest, s_rng, fe, fp,
                     ford, s_tokp);
}

template <typename T>
__global__ void __launch_bounds__(kSliceThreads, 4) slice_kernel(const SliceArgs A) {
  slice_body<T, false>(A);
}

// Launches whose list length (kcap) is above kTQK: the fine sketch for the
// long lists, two CTAs per SM (room for its sketch and a 2048-id history).
template <typename T>
__global__ void __launch_bounds__(kSliceThreads, 2) slice_long_kernel(const SliceArgs A) {
  slice_body<T, true>(A);
}


// ---------------------------------------------------------------------------
// full_kernel: rows that need the whole row's distribution (k = 0).
//
// One CTA per row (the grid loops over the rows slice_kernel handed over).
//   pass 1   index order: e_i = exp(v_i - max) for the values the max-20
//            filter keeps (top_p.c:57-65) or for every value (softmax.c:12-16),
//            stored to scratch; the reference's sequential float normaliser
//            replayed exactly (pz_seqsum.cuh); top-p rows also count the e
//            values into 512 bins (16 per binade).
//   softmax  the CDF walk in index order over fl(e_i * inv)
//            (generate.c:159-167), a second exact replay.
//   top-p    a probability bound P whose mass (a lower bound from the bins)
//            clears top_p with room to spare; the entries with
//            prob = fl(e_i * inv) >= P are exactly a prefix of the
//            reference's stable sort (prob desc, index asc, top_p.c:77), so
//            only they are collected (in index order) and sorted (stable
//            radix sort, in shared memory when they fit).  The cumulative
//            cutoff (:80-88), the truncated sum (:91-93) and the draw
//            (:96-105) are replayed over that prefix; if the cutoff is not
//            inside it (the bound was not conservative enough), every entry
//            is collected instead.
// ---------------------------------------------------------------------------
constexpr int kEBins = 2048;
constexpr int kSeqHead = 1024;  // terms of each sum added in order by one thread
// Bin of a positive e value: 64 bins per binade, from 2^-32 up (e <= 1).
// The bins' lower edges give a lower bound of the mass above a bin, within
// 2^(1/64) (1.1 %) of it, so the collected prefix ends close to the cutoff.
__device__ __forceinline__ int ebin(float e) {
  const int b = static_cast<int>(__float_as_uint(e) >> 17) - (95 << 6);
  return b < 0 ? 0 : (b >= kEBins ? kEBins - 1 : b);
}
// Smallest e of bin b (bin 0 also holds everything below 2^-32).
__device__ __forceinline__ float ebin_low(int b) {
  return b == 0 ? 0.0f : __uint_as_float(static_cast<uint32_t>(b + (95 << 6)) << 17);
}

__host__ __device__ size_t full_smem_fixed(int V, int hcap) {
  (void)V;
  return sizeof(int32_t) * static_cast<size_t>(hcap) +
         sizeof(uint32_t) * (kFullThreads / 32) * 256 + sizeof(uint32_t) * 256 * 2 +
         sizeof(uint32_t) * kEBins + sizeof(float) * kSeqHead;
}

size_t full_smem_bytes(int V, int hcap) {
  // the fixed part, then as much room for in-smem sorts as fits with
  // kFullCtasPerSm CTAs on an SM (each also holds ~1 KB static and the
  // 1 KB the hardware reserves per CTA)
  const size_t fixed = (full_smem_fixed(V, hcap) + 15) / 16 * 16;
  int dev = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  size_t cap = static_cast<size_t>(per_sm) / kFullCtasPerSm - 4096;
  cap = cap / 16 * 16;
  const size_t mx = static_cast<size_t>(max_dynamic_smem());
  if (cap > mx) cap = mx;
  return fixed < cap ? cap : fixed;
}

// Stable LSD radix sort of (key, value) u32 pairs ascending by key, by one
// block, in shared or global memory (generic pointers).  Each warp owns a
// contiguous segment; within a segment elements keep their order, so equal
// keys keep input order.  Digits on which every key agrees are skipped.
// Returns true when the result is in (k1, v1).
template <int NT>
__device__ __noinline__ bool block_radix_sort(uint32_t *k0, uint32_t *v0, uint32_t *k1,
                                 uint32_t *v1, int n, uint32_t *whist,
                                 uint32_t *tot, int *s_flag, int shift0) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = (n + NW - 1) / NW;
  const int s0 = min(n, warp * seg), s1 = min(n, s0 + seg);
  bool in1 = false;
  for (int shift = shift0; shift < 32; shift += 8) {
    uint32_t *ki = in1 ? k1 : k0, *vi = in1 ? v1 : v0;
    uint32_t *ko = in1 ? k0 : k1, *vo = in1 ? v0 : v1;
    for (int i = tid; i < NW * 256; i += NT) whist[i] = 0u;
    __syncthreads();
    for (int j0 = s0; j0 < s1; j0 += 32 * 8) {
      uint32_t kk[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int j = j0 + u * 32 + lane;
        kk[u] = j < s1 ? ki[j] : 0u;
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (j0 + u * 32 + lane < s1) atomicAdd(&whist[warp * 256 + ((kk[u] >> shift) & 255u)], 1u);
    }
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
    // the warp's segment in order, 4 x 32 entries a round: the round's
    // loads first (in flight together), then its 4 groups of 32 in order
    constexpr int RU = 8;
    for (int j0 = s0; j0 < s1; j0 += 32 * RU) {
      uint32_t key[RU], val[RU];
#pragma unroll
      for (int u = 0; u < RU; u++) {
        const int j = j0 + u * 32 + lane;
        key[u] = j < s1 ? ki[j] : 0u;
        val[u] = j < s1 ? vi[j] : 0u;
      }
#pragma unroll
      for (int u = 0; u < RU; u++) {
        const int j = j0 + u * 32 + lane;
        const bool act = j < s1;
        const uint32_t d = act ? ((key[u] >> shift) & 255u) : (256u + lane);
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
        if (act) {
          const uint32_t pos = whist[warp * 256 + d] + __popc(peers & lanemask_lt());
          ko[pos] = key[u];
          vo[pos] = val[u];
        }
        __syncwarp();
        if (act && lane == __ffs(peers) - 1) whist[warp * 256 + d] += __popc(peers);
        __syncwarp();
      }
    }
    __threadfence_block();
    __syncthreads();
    in1 = !in1;
  }
  return in1;
}

// Collects the entries i < V with e[i] > 0 and prob = fl(e[i] * inv) >= pmin
// as (~prob bits, i), with no block barrier per chunk: warp w scans the terms
// [w * span, (w + 1) * span) (span = collect_span(V)) in index order and
// writes its entries to ko/vo from place w * span on; seg_n[w] = their
// number.  The warps' segments in warp order are the index order.  Also
// counts each warp's keys by their low byte into whist[w * 256 + d] (the
// first radix pass's histogram).  Block-wide; e is 16-byte aligned and
// ko/vo hold V entries.  Returns the total.
template <int NT>
__host__ __device__ inline int collect_span(int V) {
  return ((V + NT / 32 - 1) / (NT / 32) + 255) / 256 * 256;
}

template <int NT>
__device__ __noinline__ int collect_segments(const float *e, int V, float inv, float pmin, uint32_t *ko,
                                             uint32_t *vo, int *seg_n, uint32_t *whist) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < NW * 256; i += NT) whist[i] = 0u;
  __syncthreads();
  const int span = collect_span<NT>(V);
  const int a = min(V, warp * span), b = min(V, a + span);
  uint32_t *wh = whist + warp * 256;
  int cnt = 0;
  float x[8], xn[8], xm[8];
  auto fetch = [&](int j, float(&d)[8]) {
    if (j + 8 <= b) {
      const float4 p = *reinterpret_cast<const float4 *>(e + j);
      const float4 q = *reinterpret_cast<const float4 *>(e + j + 4);
      d[0] = p.x; d[1] = p.y; d[2] = p.z; d[3] = p.w;
      d[4] = q.x; d[5] = q.y; d[6] = q.z; d[7] = q.w;
    } else {
#pragma unroll
      for (int u = 0; u < 8; u++) d[u] = j + u < b ? e[j + u] : 0.0f;
    }
  };
  // two groups ahead in flight while this one is tested
  if (a < b) fetch(a + lane * 8, x);
  if (a + 256 < b) fetch(a + 256 + lane * 8, xn);
  for (int j0 = a; j0 < b; j0 += 256) {
    if (j0 + 512 < b) fetch(j0 + 512 + lane * 8, xm);
    const int i0 = j0 + lane * 8;
    uint32_t keep = 0;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      if (i0 + u < b && x[u] > 0.0f) {
        x[u] = __fmul_rn(x[u], inv);                                    // top_p.c:73-74
        if (x[u] >= pmin) keep |= 1u << u;
      }
    }
    if (!__any_sync(0xFFFFFFFFu, keep != 0u)) {  // most groups keep nothing
#pragma unroll
      for (int u = 0; u < 8; u++) {
        x[u] = xn[u];
        xn[u] = xm[u];
      }
      continue;
    }
    const int c = __popc(keep);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += t;
    }
    int pos = a + cnt + incl - c;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      if ((keep >> u) & 1u) {
        const uint32_t key = ~__float_as_uint(x[u]);
        ko[pos] = key;
        vo[pos] = static_cast<uint32_t>(i0 + u);
        atomicAdd(&wh[key & 255u], 1u);
        pos++;
      }
    }
    cnt += __shfl_sync(0xFFFFFFFFu, incl, 31);
#pragma unroll
    for (int u = 0; u < 8; u++) {
      x[u] = xn[u];
      xn[u] = xm[u];
    }
  }
  if (lane == 0) seg_n[warp] = cnt;
  __threadfence_block();
  __syncthreads();
  int tot = 0;
  for (int w = 0; w < NW; w++) tot += seg_n[w];
  return tot;
}

// The first (low-byte) pass of block_radix_sort over collect_segments'
// output: warp w's input is its segment (ks/vs from w * span, seg_n[w]
// entries), whist holds the warps' low-byte counts; the n entries go to
// ko/vo in order, stably.
template <int NT>
__device__ __noinline__ void radix_first_pass(const uint32_t *ks, const uint32_t *vs, const int *seg_n,
                                              int span, uint32_t *ko, uint32_t *vo, uint32_t *whist,
                                              uint32_t *tot) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 256) {
    uint32_t run = 0;
    for (int w = 0; w < NW; w++) {
      const uint32_t c = whist[w * 256 + tid];
      whist[w * 256 + tid] = run;
      run += c;
    }
    tot[tid] = run;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t run = 0;
    for (int d = 0; d < 256; d++) {
      const uint32_t c = tot[d];
      tot[d] = run;
      run += c;
    }
  }
  __syncthreads();
  if (tid < 256)
    for (int w = 0; w < NW; w++) whist[w * 256 + tid] += tot[tid];
  __syncthreads();
  const int s0 = warp * span, s1 = s0 + seg_n[warp];
  constexpr int RU = 8;
  for (int j0 = s0; j0 < s1; j0 += 32 * RU) {
    uint32_t key[RU], val[RU];
#pragma unroll
    for (int u = 0; u < RU; u++) {
      const int j = j0 + u * 32 + lane;
      key[u] = j < s1 ? ks[j] : 0u;
      val[u] = j < s1 ? vs[j] : 0u;
    }
#pragma unroll
    for (int u = 0; u < RU; u++) {
      const int j = j0 + u * 32 + lane;
      const bool act = j < s1;
      const uint32_t d = act ? (key[u] & 255u) : (256u + lane);
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      if (act) {
        const uint32_t pos = whist[warp * 256 + d] + __popc(peers & lanemask_lt());
        ko[pos] = key[u];
        vo[pos] = val[u];
      }
      __syncwarp();
      if (act && lane == __ffs(peers) - 1) whist[warp * 256 + d] += __popc(peers);
      __syncwarp();
    }
  }
  __threadfence_block();
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kFullThreads, kFullCtasPerSm) full_kernel(const FullArgs A) {
  constexpr int NT = kFullThreads;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ SeqShared ssh;
  __shared__ int s_seg[NT / 32];
  __shared__ int s_nh, s_flag, s_pbin;
  __shared__ float s_pmin;
  const int tid = threadIdx.x;
  int32_t *hl = reinterpret_cast<int32_t *>(smem);
  uint32_t *whist = reinterpret_cast<uint32_t *>(hl + A.hcap);
  uint32_t *tot = whist + (NT / 32) * 256;
  uint32_t *bins = tot + 256 * 2;
  float *head = reinterpret_cast<float *>(bins + kEBins);
  // in-smem sort room: two (key, value) buffers of sm_cap entries
  const size_t fixed = (full_smem_fixed(A.V, A.hcap) + 15) / 16 * 16;
  uint32_t *sm_k0 = reinterpret_cast<uint32_t *>(smem + fixed);
  const int sm_cap = A.smem_sort_cap;
  uint32_t *sm_v0 = sm_k0 + sm_cap, *sm_k1 = sm_v0 + sm_cap, *sm_v1 = sm_k1 + sm_cap;
  // global scratch of this CTA: e values, then two (key, value) buffers
  float *E = A.escr + static_cast<size_t>(blockIdx.x) * A.e_stride;
  uint32_t *g_k0 = A.sort_a + static_cast<size_t>(blockIdx.x) * A.sort_stride;
  uint32_t *g_v0 = g_k0 + A.sort_stride / 2;
  uint32_t *g_k1 = A.sort_b + static_cast<size_t>(blockIdx.x) * A.sort_stride;
  uint32_t *g_v1 = g_k1 + A.sort_stride / 2;
  // rows by cost class, claimed heaviest class first (an atomic counter:
  // a CTA takes the next row when it is done with one, so long rows do not
  // pile up on a few CTAs)
  int cls_n[kFullClasses];
  int n_full = 0;
#pragma unroll
  for (int c = 0; c < kFullClasses; c++) {
    cls_n[c] = A.n_full[c];
    n_full += cls_n[c];
  }
  __shared__ int s_w;
  // the sort room is free until the nucleus is collected: the row's tile
  // sums (from pass 1a) and the exact replay's tile workspace go there
  static_assert(kSeqHead % kSeqTile == 0 && kSeqHead / kSeqTile <= 8, "head tiles");
  const int n_rtiles = (A.V + kSeqTile - 1) / kSeqTile;
  const size_t rt_bytes = (static_cast<size_t>(n_rtiles) * 4 + 15) / 16 * 16;
  const bool row_tsum = rt_bytes + 16 * kSeqMinTiles <= static_cast<size_t>(sm_cap) * 16;
  float *tsum_row = reinterpret_cast<float *>(sm_k0);
  const SeqTiles tw1 =
      row_tsum ? seq_tiles_at(smem + fixed + rt_bytes, static_cast<size_t>(sm_cap) * 16 - rt_bytes)
               : seq_tiles_at(sm_k0, static_cast<size_t>(sm_cap) * 16);

  for (;;) {
    if (tid == 0) s_w = atomicAdd(A.n_full + kFullClasses, 1);
    __syncthreads();
    const int w = s_w;
    if (w >= n_full) break;
    int cls = kFullClasses - 1, pos = w;
    while (pos >= cls_n[cls]) {
      pos -= cls_n[cls];
      cls--;
    }
    const int row = A.full_rows[cls * A.full_stride + pos];
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
    for (int i = tid; i < kEBins; i += NT) bins[i] = 0u;
    if (row_tsum)
      for (int i = tid; i < n_rtiles; i += NT) tsum_row[i] = 0.0f;
    __syncthreads();
    int nh = 0;
    if (hist_on) {
      for (int j = tid; j < H; j += NT) {
        const int t = hrow[j];
        if (t >= 0 && t < V) hl[atomicAdd(&s_nh, 1)] = t;
      }
      __syncthreads();
      nh = s_nh;
      int np2 = 1;
      while (np2 < nh) np2 <<= 1;
      for (int i = nh + tid; i < np2; i += NT) hl[i] = INT_MAX;
      block_sort_asc_i32<NT>(hl, np2);
    }
    const float mx = key_val(A.row_best[row]);
    unsigned long long rs = A.rng[row];
    const bool topp = P.mode != kModeSoftmaxFull;
    const float thr = __fsub_rn(mx, 20.0f);                             // top_p.c:53
    // pass 1a: e values (stored) and the bins, the row read with 16-byte
    // loads, no barriers; with row_tsum, also each 256-term tile's sum of e
    // values (float, in any order: the exact replay only uses it to predict
    // the running sum's binade).  History ids are taken unpenalised here and
    // corrected in pass 1a' (a few thousand ids against ~10^5 values: the
    // main pass carries no lookup).
    {
      // e_i (0 where the max-20 filter drops the value); cnt: counted in the bins
      auto elem = [&](int i, float x, bool &cnt) -> float {
        (void)i;
        const float v = temper(x, P);
        cnt = false;
        if (!topp || v >= thr) {                                         // top_p.c:58
          cnt = topp;
          return cr_expf(__fsub_rn(v, mx));                              // :59, softmax.c:13
        }
        return 0.0f;
      };
      auto elem_store = [&](int i, float x) -> float {
        bool cnt;
        const float e = elem(i, x, cnt);
        if (cnt) atomicAdd(&bins[ebin(e)], 1u);
        E[i] = e;
        return e;
      };
      constexpr int VEC = Vec16<T>::N;
      const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp);
      int lead = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
      if (lead > V) lead = V;
      const int nvec = (V - lead) / VEC;
      const int body_end = lead + nvec * VEC;
      for (int i = tid; i < lead; i += NT) {
        const float e = elem_store(i, load_scalar<T>(rowp, i));
        if (row_tsum) atomicAdd(&tsum_row[i >> 8], e);
      }
      for (int i = body_end + tid; i < V; i += NT) {
        const float e = elem_store(i, load_scalar<T>(rowp, i));
        if (row_tsum) atomicAdd(&tsum_row[i >> 8], e);
      }
      const bool vst = (lead & 3) == 0;  // E + lead + 4m is 16-byte aligned
      const T *body = rowp + lead;
      const int lane = tid & 31;
      // U consecutive vectors per lane per trip: a warp's trip covers one
      // 256-term tile (U = 1 for bf16, 2 for f32)
      constexpr int U = 256 / (32 * VEC) > 0 ? 256 / (32 * VEC) : 1;
      constexpr int SPAN = U * VEC;
      const int nunit = (nvec + U - 1) / U;
      constexpr int UNR = U == 1 ? 2 : 1;  // two vectors in flight per lane
#pragma unroll UNR
      for (int q0 = tid - lane; q0 < nunit; q0 += NT) {  // warp-uniform trips
        const int qu = q0 + lane;
        const int i0 = lead + qu * SPAN;
        float vs = 0.0f;
#pragma unroll
        for (int u = 0; u < U; u++) {
          const int q = qu * U + u;
          if (q < nvec) {
            float xv[VEC];
            Vec16<T>::load(body, q, xv);
            const int iv = i0 + u * VEC;
#pragma unroll
            for (int w = 0; w < VEC; w++) {
              bool cnt;
              xv[w] = elem(iv + w, xv[w], cnt);
              if (cnt) atomicAdd(&bins[ebin(xv[w])], 1u);
              vs += xv[w];
            }
            if (vst) {
#pragma unroll
              for (int w = 0; w < VEC; w += 4)
                *reinterpret_cast<float4 *>(E + iv + w) = make_float4(xv[w], xv[w + 1], xv[w + 2], xv[w + 3]);
            } else {
#pragma unroll
              for (int w = 0; w < VEC; w++) E[iv + w] = xv[w];
            }
          }
        }
        if (row_tsum) {
          // the warp's vectors in one tile: one add per warp
          const int t0w = __shfl_sync(0xFFFFFFFFu, i0, 0) >> 8;
          const bool one = qu >= nunit || ((i0 >> 8) == t0w && ((i0 + SPAN - 1) >> 8) == t0w);
          if (__all_sync(0xFFFFFFFFu, one)) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) vs += __shfl_xor_sync(0xFFFFFFFFu, vs, o);
            if (lane == 0) atomicAdd(&tsum_row[t0w], vs);
          } else if (qu < nunit) {
            const int iend = min(i0 + SPAN, body_end);
            if ((i0 >> 8) == ((iend - 1) >> 8)) {
              atomicAdd(&tsum_row[i0 >> 8], vs);
            } else {
              for (int i = i0; i < iend; i++) atomicAdd(&tsum_row[i >> 8], E[i]);
            }
          }
        }
      }
    }
    __syncthreads();
    // pass 1a': each distinct history id's e value with its penalty
    // (penalize, with the id's count in the history), replacing the
    // unpenalised one: the bins and the tile sums move with it
    if (hist_on) {
      auto e_of = [&](float x, bool &cnt) -> float {
        const float v = temper(x, P);
        cnt = topp && v >= thr;
        return (!topp || v >= thr) ? cr_expf(__fsub_rn(v, mx)) : 0.0f;  // top_p.c:58-59
      };
      for (int j = tid; j < nh; j += NT) {
        const int t = hl[j];
        if (j > 0 && hl[j - 1] == t) continue;  // the id's first place only
        int c = 1;
        while (j + c < nh && hl[j + c] == t) c++;
        const float x = load_scalar<T>(rowp, t);
        bool c0, c1;
        const float e0 = e_of(x, c0);
        const float e1 = e_of(penalize(x, c, P), c1);
        E[t] = e1;
        if (c0) atomicSub(&bins[ebin(e0)], 1u);
        if (c1) atomicAdd(&bins[ebin(e1)], 1u);
        if (row_tsum) atomicAdd(&tsum_row[t >> 8], e1 - e0);
      }
      __syncthreads();
    }
    // pass 1b: the exact normaliser over the stored e values
    const SeqResult s1 = seq_scan<NT>(V, SeqSrcF32{E, 0.0f, false}, kSeqNone, 0.0f, ssh, head,
                                      kSeqHead, tw1, 0, row_tsum ? tsum_row : nullptr, 1.0f);
    const float inv = __fdiv_rn(1.0f, s1.s);                            // :72, softmax.c:18
    int tok;
    if (!topp) {
      // generate.c:159-167: r = rng_float(), first i with r < cdf
      const float r = rng_next(rs);
      const SeqResult s2 =
          seq_scan<NT>(V, SeqSrcF32{E, inv, true}, kSeqGT, r, ssh, head, kSeqHead, tw1, 0,
                       row_tsum ? tsum_row : nullptr, inv);
      tok = s2.hit >= 0 ? s2.hit : V - 1;
    } else {
      // the probability bound: bins from the top until a lower bound of the
      // float cumulative over them clears top_p (with margin)
      // (every thread a run of kEBins / NT bins from the top, a block scan of
      // the counts and masses above it; the highest bin whose bound clears
      // the target wins)
      {
        static_assert(kEBins % NT == 0, "bins per thread");
        constexpr int BPT = kEBins / NT;
        const double want = static_cast<double>(P.p) + 1e-3;
        const double dinv = static_cast<double>(inv);
        const int btop = kEBins - 1 - tid * BPT;  // this thread's bins: btop down to btop - BPT + 1
        double c_run = 0.0, m_run = 0.0;
#pragma unroll
        for (int j = 0; j < BPT; j++) {
          const int b = btop - j;
          if (b > 0) {
            const double c = static_cast<double>(bins[b]);
            c_run += c;
            m_run += c * static_cast<double>(ebin_low(b)) * dinv;
          }
        }
        if (tid == 0) s_pbin = -1;
        double cnt = seq_block_exscan_d<NT>(c_run, ssh);
        double mass = seq_block_exscan_d<NT>(m_run, ssh);
        if (want < 0.999) {
          for (int j = 0; j < BPT; j++) {
            const int b = btop - j;
            if (b <= 0) break;
            const uint32_t c = bins[b];
            if (c == 0u) continue;
            cnt += c;
            mass += static_cast<double>(c) * static_cast<double>(ebin_low(b)) * dinv;
            const double bound = mass * (1.0 - 5.97e-8) * (1.0 - (cnt + 1.0) * 5.97e-8);
            if (bound >= want) {
              atomicMax(&s_pbin, b);
              break;
            }
          }
        }
        __syncthreads();
        if (tid == 0) s_pmin = s_pbin > 0 ? __fmul_rn(ebin_low(s_pbin), inv) : 0.0f;
      }
      __syncthreads();
      float pmin = s_pmin;
      int cutoff = 0, pos = 0, nf = 0;
      const uint32_t *ks = nullptr, *vs = nullptr;
      for (int attempt = 0; attempt < 2; attempt++) {
        // the nucleus candidates, each warp's in its own segment of g_k0/g_v0
        // (index order), then the stable radix sort: its first pass gathers
        // the segments
        nf = collect_segments<NT>(E, V, inv, pmin, g_k0, g_v0, s_seg, whist);
        const int span = collect_span<NT>(V);
        bool in1;
        if (nf <= sm_cap) {
          radix_first_pass<NT>(g_k0, g_v0, s_seg, span, sm_k0, sm_v0, whist, tot);
          in1 = block_radix_sort<NT>(sm_k0, sm_v0, sm_k1, sm_v1, nf, whist, tot, &s_flag, 8);
          ks = in1 ? sm_k1 : sm_k0;
          vs = in1 ? sm_v1 : sm_v0;
        } else {
          radix_first_pass<NT>(g_k0, g_v0, s_seg, span, g_k1, g_v1, whist, tot);
          in1 = block_radix_sort<NT>(g_k1, g_v1, g_k0, g_v0, nf, whist, tot, &s_flag, 8);
          ks = in1 ? g_k0 : g_k1;
          vs = in1 ? g_v0 : g_v1;
        }
        // cumulative to the cutoff (:80-88) and the truncated sum (:91-93)
        // tile workspace: the sort room's pair that does not hold the result
        const SeqTiles tw3 =
            nf <= sm_cap ? seq_tiles_at(in1 ? sm_k0 : sm_k1, static_cast<size_t>(sm_cap) * 8)
                         : seq_tiles_at(sm_k0, static_cast<size_t>(sm_cap) * 16);
        const SeqResult s3 =
            seq_scan<NT>(nf, SeqSrcKey{ks}, kSeqGE, P.p, ssh, head, kSeqHead, tw3, 0, nullptr, 1.0f);
        if (s3.hit < 0 && pmin > 0.0f) {  // not inside the prefix: take every entry
          pmin = 0.0f;
          continue;
        }
        cutoff = s3.hit >= 0 ? s3.hit + 1 : nf;
        const float r = __fmul_rn(rng_next(rs), s3.s);                  // :96
        // the same terms as s3 from term 0: its head and tile maps are reused
        const SeqResult s4 =
            seq_scan<NT>(cutoff, SeqSrcKey{ks}, kSeqGT, r, ssh, head, kSeqHead, tw3, nf, nullptr, 1.0f);
        pos = s4.hit >= 0 ? s4.hit : 0;                                 // :98-105
        break;
      }
      tok = nf > 0 ? static_cast<int>(vs[pos]) : key_idx(A.row_best[row]);
    }
    if (tid == 0) {
      A.out[row] = tok;
      A.rng[row] = rs;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// merge_kernel: vocab-sharded rows after the allgather, one warp per row.
// The G gathered lists of a row (each sorted, at most kcap keys, distinct
// keys across ranks) are merged into the exact global top-k (the k-th
// largest key by a warp radix select, then the keys at or above it, ranked),
// and the row is decided as in slice_kernel (top_p.c:37-105 or
// top_k.c:50-72 over the list, argmax for greedy rows).
// ---------------------------------------------------------------------------
size_t merge_warp_bytes(int kcap, int G) {
  const size_t b = sizeof(unsigned long long) * static_cast<size_t>(G) * static_cast<size_t>(kcap) +
                   12 * static_cast<size_t>(kcap) + 16;
  return (b + 15) / 16 * 16;
}

int merge_rows_per_block(int kcap, int G) {
  const size_t per = merge_warp_bytes(kcap, G);
  const size_t budget = static_cast<size_t>(max_dynamic_smem());
  int r = static_cast<int>(budget / per);
  return r < 1 ? 1 : (r > kSliceWarps ? kSliceWarps : r);
}

__global__ void __launch_bounds__(kSliceThreads) merge_kernel(const MergeArgs A, int rows_per_block,
                                                              int warp_bytes) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * rows_per_block + warp;
  if (warp >= rows_per_block || row >= A.B) return;  // whole warps; no block barrier below
  unsigned char *ws = smem + static_cast<size_t>(warp) * warp_bytes;
  unsigned long long *lst = reinterpret_cast<unsigned long long *>(ws);
  float *fe = reinterpret_cast<float *>(lst + static_cast<size_t>(A.G) * A.kcap);
  float *fp = fe + A.kcap;
  int *ford = reinterpret_cast<int *>(fp + A.kcap);
  int *s_tok = ford + A.kcap;
  const RowPlan P = plan_row(A.cfg[row], A.V_global);
  const bool k_fits = P.keff <= A.kcap && P.keff <= A.kmax;
  const bool topk = P.mode == kModeTopK;
  const int k_sel = (topk && k_fits) ? P.keff : 1;
  const unsigned long long tau0 = topk ? key_topk_floor() : 0ull;
  const size_t stride = static_cast<size_t>(A.kcap) + 1;
  auto gslot = [&](int g) -> const unsigned long long * {
    return A.gathered + (static_cast<size_t>(g) * A.B + row) * stride;
  };
  // each rank's count and flags (slot kcap): count | x0nan<<30 | too_long<<29 | bad_k<<28 | timeout<<27
  int flags = 0;
  for (int g = lane; g < A.G; g += 32) flags |= static_cast<int>(gslot(g)[A.kcap]) & (15 << 27);
  flags = __reduce_or_sync(0xFFFFFFFFu, flags);
  int n_sel = 0;
  unsigned long long gbest = 0ull;
  if (topk && k_sel > 1) {
    int n = 0;
    for (int g = 0; g < A.G; g++) {
      const unsigned long long *src = gslot(g);
      const int c = min(static_cast<int>(src[A.kcap]) & ((1 << 27) - 1), A.kcap);
      for (int i = lane; i < c; i += 32) lst[n + i] = src[i];
      n += c;
    }
    __syncwarp();
    if (n > k_sel) {
      const unsigned long long kth = warp_kth(lst, n, k_sel);
      n = warp_compact_ge(lst, n, kth);
    }
    n_sel = n;
    if (A.kcap <= 64) {
      warp_rank_sort_desc(lst, n_sel);
      for (int i = n_sel + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      __syncwarp();
    } else {
      for (int i = n_sel + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      warp_sort_desc(lst, A.kcap);
    }
  } else {
    unsigned long long bl = 0ull;
    for (int g = lane; g < A.G; g += 32) {
      const unsigned long long *src = gslot(g);
      if ((static_cast<int>(src[A.kcap]) & ((1 << 27) - 1)) > 0) bl = src[0] > bl ? src[0] : bl;
    }
    gbest = warp_max_u64(bl);
    if (topk) {  // k_eff == 1: the single best admitted key
      n_sel = gbest > tau0 ? 1 : 0;
      if (lane == 0) lst[0] = gbest;
      for (int i = 1 + lane; i < A.kcap; i += 32) lst[i] = 0ull;
      __syncwarp();
    }
  }
  const bool x0nan = (flags >> 30) & 1;
  const bool too_long = (flags >> 29) & 1;
  const bool bad_k = ((flags >> 28) & 1) || (topk && !k_fits);
  const bool timed_out = (flags >> 27) & 1;
  unsigned long long rs = A.rng[row];
  int tok = -1;
  int status = too_long ? PZ_ROW_HISTORY_TOO_LONG : PZ_ROW_OK;
  const bool want_cand = A.cand_ids != nullptr || A.cand_probs != nullptr;
  int32_t *cids = A.cand_ids ? A.cand_ids + static_cast<size_t>(row) * A.cand_stride : nullptr;
  float *cprobs = A.cand_probs ? A.cand_probs + static_cast<size_t>(row) * A.cand_stride : nullptr;
  bool listed = false;
  if (timed_out) {
    status = PZ_ROW_TIMEOUT;
  } else if (too_long) {
    tok = -1;
  } else if (bad_k) {
    status = PZ_ROW_HINT_VIOLATED;
  } else if (P.mode == kModeGreedy) {
    tok = x0nan ? 0 : (gbest ? key_idx(gbest) : 0);
  } else if (topk) {
    int t = INT_MIN;
    if (P.keff <= 64) {
      t = warp_sample_small(lst, n_sel, P, rs, fe, fp, want_cand ? cprobs : nullptr);
      if (t != INT_MIN && cids != nullptr)
        for (int i = lane; i < P.keff; i += 32) cids[i] = i < n_sel ? key_idx(lst[i]) : -1;
    }
    if (t == INT_MIN)
      t = sample_list<32>(lst, n_sel, P, rs, fe, fp, ford, s_tok, want_cand ? cids : nullptr,
                          want_cand ? cprobs : nullptr);
    tok = t;
    listed = true;
  } else {
    status = PZ_ROW_HINT_VIOLATED;
  }
  if (lane == 0) {
    A.out[row] = tok;
    A.rng[row] = rs;
    if (A.n_cand) A.n_cand[row] = listed ? P.keff : 0;
    if (A.row_status) A.row_status[row] = status;
  }
  if (want_cand && !listed) {
    for (int i = lane; i < A.cand_stride; i += 32) {
      if (cids) cids[i] = -1;
      if (cprobs) cprobs[i] = 0.0f;
    }
  }
}

// ---------------------------------------------------------------------------
// logprob_kernel: OpenAI-style log-probabilities from the same row (no
// counterpart in the reference, whose loop returns ids only).  The
// distribution is the one the sampler draws from before any truncation:
// softmax over the whole row of the penalised, tempered values (greedy rows:
// of the penalised values).  One CTA per row: the row read once with 16-byte
// loads, an online log-sum-exp per thread (running maximum, rescaled sum),
// combined in double; then v_token - LSE and v_entry - LSE for the row's
// list.  fp32 exps, so the outputs are accurate to ~1e-5 (not bit-exact
// with anything: the reference has no such output).
// ---------------------------------------------------------------------------
size_t logprob_smem_bytes(int V, int hcap) {
  return sizeof(uint32_t) * (static_cast<size_t>(V) / 32 + 2) + sizeof(int32_t) * static_cast<size_t>(hcap);
}

template <typename T>
__global__ void __launch_bounds__(kSliceThreads) logprob_kernel(const LogprobArgs A) {
  constexpr int NT = kSliceThreads;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ double s_m[NT / 32], s_s[NT / 32];
  __shared__ int s_nh;
  __shared__ float s_lse;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = A.V;
  const int bm_words = V / 32 + 2;
  uint32_t *bitmap = reinterpret_cast<uint32_t *>(smem);
  int32_t *hl = reinterpret_cast<int32_t *>(bitmap + bm_words);
  const RowPlan P = plan_row(A.cfg[row], V);
  const bool greedy = P.mode == kModeGreedy;
  const T *rowp = static_cast<const T *>(A.logits) + static_cast<size_t>(row) * static_cast<size_t>(A.ld);
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
  auto value = [&](int i, float x) -> float {  // the drawn-from value of column i
    if (hist_on && ((bitmap[i >> 5] >> (i & 31)) & 1u)) x = penalize(x, sorted_count(hl, nh, i), P);
    return greedy ? x : temper(x, P);
  };
  float m = -INFINITY, sum = 0.0f;
  auto add = [&](float v) {
    if (!(v > -INFINITY)) return;  // -inf adds nothing; NaN is left out
    if (v > m) {
      sum = sum * expf(m - v) + 1.0f;
      m = v;
    } else {
      sum += expf(v - m);
    }
  };
  constexpr int VEC = Vec16<T>::N;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp);
  int lead = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
  if (lead > V) lead = V;
  const int nvec = (V - lead) / VEC;
  const int body_end = lead + nvec * VEC;
  for (int i = tid; i < lead; i += NT) add(value(i, load_scalar<T>(rowp, i)));
  for (int i = body_end + tid; i < V; i += NT) add(value(i, load_scalar<T>(rowp, i)));
  const T *body = rowp + lead;
  for (int q = tid; q < nvec; q += NT) {
    float xv[VEC];
    Vec16<T>::load(body, q, xv);
#pragma unroll
    for (int w = 0; w < VEC; w++) add(value(lead + q * VEC + w, xv[w]));
  }
  // combine (m, sum) pairs: warp, then block, in double
  double dm = m, ds = sum;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double om = __shfl_xor_sync(0xFFFFFFFFu, dm, o), os = __shfl_xor_sync(0xFFFFFFFFu, ds, o);
    const double nm = dm > om ? dm : om;
    ds = (nm == -INFINITY) ? 0.0 : ds * exp(dm - nm) + os * exp(om - nm);
    dm = nm;
  }
  if (lane == 0) {
    s_m[warp] = dm;
    s_s[warp] = ds;
  }
  __syncthreads();
  if (tid == 0) {
    double M = -INFINITY, S = 0.0;
    for (int w = 0; w < NT / 32; w++) {
      const double nm = M > s_m[w] ? M : s_m[w];
      S = (nm == -INFINITY) ? 0.0 : S * exp(M - nm) + s_s[w] * exp(s_m[w] - nm);
      M = nm;
    }
    s_lse = static_cast<float>(M + log(S));
  }
  __syncthreads();
  const float lse = s_lse;
  auto logp = [&](int id) -> float {
    if (id < 0 || id >= V) return -INFINITY;
    return __fsub_rn(value(id, load_scalar<T>(rowp, id)), lse);
  };
  if (A.token_logprob != nullptr && tid == 0) {
    const int tok = A.tokens[row];
    A.token_logprob[row] = tok >= 0 ? logp(tok) : __int_as_float(0x7FC00000);
  }
  if (A.cand_logprobs != nullptr) {
    const int n = A.n_cand ? A.n_cand[row] : 0;
    for (int j = tid; j < A.cand_stride; j += NT) {
      const int id = (j < n && A.cand_ids) ? A.cand_ids[static_cast<size_t>(row) * A.cand_stride + j] : -1;
      A.cand_logprobs[static_cast<size_t>(row) * A.cand_stride + j] = j < n ? logp(id) : -INFINITY;
    }
  }
}

// ---------------------------------------------------------------------------
// lm_head_kernel: the classifier of reference src/transformer/forward.c
// :102-165 (parallel_matmul_bf16: fp32 activations x bf16 weight rows ->
// fp32 logits), producing the sampler's logits buffer on the same stream.
// logits[b][v] = sum_d x[b][d] * w[v][d], the bf16 weights widened exactly,
// fp32 fused multiply-adds (its sum order is not the reference's: the LM
// head is outside the sampler's parity contract).  HBM-bound on the weights
// (V x dim x 2 bytes per launch): each warp takes one weight row at a time
// with 16-byte loads and dots it with kLmRows activation rows staged in
// shared memory.
// ---------------------------------------------------------------------------
constexpr int kLmRows = 8;   // activation rows per pass over the weights

__global__ void __launch_bounds__(kSliceThreads) lm_head_kernel(const float *x, int B, int dim,
                                                                const uint16_t *w, int V,
                                                                float *logits, int64_t ld) {
  extern __shared__ __align__(16) unsigned char smem[];
  float *xs = reinterpret_cast<float *>(smem);  // [kLmRows][dim]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = dim / 8;                     // dim % 8 == 0 (host-checked)
  for (int b0 = 0; b0 < B; b0 += kLmRows) {
    const int nb = min(kLmRows, B - b0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * dim; i += blockDim.x) xs[i] = x[static_cast<size_t>(b0) * dim + i];
    __syncthreads();
    for (int v = blockIdx.x * kSliceWarps + warp; v < V; v += gridDim.x * kSliceWarps) {
      const uint4 *wr = reinterpret_cast<const uint4 *>(w + static_cast<size_t>(v) * dim);
      float acc[kLmRows];
#pragma unroll
      for (int r = 0; r < kLmRows; r++) acc[r] = 0.0f;
      for (int q = lane; q < nvec; q += 32) {
        const uint4 u = __ldg(wr + q);
        const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
        float wf[8];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          wf[2 * j] = __uint_as_float(ww[j] << 16);
          wf[2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
        }
#pragma unroll
        for (int r = 0; r < kLmRows; r++) {
          if (r < nb) {
            const float4 a0 = reinterpret_cast<const float4 *>(xs + r * dim)[2 * q];
            const float4 a1 = reinterpret_cast<const float4 *>(xs + r * dim)[2 * q + 1];
            float t = acc[r];
            t = __fmaf_rn(a0.x, wf[0], t);
            t = __fmaf_rn(a0.y, wf[1], t);
            t = __fmaf_rn(a0.z, wf[2], t);
            t = __fmaf_rn(a0.w, wf[3], t);
            t = __fmaf_rn(a1.x, wf[4], t);
            t = __fmaf_rn(a1.y, wf[5], t);
            t = __fmaf_rn(a1.z, wf[6], t);
            t = __fmaf_rn(a1.w, wf[7], t);
            acc[r] = t;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kLmRows; r++) {
        float t = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
        if (lane == 0 && r < nb) logits[static_cast<size_t>(b0 + r) * ld + v] = t;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// small kernels
// ---------------------------------------------------------------------------
__global__ void temperature_kernel(float *x, int n, float inv) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fmul_rn(x[i], inv);   // temperature.c:11-20
}

// The generate loop's history window: each row's sampled id goes to slot
// (*counter % W) of its W-slot ring (penalties count ids, so the ring's
// order does not matter; slots never written hold -1, which the contract
// ignores).  counter_step_kernel then moves to the next slot.
__global__ void history_append_kernel(int32_t *ring, int B, int W, const int32_t *tokens,
                                      const int32_t *counter) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < B) {
    const int pos = *counter % W;
    ring[static_cast<size_t>(r) * W + pos] = tokens[r];
  }
}

__global__ void counter_step_kernel(int32_t *counter) { *counter += 1; }

// Both steps in one block when the batch fits one (one launch fewer per
// decode step): every thread reads the counter before the barrier, then
// thread 0 advances it.
__global__ void history_append_step_kernel(int32_t *ring, int B, int W, const int32_t *tokens,
                                           int32_t *counter) {
  const int r = threadIdx.x;
  const int pos = *counter % W;
  if (r < B) ring[static_cast<size_t>(r) * W + pos] = tokens[r];
  __syncthreads();
  if (r == 0) *counter += 1;
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
// Opt-in dynamic shared memory: the device's per-block maximum minus the
// largest static shared footprint of these kernels (< 4 KB).
int max_dynamic_smem() {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return optin - 4096;
}

cudaError_t set_kernel_attributes() {
  cudaError_t e;
  const int big = max_dynamic_smem();
  e = cudaFuncSetAttribute(slice_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(slice_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(slice_long_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(slice_long_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(full_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(full_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(logprob_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(logprob_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  return e;
}

cudaError_t launch_slice(const SliceArgs &a, int dtype, size_t smem, cudaStream_t st) {
  // rows [0, B1) one CTA each, then S CTAs for each later row
  const unsigned grid = static_cast<unsigned>(a.B1) + static_cast<unsigned>(a.B - a.B1) * a.S;
  if (a.kcap > kTQK) {
    if (dtype == PZ_DTYPE_F32)
      slice_long_kernel<float><<<grid, kSliceThreads, smem, st>>>(a);
    else
      slice_long_kernel<uint16_t><<<grid, kSliceThreads, smem, st>>>(a);
  } else if (dtype == PZ_DTYPE_F32) {
    slice_kernel<float><<<grid, kSliceThreads, smem, st>>>(a);
  } else {
    slice_kernel<uint16_t><<<grid, kSliceThreads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_full(const FullArgs &a, int dtype, int grid, size_t smem, cudaStream_t st) {
  if (dtype == PZ_DTYPE_F32)
    full_kernel<float><<<grid, kFullThreads, smem, st>>>(a);
  else
    full_kernel<uint16_t><<<grid, kFullThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_merge(const MergeArgs &a, cudaStream_t st) {
  const int r = merge_rows_per_block(a.kcap, a.G);
  const size_t wb = merge_warp_bytes(a.kcap, a.G);
  if (wb * static_cast<size_t>(r) > static_cast<size_t>(max_dynamic_smem())) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((a.B + r - 1) / r);
  merge_kernel<<<grid, kSliceThreads, wb * r, st>>>(a, r, static_cast<int>(wb));
  return cudaGetLastError();
}

cudaError_t launch_temperature(float *x, int n, float T, cudaStream_t st) {
  if (T < 1e-6f) T = 1e-6f;                 // temperature.c:10
  const float inv = 1.0f / T;
  temperature_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, n, inv);
  return cudaGetLastError();
}

cudaError_t launch_logprob(const LogprobArgs &a, int dtype, cudaStream_t st) {
  const size_t smem = logprob_smem_bytes(a.V, a.hcap);
  if (dtype == PZ_DTYPE_F32)
    logprob_kernel<float><<<a.B, kSliceThreads, smem, st>>>(a);
  else
    logprob_kernel<uint16_t><<<a.B, kSliceThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_lm_head(const float *x, int B, int dim, const uint16_t *w, int V, float *logits,
                           int64_t ld, int num_sms, cudaStream_t st) {
  const size_t smem = sizeof(float) * kLmRows * static_cast<size_t>(dim);
  const int grid = min(num_sms * 8, (V + kSliceWarps - 1) / kSliceWarps);
  lm_head_kernel<<<grid, kSliceThreads, smem, st>>>(x, B, dim, w, V, logits, ld);
  return cudaGetLastError();
}

cudaError_t launch_history_append(int32_t *ring, int B, int W, const int32_t *tokens,
                                  int32_t *counter, cudaStream_t st) {
  if (B > 0) {
    if (B <= 1024) {
      history_append_step_kernel<<<1, (B + 31) / 32 * 32, 0, st>>>(ring, B, W, tokens, counter);
      return cudaGetLastError();
    }
    history_append_kernel<<<(B + 255) / 256, 256, 0, st>>>(ring, B, W, tokens, counter);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  counter_step_kernel<<<1, 1, 0, st>>>(counter);
  return cudaGetLastError();
}

cudaError_t launch_rng_seed(unsigned long long *s, int B, unsigned long long base,
                            const unsigned long long *seeds, cudaStream_t st) {
  rng_seed_kernel<<<(B + 255) / 256, 256, 0, st>>>(s, B, base, seeds);
  return cudaGetLastError();
}

}  // namespace pz
