// pz_seqsum.cuh — exact parallel replay of a sequential float sum.
//
// The reference accumulates softmax normalisers and CDFs one element at a
// time in float (reference src/sampling/top_p.c:57-65, :80-105;
// src/math/softmax.c:12-16; generate.c:160-167).  Its rounding error over
// 1e5 terms is ~1e-4 relative, far above the parity tolerance, so a GPU
// tree reduction cannot reproduce its decisions.  This file reproduces the
// sequential sum bit for bit, in parallel:
//
// While the running sum s stays inside one binade [2^E, 2^(E+1)), every
// representable s is an integer N times the binade's ulp u = 2^(E-23), and
// fl(s + x) = (N + round_u(x)) * u, where round_u rounds x/u to an integer
// and breaks exact halves towards an even result (so the increment for a
// half depends only on the parity of N).  An element is therefore the map
// N -> N + a[N & 1], maps of this form are closed under composition, and
// composition is associative: a block-wide scan of the maps gives every
// prefix sum exactly.  When a prefix leaves the binade, that one element is
// added with a real FADD and the scan restarts from the next element on the
// new binade's grid.  Sums of non-negative terms only grow, so a pass sees
// at most ~30 such restarts (one per doubling of the sum).
#pragma once

#include "pz_device.cuh"

namespace pz {

// Increments are kept in 32 bits, saturating at kSeqClamp: a sum that
// reaches 2^24 has left the binade (N < 2^24 inside it), so past that only
// "crossed" matters, never the exact count.
struct SeqMap {
  uint32_t e, o;  // increment of N when N is even / odd
};

__device__ __forceinline__ SeqMap seq_identity() { return SeqMap{0ull, 0ull}; }

constexpr uint32_t kSeqClamp = 1u << 30;

// f applied first, then g.
__device__ __forceinline__ SeqMap seq_compose(SeqMap f, SeqMap g) {
  SeqMap h;
  h.e = min(f.e + ((f.e & 1u) ? g.o : g.e), kSeqClamp);
  h.o = min(f.o + ((f.o & 1u) ? g.e : g.o), kSeqClamp);
  return h;
}

// N < 2^24 + 2 * kSeqClamp (an applied prefix, then one more element):
// the result stays below 2^32.
__device__ __forceinline__ uint32_t seq_apply(SeqMap f, uint32_t N) {
  return N + ((N & 1u) ? f.o : f.e);
}

// Grid exponent eu (u = 2^eu) of the binade holding s >= 0.  Zero,
// subnormals and [2^-126, 2^-125) share the grid 2^-149.
__device__ __forceinline__ int seq_grid_exp(float s) {
  const int ex = (__float_as_uint(s) >> 23) & 0xFF;
  return (ex == 0 ? 1 : ex) - 150;
}
// s = N * 2^eu, with N < 2^24.
__device__ __forceinline__ uint32_t seq_N(float s) {
  const uint32_t b = __float_as_uint(s);
  const int ex = (b >> 23) & 0xFF;
  const uint32_t m = b & 0x7FFFFFu;
  return ex == 0 ? m : (m | 0x800000u);
}
__device__ __forceinline__ float seq_float(uint32_t N, int eu) {
  return __uint_as_float(static_cast<uint32_t>((eu + 149) << 23) +
                         static_cast<uint32_t>(N));
}

constexpr uint32_t kSeqLimit = 1u << 24;

// The map of adding x >= 0 on grid 2^eu.
__device__ __forceinline__ SeqMap seq_elem(float x, int eu) {
  const uint32_t b = __float_as_uint(x);
  const int ex = (b >> 23) & 0xFF;
  uint32_t M = b & 0x7FFFFFu;
  int E2;
  if (ex == 0) {
    E2 = -149;
  } else {
    M |= 0x800000u;
    E2 = ex - 150;
  }
  uint32_t m = 0;
  bool tie = false;
  if (M != 0) {
    const int sh = E2 - eu;
    if (sh >= 0) {
      // M < 2^24: shifts up to 6 stay below 2^30
      m = sh >= 7 ? kSeqClamp : min(M << sh, kSeqClamp);
    } else {
      const int q = -sh;
      if (q < 26) {
        m = M >> q;
        const uint32_t rem = M & ((1u << q) - 1u);
        const uint32_t half = 1u << (q - 1);
        if (rem > half)
          m++;
        else if (rem == half)
          tie = true;
      }
    }
  }
  SeqMap f{m, m};
  if (tie) {
    if (m & 1u)
      f.e = m + 1;
    else
      f.o = m + 1;
  }
  return f;
}

// The map of adding x >= 0 on grid 2^eu for a normal running sum
// (-126 <= eu), in float arithmetic, with sc = 2^-eu:
//   y = x * sc is exact (a power-of-two scaling; a product below 2^-126 may
//     round, but it is then far below 1/2 and adds nothing);
//   rint(y) (ties to even) is read off y + 2^23, exact for 0 <= y < 2^23;
//   d = rint(y) - y is exact, and |d| = 1/2 exactly at a tie.
// The even increment rint(y) serves an even N; at a tie an odd N takes the
// other neighbour, rint(y) - 2d.  On a normal grid N >= 2^23, so y >= 2^23
// leaves the binade whatever N is: the increment is then reported as 2^24.
// Agrees with seq_elem wherever seq_elem's increment is below 2^23.
__device__ __forceinline__ SeqMap seq_elem_fast(float x, float sc, bool &tie) {
  const float y = __fmul_rn(x, sc);
  const float r = __fadd_rn(y, 8388608.0f);
  uint32_t m = __float_as_uint(r) - 0x4B000000u;
  const float d = __fsub_rn(__fsub_rn(r, 8388608.0f), y);
  tie = fabsf(d) == 0.5f;
  if (!(y < 8388608.0f)) {  // also NaN and inf terms
    m = kSeqLimit;
    tie = false;
  }
  SeqMap f{m, m};
  if (tie) f.o = d < 0.0f ? m + 1u : m - 1u;
  return f;
}

// 2^-eu as a float, for -126 <= eu <= 127.
__device__ __forceinline__ float seq_scale(int eu) {
  return __uint_as_float(static_cast<uint32_t>(127 - eu) << 23);
}

enum SeqTarget : int { kSeqNone = 0, kSeqGE = 1, kSeqGT = 2 };

__device__ __forceinline__ bool seq_meets(float s, int kind, float target) {
  return (kind == kSeqGE && s >= target) || (kind == kSeqGT && s > target);
}

// Integer form of the target on grid 2^eu: s = N * 2^eu meets it iff
// N >= the returned value (0xFFFFFFFF: never on this grid).
__device__ __forceinline__ uint32_t seq_thr(int kind, float target, int eu) {
  if (kind == kSeqNone) return 0xFFFFFFFFu;
  const double q = static_cast<double>(target) *
                   __longlong_as_double(static_cast<long long>(1023 - eu) << 52);
  if (q != q) return 0xFFFFFFFFu;
  if (kind == kSeqGE) {  // N >= q  <=>  N >= ceil(q)
    const double c = ceil(q);
    return c <= 0.0 ? 0u : (c >= 4294967295.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(c));
  }
  const double f = floor(q);  // N > q  <=>  N >= floor(q) + 1
  return f < 0.0 ? 0u : (f >= 4294967294.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(f) + 1u);
}

// Composite map of the warp's terms (lane l holds the 8 consecutive terms
// x[0..7] that follow lane l-1's) on grid 2^eu; every lane gets it.  On a
// normal grid a run without ties adds a constant, so the usual case is one
// integer sum; a run with a tie, or a subnormal grid, composes the maps in
// order (lane runs first, then an ordered shuffle tree).
__device__ __forceinline__ SeqMap seq_warp_map(const float (&x)[8], int eu) {
  const int lane = threadIdx.x & 31;
  if (eu >= -126) {
    const float sc = seq_scale(eu);
    uint32_t sum = 0;
    bool tie_any = false;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      bool tie;
      const SeqMap f = seq_elem_fast(x[e], sc, tie);
      sum += f.e;  // <= 8 * 2^24
      tie_any |= tie;
    }
    if (!__any_sync(0xFFFFFFFFu, tie_any)) {
      const uint32_t t = __reduce_add_sync(0xFFFFFFFFu, min(sum, kSeqLimit));  // <= 2^29
      return SeqMap{t, t};
    }
  }
  SeqMap F = seq_identity();
  if (eu >= -126) {
    const float sc = seq_scale(eu);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      bool tie;
      F = seq_compose(F, seq_elem_fast(x[e], sc, tie));
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; e++) F = seq_compose(F, seq_elem(x[e], eu));
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    SeqMap g;
    g.e = __shfl_down_sync(0xFFFFFFFFu, F.e, o);
    g.o = __shfl_down_sync(0xFFFFFFFFu, F.o, o);
    if ((lane & (2 * o - 1)) == 0) F = seq_compose(F, g);
  }
  F.e = __shfl_sync(0xFFFFFFFFu, F.e, 0);
  F.o = __shfl_sync(0xFFFFFFFFu, F.o, 0);
  return F;
}

// Exact replay, warp-wide, of the terms j in [start, j1) of the tile that
// starts at term j0 (lane l loads terms j0 + 8l .. j0 + 8l + 7), from the
// running sum s
// (uniform arguments).  Returns the sum after the last term replayed;
// hit = the first j whose sum meets the target (the replay stops there), or
// -1.  Inside a binade the maps give every prefix (an exclusive warp scan);
// the one term that leaves the binade is added with a real FADD, and the
// replay goes on from the next term on the new grid.
struct SeqResult {
  float s;   // sum of all n terms, or the prefix sum at the hit
  int hit;   // first j whose prefix meets the target, or -1
};

template <typename Src>
__device__ __noinline__ SeqResult seq_tile_exact(const Src src, int j0, int start, int j1, float s,
                                                 int kind, float target) {
  const int lane = threadIdx.x & 31;
  float x[8];
  src.load8(j0 + 8 * lane, j1, x);
  while (start < j1) {
    if (!(s <= 3.40282347e38f))  // NaN or +inf: every later sum is s
      return SeqResult{s, seq_meets(s, kind, target) ? start : -1};
    const int eu = seq_grid_exp(s);
    const uint32_t N0 = seq_N(s);
    const uint32_t thrN = seq_thr(kind, target, eu);
    // the lane's element maps on this grid (identity outside [start, j1))
    SeqMap m[8];
    const float sc = seq_scale(eu < -126 ? -126 : eu);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int j = j0 + 8 * lane + e;
      bool tie;
      m[e] = (j < start || j >= j1) ? seq_identity()
             : (eu >= -126 ? seq_elem_fast(x[e], sc, tie) : seq_elem(x[e], eu));
    }
    SeqMap incl = m[0];
#pragma unroll
    for (int e = 1; e < 8; e++) incl = seq_compose(incl, m[e]);
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
    uint32_t N = seq_apply(ex, N0);
    int ev = 0x7FFFFFFF;
    bool cross = false;
    uint32_t Nev = 0;
    float xev = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int j = j0 + 8 * lane + e;
      if (j >= start && j < j1 && ev == 0x7FFFFFFF) {
        const uint32_t Nn = seq_apply(m[e], N);
        if (Nn >= kSeqLimit) {
          ev = j;
          cross = true;
          Nev = N;
          xev = x[e];
        } else if (Nn >= thrN) {
          ev = j;
          Nev = Nn;
        }
        N = Nn;
      }
    }
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, ev != 0x7FFFFFFF);
    if (bal == 0u) {
      SeqMap tot;
      tot.e = __shfl_sync(0xFFFFFFFFu, incl.e, 31);
      tot.o = __shfl_sync(0xFFFFFFFFu, incl.o, 31);
      return SeqResult{seq_float(seq_apply(tot, N0), eu), -1};
    }
    const int src = __ffs(bal) - 1;  // lanes hold consecutive runs: the lowest lane is first
    ev = __shfl_sync(0xFFFFFFFFu, ev, src);
    cross = __shfl_sync(0xFFFFFFFFu, cross, src);
    Nev = __shfl_sync(0xFFFFFFFFu, Nev, src);
    xev = __shfl_sync(0xFFFFFFFFu, xev, src);
    if (!cross) return SeqResult{seq_float(Nev, eu), ev};
    s = __fadd_rn(seq_float(Nev, eu), xev);
    if (seq_meets(s, kind, target)) return SeqResult{s, ev};
    start = ev + 1;
  }
  return SeqResult{s, -1};
}

// Term sources for seq_scan.  at(j) is term j; load8(j, n, x) fills x with
// terms j..j+7 (0 past n), with 16-byte loads when they are aligned.
struct SeqSrcF32 {  // x_j = p[j], or fl(p[j] * scale) when scaled
  const float *p;
  float scale;
  bool scaled;
  __device__ __forceinline__ float at(int j) const {
    return scaled ? __fmul_rn(p[j], scale) : p[j];
  }
  __device__ __forceinline__ void load8(int j, int n, float (&x)[8]) const {
    if (j + 8 <= n && (reinterpret_cast<uintptr_t>(p + j) & 15u) == 0u) {
      const float4 a = *reinterpret_cast<const float4 *>(p + j);
      const float4 b = *reinterpret_cast<const float4 *>(p + j + 4);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      if (scaled) {
#pragma unroll
        for (int e = 0; e < 8; e++) x[e] = __fmul_rn(x[e], scale);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) x[e] = j + e < n ? at(j + e) : 0.0f;
    }
  }
};

struct SeqSrcKey {  // x_j = the float whose bits are ~k[j]
  const uint32_t *k;
  __device__ __forceinline__ float at(int j) const { return __uint_as_float(~k[j]); }
  __device__ __forceinline__ void load8(int j, int n, float (&x)[8]) const {
    if (j + 8 <= n && (reinterpret_cast<uintptr_t>(k + j) & 15u) == 0u) {
      const uint4 a = *reinterpret_cast<const uint4 *>(k + j);
      const uint4 b = *reinterpret_cast<const uint4 *>(k + j + 4);
      x[0] = __uint_as_float(~a.x); x[1] = __uint_as_float(~a.y);
      x[2] = __uint_as_float(~a.z); x[3] = __uint_as_float(~a.w);
      x[4] = __uint_as_float(~b.x); x[5] = __uint_as_float(~b.y);
      x[6] = __uint_as_float(~b.z); x[7] = __uint_as_float(~b.w);
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) x[e] = j + e < n ? at(j + e) : 0.0f;
    }
  }
};

constexpr int kSeqMinTiles = 16;

struct SeqShared {
  double warp_tot[32];
  float head_tsum[8];  // head tiles' sums (head_cap <= 8 tiles)
  __align__(16) unsigned char spare[kSeqMinTiles * 16];  // tile workspace when the caller has none
  float s;
  int done_pos;
};

constexpr int kSeqTile = 256;  // terms per tile: 8 per lane of a warp

// Per-tile workspace of seq_scan (shared memory, cap tiles; 16 B a tile):
// the tile's term sum, the predicted grid of the running sum at its start,
// and its composite map on that grid.
struct SeqTiles {
  float *tsum;
  int *eu;
  SeqMap *map;
  int cap;
};

__device__ __forceinline__ SeqTiles seq_tiles_at(void *base, size_t bytes) {
  SeqTiles w;
  const int cap = static_cast<int>(bytes / 16);
  w.map = reinterpret_cast<SeqMap *>(base);
  w.tsum = reinterpret_cast<float *>(w.map + cap);
  w.eu = reinterpret_cast<int *>(w.tsum + cap);
  w.cap = cap;
  return w;
}

// Exclusive block scan of doubles (NT threads).
template <int NT>
__device__ __forceinline__ double seq_block_exscan_d(double v, SeqShared &sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double w = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += w;
  }
  if (lane == 31) sh.warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double t = lane < NT / 32 ? sh.warp_tot[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double w = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += w;
    }
    if (lane < NT / 32) sh.warp_tot[lane] = t;
  }
  __syncthreads();
  const double r = (warp ? sh.warp_tot[warp - 1] : 0.0) + incl - v;
  __syncthreads();
  return r;
}

// The head: terms 0..K-1 of head_buf added in order by the calling thread;
// returns the first j whose sum meets the target, or -1 (then s is the sum
// of all K terms).  8 terms a round: the round's loads first, then the
// chain of adds (padding terms are 0: adding 0 leaves s as it is), then the
// round's prefixes tested against the target off the chain.
__device__ __forceinline__ int seq_head(const float *head_buf, int K, int kind, float target,
                                        float &s_out) {
  float s = 0.0f;
  int done = -1;
  for (int j0 = 0; j0 < K && done < 0; j0 += 8) {
    float h[8];
#pragma unroll
    for (int e = 0; e < 8; e++) h[e] = j0 + e < K ? head_buf[j0 + e] : 0.0f;
    float ps[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      s = __fadd_rn(s, h[e]);
      ps[e] = s;
    }
    if (kind != kSeqNone) {
#pragma unroll
      for (int e = 7; e >= 0; e--)
        if (j0 + e < K && seq_meets(ps[e], kind, target)) done = j0 + e;
      if (done >= 0) s = ps[done - j0];
    }
  }
  s_out = s;
  return done;
}

// Replays s = fl(s + x_j) for j = 0..n-1 (x_j >= 0) starting from s = 0.
// With a target, stops at the first j where s_j >= target (kSeqGE) or
// s_j > target (kSeqGT).  Block-wide call (NT threads, uniform arguments).
//
// The first head_cap terms (a multiple of kSeqTile; the running sum leaves
// its binade most often early on, about once per doubling of the terms
// seen) are added in order by one thread.  The rest is cut into tiles of
// 256 terms, with no barrier per tile:
//   1. tile sums (float; estimates only): computed by the warps, or given
//      by the caller (tsum_in[u] * tsum_scale for the tile of terms
//      256u .. 256u + 255, head tiles included);
//   2. a block scan of those sums predicts the running sum at each tile's
//      start, hence its grid;
//   3. every warp computes its tiles' composite maps on the predicted grids
//      (seq_warp_map) while one thread of warp 0 runs the head;
//   4. warp 0 walks the tiles in order: a tile whose predicted grid is the
//      current one costs one integer add, since N only grows and a tile
//      leaves the binade, or meets the target, iff its end does; any other
//      tile (it leaves the binade, meets the target, or was predicted on
//      another grid) is replayed exactly (seq_tile_exact).
// The float sum differs from the exact one by far less than a binade, so
// only tiles where the sum crosses a power of two miss their prediction.
// tw holds the tiles' grids and maps; when the tiles outnumber it they are
// walked in segments, each predicted from the exact sum at its start.
// With reuse_n > 0 (the n of the previous call, over the same terms from
// the same term 0, with the same head_cap and tw; reuse_n >= n), the head's
// terms and, when that call's tiles fitted tw in one segment, its maps are
// reused: steps 1-3 are skipped and only the head and the walk run, with
// this call's target.  A map is only used for a tile that lies wholly
// below n.
template <int NT, typename Src>
__device__ __noinline__ SeqResult seq_scan(int n, const Src src, int kind, float target,
                                           SeqShared &sh, float *head_buf, int head_cap,
                                           SeqTiles tw, int reuse_n, const float *tsum_in,
                                           float tsum_scale) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tw.cap < kSeqMinTiles) tw = seq_tiles_at(sh.spare, sizeof sh.spare);
  const int K = n < head_cap ? n : head_cap;
  const int Kt = K / kSeqTile;  // head tiles (all full when there are walk tiles)
  const int ntiles = (n - K + kSeqTile - 1) / kSeqTile;
  bool reuse = reuse_n > 0;
  if (reuse) {
    const int Kp = reuse_n < head_cap ? reuse_n : head_cap;
    if ((reuse_n - Kp + kSeqTile - 1) / kSeqTile > tw.cap) reuse = false;
  }
  if (ntiles == 0 || reuse) {
    if (reuse_n == 0)
      for (int j = tid; j < K; j += NT) head_buf[j] = src.at(j);
    __syncthreads();
    if (tid == 0) sh.done_pos = seq_head(head_buf, K, kind, target, sh.s);
    __syncthreads();
    if (ntiles == 0 || sh.done_pos >= 0) {
      SeqResult r{sh.s, sh.done_pos};
      __syncthreads();
      return r;
    }
  }
  for (int g0 = 0; g0 < ntiles; g0 += tw.cap) {
    const int nt = min(tw.cap, ntiles - g0);
    if (!reuse) {
      const bool first = g0 == 0;
      const int hk = first ? Kt : 0;  // head tiles summed in this segment
      // 1. tile sums; the first segment also fills head_buf
      if (tsum_in == nullptr) {
        for (int u = warp; u < hk + nt; u += NW) {
          const int j0 = u < hk ? u * kSeqTile : K + (g0 + u - hk) * kSeqTile;
          float x[8];
          src.load8(j0 + lane * 8, n, x);
          float a = 0.0f;
#pragma unroll
          for (int e = 0; e < 8; e++) a += x[e];
          if (u < hk) {
#pragma unroll
            for (int e = 0; e < 8; e++) head_buf[j0 + lane * 8 + e] = x[e];
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
          if (lane == 0) {
            if (u < hk)
              sh.head_tsum[u] = a;
            else
              tw.tsum[u - hk] = a;
          }
        }
      } else {
        if (first)
          for (int j = tid; j < K; j += NT) head_buf[j] = src.at(j);
        for (int u = tid; u < hk + nt; u += NT) {
          const float a = __fmul_rn(tsum_in[u < hk ? u : Kt + g0 + u - hk], tsum_scale);
          if (u < hk)
            sh.head_tsum[u] = a;
          else
            tw.tsum[u - hk] = a;
        }
      }
      __syncthreads();
      // 2. predicted grids: each thread a run of consecutive tiles
      double base = 0.0;
      if (first) {
        for (int u = 0; u < hk; u++) base += static_cast<double>(sh.head_tsum[u]);
      } else {
        base = static_cast<double>(sh.s);
      }
      const int per = (nt + NT - 1) / NT;
      const int r0 = min(nt, tid * per), r1 = min(nt, r0 + per);
      double run = 0.0;
      for (int t = r0; t < r1; t++) run += static_cast<double>(tw.tsum[t]);
      double pre = base + seq_block_exscan_d<NT>(run, sh);
      for (int t = r0; t < r1; t++) {
        tw.eu[t] = seq_grid_exp(static_cast<float>(pre));
        pre += static_cast<double>(tw.tsum[t]);
      }
      __syncthreads();
      // 3. maps on the predicted grids; in the first segment warp 0 runs
      // the head meanwhile
      if (first && warp == 0) {
        if (lane == 0) sh.done_pos = seq_head(head_buf, K, kind, target, sh.s);
      } else {
        const int w0 = first ? warp - 1 : warp, ws = first ? NW - 1 : NW;
        for (int t = w0; t < nt; t += ws) {
          float x[8];
          src.load8(K + (g0 + t) * kSeqTile + lane * 8, n, x);
          const SeqMap f = seq_warp_map(x, tw.eu[t]);
          if (lane == 0) tw.map[t] = f;
        }
      }
      __syncthreads();
      if (first && sh.done_pos >= 0) break;
    }
    // 4. the walk, 32 tiles a step: lane l takes tile t0 + l; an inclusive
    // warp scan of the maps gives N after every tile; the first tile that
    // is not a plain add (predicted on another grid, a partial tile under
    // reuse, or N at its end leaves the binade or meets the target) is
    // replayed exactly and the next step starts after it
    if (warp == 0) {
      float s = sh.s;
      int done = -1;
      int eu = seq_grid_exp(s);
      uint32_t N = seq_N(s);
      uint32_t thrN = seq_thr(kind, target, eu);
      bool cur = true;  // s matches (eu, N)
      int t0 = 0;
      while (t0 < nt) {
        if (!(s <= 3.40282347e38f)) {  // NaN or +inf: every later sum is s
          if (seq_meets(s, kind, target)) done = K + (g0 + t0) * kSeqTile;
          break;
        }
        const int t = t0 + lane;
        const bool valid = t < nt;
        SeqMap f = seq_identity();
        bool ok = false;
        if (valid) {
          f = tw.map[t];
          ok = tw.eu[t] == eu && (!reuse || K + (g0 + t + 1) * kSeqTile <= n);
        }
        SeqMap incl = f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          SeqMap w;
          w.e = __shfl_up_sync(0xFFFFFFFFu, incl.e, o);
          w.o = __shfl_up_sync(0xFFFFFFFFu, incl.o, o);
          if (lane >= o) incl = seq_compose(w, incl);
        }
        const uint32_t Na = seq_apply(incl, N);
        const bool bad = valid && (!ok || Na >= kSeqLimit || Na >= thrN);
        const unsigned bal = __ballot_sync(0xFFFFFFFFu, bad);
        if (bal == 0u) {
          const int last = min(31, nt - 1 - t0);
          N = __shfl_sync(0xFFFFFFFFu, Na, last);
          cur = false;
          t0 += 32;
          continue;
        }
        const int b = __ffs(bal) - 1;
        const uint32_t Nb = __shfl_sync(0xFFFFFFFFu, Na, b > 0 ? b - 1 : 0);
        if (b > 0) {
          N = Nb;
          cur = false;
        }
        if (!cur) s = seq_float(N, eu);
        const int j0 = K + (g0 + t0 + b) * kSeqTile, j1 = min(n, j0 + kSeqTile);
        const SeqResult rt = seq_tile_exact(src, j0, j0, j1, s, kind, target);
        s = rt.s;
        cur = true;
        if (rt.hit >= 0) {
          done = rt.hit;
          break;
        }
        const int eun = seq_grid_exp(s);
        if (eun != eu) {
          eu = eun;
          thrN = seq_thr(kind, target, eu);
        }
        N = seq_N(s);
        t0 += b + 1;
      }
      if (!cur) s = seq_float(N, eu);
      if (lane == 0) {
        sh.s = s;
        sh.done_pos = done;
      }
    }
    __syncthreads();
    if (sh.done_pos >= 0) break;
  }
  SeqResult r{sh.s, sh.done_pos};
  __syncthreads();
  return r;
}

}  // namespace pz
