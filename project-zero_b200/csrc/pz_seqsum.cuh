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

struct SeqShared {
  SeqMap warp_tot[32];
  float s;
  int cross;
  int hit;
  int done_pos;
  float hit_s;
};

// Exclusive block scan of SeqMap; also returns the block total.
template <int NT>
__device__ __forceinline__ SeqMap seq_block_exscan(SeqMap v, SeqMap &total,
                                                   SeqShared &sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  SeqMap incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    SeqMap w;
    w.e = __shfl_up_sync(0xFFFFFFFFu, incl.e, o);
    w.o = __shfl_up_sync(0xFFFFFFFFu, incl.o, o);
    if (lane >= o) incl = seq_compose(w, incl);
  }
  if (lane == 31) sh.warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    constexpr int NW = NT / 32;
    SeqMap t = lane < NW ? sh.warp_tot[lane] : seq_identity();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      SeqMap w;
      w.e = __shfl_up_sync(0xFFFFFFFFu, t.e, o);
      w.o = __shfl_up_sync(0xFFFFFFFFu, t.o, o);
      if (lane >= o) t = seq_compose(w, t);
    }
    if (lane < NW) sh.warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  SeqMap before_warp = warp ? sh.warp_tot[warp - 1] : seq_identity();
  total = sh.warp_tot[NT / 32 - 1];
  // exclusive within the warp
  SeqMap ex;
  ex.e = __shfl_up_sync(0xFFFFFFFFu, incl.e, 1);
  ex.o = __shfl_up_sync(0xFFFFFFFFu, incl.o, 1);
  if (lane == 0) ex = seq_identity();
  __syncthreads();  // warp_tot may be rewritten by the next scan
  return seq_compose(before_warp, ex);
}

enum SeqTarget : int { kSeqNone = 0, kSeqGE = 1, kSeqGT = 2 };

struct SeqResult {
  float s;   // sum of all n terms, or the prefix sum at the hit
  int hit;   // first j whose prefix meets the target, or -1
};

// Replays s = fl(s + x_j) for j = 0..n-1 (x_j = get(j) >= 0) starting from
// s = 0.  With a target, stops at the first j where s_j >= target (kSeqGE)
// or s_j > target (kSeqGT).  Block-wide call.  get must be a pure function
// of j (the next chunk's terms are fetched while the current one is
// scanned).
//
// The first head_cap terms (the running sum doubles, and so leaves its
// binade, most often early on: about once per doubling of the terms seen)
// are evaluated by all threads into head_buf and added in order by one
// thread; the rest go E consecutive terms per thread per chunk through the
// parallel replay, which restarts only at the few binade crossings left.
// The maps of a thread's terms are not kept: they are recomputed from the
// terms (a few integer operations) where the prefixes are needed.
template <int NT, int E, typename Get>
__device__ SeqResult seq_scan(int n, Get get, int kind, float target,
                              SeqShared &sh, float *head_buf, int head_cap) {
  const int tid = threadIdx.x;
  const int K = n < head_cap ? n : head_cap;
  for (int j = tid; j < K; j += NT) head_buf[j] = get(j);
  __syncthreads();
  if (tid == 0) {
    float s = 0.0f;
    int done = -1;
    for (int j = 0; j < K; j++) {
      s = __fadd_rn(s, head_buf[j]);
      if ((kind == kSeqGE && s >= target) || (kind == kSeqGT && s > target)) {
        done = j;
        break;
      }
    }
    sh.s = s;
    sh.done_pos = done;
  }
  __syncthreads();
  float x[E], xn[E];
  auto fetch = [&](int c, float(&dst)[E]) {
#pragma unroll
    for (int e = 0; e < E; e++) {
      const int j = c + tid * E + e;
      dst[e] = j < n ? get(j) : 0.0f;
    }
  };
  if (K < n && sh.done_pos < 0) fetch(K, x);
  for (int c0 = K; c0 < n && sh.done_pos < 0; c0 += NT * E) {
    if (c0 + NT * E < n) fetch(c0 + NT * E, xn);  // in flight during this chunk
    int start = c0;
    bool chunk_done = false;
    while (!chunk_done) {
      const float s = sh.s;
      const int eu = seq_grid_exp(s);
      const uint32_t N0 = seq_N(s);
      // integer form of the target on this grid
      unsigned long long thrN = ~0ull;
      if (kind != kSeqNone) {
        const double q = static_cast<double>(target) * exp2(static_cast<double>(-eu));
        if (kind == kSeqGE) {
          // s_j >= target  <=>  N_j >= ceil(q)
          const double c = ceil(q);
          thrN = (q != q) ? ~0ull : (c <= 0.0 ? 0ull : (c >= 1e15 ? ~0ull : static_cast<unsigned long long>(c)));
        } else {
          // s_j > target  <=>  N_j > floor(q)  <=>  N_j >= floor(q) + 1
          const double f = floor(q);
          thrN = (q != q) ? ~0ull : (f < 0.0 ? 0ull : (f >= 1e15 ? ~0ull : static_cast<unsigned long long>(f) + 1ull));
        }
      }
      SeqMap F = seq_identity();
#pragma unroll
      for (int e = 0; e < E; e++) {
        const int j = c0 + tid * E + e;
        if (j >= start && j < n) F = seq_compose(F, seq_elem(x[e], eu));
      }
      if (tid == 0) {
        sh.cross = 0x7FFFFFFF;
        sh.hit = 0x7FFFFFFF;
      }
      SeqMap total;
      const SeqMap P = seq_block_exscan<NT>(F, total, sh);
      uint32_t N = seq_apply(P, N0);
      int mycross = 0x7FFFFFFF, myhit = 0x7FFFFFFF;
      uint32_t Nc = 0, Nh = 0;
      float xc = 0.0f;
#pragma unroll
      for (int e = 0; e < E; e++) {
        const int j = c0 + tid * E + e;
        if (j >= start && j < n && mycross == 0x7FFFFFFF && myhit == 0x7FFFFFFF) {
          const uint32_t Nn = seq_apply(seq_elem(x[e], eu), N);
          if (Nn >= kSeqLimit) {
            mycross = j;
            Nc = N;
            xc = x[e];
          } else if (Nn >= thrN) {
            myhit = j;
            Nh = Nn;
          }
          N = Nn;
        }
      }
      if (mycross != 0x7FFFFFFF) atomicMin(&sh.cross, mycross);
      if (myhit != 0x7FFFFFFF) atomicMin(&sh.hit, myhit);
      __syncthreads();
      const int cross = sh.cross, hit = sh.hit;
      __syncthreads();
      if (hit < cross) {
        if (myhit == hit) {
          sh.s = seq_float(Nh, eu);
          sh.done_pos = hit;
        }
        chunk_done = true;
      } else if (cross != 0x7FFFFFFF) {
        if (mycross == cross) {
          const float sn = __fadd_rn(seq_float(Nc, eu), xc);
          sh.s = sn;
          if ((kind == kSeqGE && sn >= target) || (kind == kSeqGT && sn > target))
            sh.done_pos = cross;
        }
        start = cross + 1;
      } else {
        if (tid == 0) sh.s = seq_float(seq_apply(total, N0), eu);
        chunk_done = true;
      }
      __syncthreads();
      if (sh.done_pos >= 0) break;
    }
#pragma unroll
    for (int e = 0; e < E; e++) x[e] = xn[e];
  }
  SeqResult r;
  r.s = sh.s;
  r.hit = sh.done_pos;
  __syncthreads();
  return r;
}

}  // namespace pz
