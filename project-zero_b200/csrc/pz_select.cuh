// pz_select.cuh — block-level candidate buffer with exact top-k selection.
//
// The buffer holds 64-bit ordered keys (see pz_device.cuh) in shared
// memory.  Threads append keys above the running threshold `tau` (the k-th
// best key kept so far); when the buffer passes its high-water mark, an
// MSD radix select over the keys (8-bit digits, shared-memory histogram)
// finds the k-th largest key exactly, keeps the k best and raises `tau`.
// Keys are unique per element, so the kept set is exactly the reference's
// top-k set (value desc, lower index first among ties).
#pragma once

#include "pz_device.cuh"

namespace pz {

struct SelShared {
  uint32_t hist[256];
  unsigned long long prefix;
  unsigned long long mask;
  unsigned long long kth;
  unsigned long long tau;   // admission threshold: keys > tau may enter
  int need;
  int done;
  int digit;
  int above;
  int n;                    // keys in the buffer (may exceed cap transiently)
  int cnt;
  int overflow;
};

// Keeps the k largest of cand[0..n) in cand[0..k) (unordered) and sets
// sh.tau to the smallest kept key.  Requires k < n <= MAXPER * NT.
// All threads of the block must call it.
template <int NT, int MAXPER>
__device__ __noinline__ void block_select(unsigned long long *cand, int n, int k,
                            SelShared &sh) {
  const int tid = threadIdx.x;
  const uint32_t lane = lane_id();
  // Bytes shared by every key need no pass: start at the first byte where
  // the smallest and largest keys differ (keys are unique, n >= 2).
  unsigned long long mn = ~0ull, mx = 0ull;
  for (int i = tid; i < n; i += NT) {
    const unsigned long long key = cand[i];
    mn = key < mn ? key : mn;
    mx = key > mx ? key : mx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long a = __shfl_xor_sync(0xFFFFFFFFu, mn, o);
    const unsigned long long b = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    mn = a < mn ? a : mn;
    mx = b > mx ? b : mx;
  }
  if (tid == 0) {
    sh.prefix = ~0ull;  // running min
    sh.mask = 0ull;     // running max
  }
  __syncthreads();
  if (lane == 0) {
    atomicMin(&sh.prefix, mn);
    atomicMax(&sh.mask, mx);
  }
  __syncthreads();
  const unsigned long long gmin = sh.prefix, gmax = sh.mask;
  const int lead = __clzll(static_cast<long long>(gmin ^ gmax));  // < 64
  const int top_shift = 56 - 8 * (lead >> 3);
  __syncthreads();
  if (tid == 0) {
    const unsigned long long common = top_shift == 56 ? 0ull : (~0ull << (top_shift + 8));
    sh.prefix = gmin & common;
    sh.mask = common;
    sh.need = k;
    sh.done = 0;
    sh.kth = ~0ull;
    sh.cnt = 0;
    sh.digit = 0;
    sh.above = 0;
  }
  __syncthreads();
  const int n_up = (n + NT - 1) / NT * NT;
  for (int shift = top_shift; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += NT) sh.hist[i] = 0;
    __syncthreads();
    const unsigned long long prefix = sh.prefix, mask = sh.mask;
    for (int i = tid; i < n_up; i += NT) {
      bool act = false;
      uint32_t d = 256u + lane;
      if (i < n) {
        const unsigned long long key = cand[i];
        act = (key & mask) == prefix;
        if (act) d = static_cast<uint32_t>((key >> shift) & 0xFFu);
      }
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      if (act && lane == static_cast<uint32_t>(__ffs(peers) - 1))
        atomicAdd(&sh.hist[d], static_cast<uint32_t>(__popc(peers)));
    }
    __syncthreads();
    if (tid < kWarp) {
      // lane l owns bins 255-8l .. 248-8l, scanned from the top
      uint32_t c[8];
      int sum = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        c[j] = sh.hist[255 - 8 * tid - j];
        sum += static_cast<int>(c[j]);
      }
      const int incl = warp_incl_scan(sum);
      const int excl = incl - sum;
      const int need = sh.need;
      if (excl < need && need <= incl) {
        int run = excl;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          if (run + static_cast<int>(c[j]) >= need) {
            sh.digit = 255 - 8 * tid - j;
            sh.above = run;
            break;
          }
          run += static_cast<int>(c[j]);
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      const int d = sh.digit;
      sh.need -= sh.above;
      sh.prefix |= static_cast<unsigned long long>(d) << shift;
      sh.mask |= 0xFFull << shift;
      if (static_cast<int>(sh.hist[d]) == sh.need) sh.done = 1;
    }
    __syncthreads();
    if (sh.done) break;
  }
  // Selected: masked key above the prefix (a higher digit somewhere), or
  // equal to it (the final bucket, taken whole).
  const unsigned long long prefix = sh.prefix, mask = sh.mask;
  unsigned long long val[MAXPER];
  bool sel[MAXPER];
  unsigned long long mymin = ~0ull;
#pragma unroll
  for (int j = 0; j < MAXPER; j++) {
    const int i = tid + j * NT;
    val[j] = (i < n) ? cand[i] : 0ull;
    const unsigned long long mk = val[j] & mask;
    sel[j] = (i < n) && (mk >= prefix);
    if (i < n && mk == prefix && val[j] < mymin) mymin = val[j];
  }
  if (mymin != ~0ull) atomicMin(&sh.kth, mymin);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < MAXPER; j++) {
    const uint32_t b = __ballot_sync(0xFFFFFFFFu, sel[j]);
    if (b) {
      int base = 0;
      if (lane == static_cast<uint32_t>(__ffs(b) - 1))
        base = atomicAdd(&sh.cnt, __popc(b));
      base = __shfl_sync(0xFFFFFFFFu, base, __ffs(b) - 1);
      if (sel[j]) cand[base + __popc(b & lanemask_lt())] = val[j];
    }
  }
  __syncthreads();
  if (tid == 0) {
    sh.n = k;
    sh.tau = sh.kth;
  }
  __syncthreads();
}

// Appends the keys flagged in `q` (bit e <-> keys[e]) to the buffer with
// one shared atomic per warp.  Returns the flags of keys that did not fit.
template <int EPT>
__device__ __forceinline__ uint32_t buffer_append(
    unsigned long long *cand, int cap, SelShared &sh,
    const unsigned long long (&keys)[EPT], uint32_t q) {
  const int mine = __popc(q);
  const int incl = warp_incl_scan(mine);
  const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  if (total == 0) return 0u;
  int base = 0;
  if (lane_id() == 31) base = atomicAdd(&sh.n, total);
  base = __shfl_sync(0xFFFFFFFFu, base, 31) + (incl - mine);
  uint32_t pend = 0;
#pragma unroll
  for (int e = 0; e < EPT; e++) {
    if (q & (1u << e)) {
      if (base < cap)
        cand[base] = keys[e];
      else
        pend |= 1u << e;
      base++;
    }
  }
  return pend;
}

// One round of candidates for the top-k buffer: every thread offers up to
// EPT keys (flag bit e set in `valid` when keys[e] is a real candidate).
// Keys above tau are appended; on overflow or past the high-water mark the
// block selects the best k and retries what did not fit.  Block-wide call.
template <int NT, int MAXPER, int EPT>
__device__ void offer_round(unsigned long long *cand, int cap, int hwm, int k,
                            SelShared &sh,
                            const unsigned long long (&keys)[EPT],
                            uint32_t valid) {
  unsigned long long tau = sh.tau;
  uint32_t q = 0;
#pragma unroll
  for (int e = 0; e < EPT; e++)
    if ((valid & (1u << e)) && keys[e] > tau) q |= 1u << e;
  uint32_t pend = 0;
  if (__any_sync(0xFFFFFFFFu, q != 0)) pend = buffer_append<EPT>(cand, cap, sh, keys, q);
  int overflow = __syncthreads_or(pend != 0);
  int n = sh.n < cap ? sh.n : cap;
  if (overflow || n > hwm) {
    __syncthreads();
    if (n > k) block_select<NT, MAXPER>(cand, n, k, sh);
    else if (threadIdx.x == 0) sh.n = n;
    __syncthreads();
    while (overflow) {
      tau = sh.tau;
      q = 0;
#pragma unroll
      for (int e = 0; e < EPT; e++)
        if ((pend & (1u << e)) && keys[e] > tau) q |= 1u << e;
      pend = 0;
      if (__any_sync(0xFFFFFFFFu, q != 0)) pend = buffer_append<EPT>(cand, cap, sh, keys, q);
      overflow = __syncthreads_or(pend != 0);
      n = sh.n < cap ? sh.n : cap;
      if (overflow) {
        __syncthreads();
        if (n > k) block_select<NT, MAXPER>(cand, n, k, sh);
        else if (threadIdx.x == 0) sh.n = n;
        __syncthreads();
      }
    }
  }
}

// Bitonic sort of cand[0..npow2) descending (npow2 a power of two, padding
// keys 0 sort last).  Block-wide call.
template <int NT>
__device__ __noinline__ void block_sort_desc(unsigned long long *cand, int npow2) {
  for (int size = 2; size <= npow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < (npow2 >> 1); i += NT) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long a = cand[lo], b = cand[hi];
        if (desc ? (a < b) : (a > b)) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace pz
