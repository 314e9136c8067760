// pz_warpsel.cuh — one warp's exact selection over 64-bit ordered keys in
// shared memory: the k-th largest key (a bitwise radix select, counts by
// __reduce_add_sync), compaction to the keys at or above it, and a bitonic
// sort.  Used where a row's slice lists are merged.  Keys are unique per
// element, so the result is exactly the reference's top-k set.
#pragma once

#include "pz_device.cuh"

namespace pz {

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// The k-th largest of keys[0..n) (distinct keys, 1 <= k <= n).  Warp-wide.
__device__ __noinline__ unsigned long long warp_kth(const unsigned long long *keys, int n, int k) {
  const int lane = static_cast<int>(lane_id());
  unsigned long long mn = ~0ull, mx = 0ull;
  for (int i = lane; i < n; i += 32) {
    const unsigned long long key = keys[i];
    mn = key < mn ? key : mn;
    mx = key > mx ? key : mx;
  }
  mn = warp_min_u64(mn);
  mx = warp_max_u64(mx);
  if (k >= n) return mn;
  int b = 63 - __clzll(static_cast<long long>(mn ^ mx));
  unsigned long long mask = b == 63 ? 0ull : (~0ull << (b + 1));
  unsigned long long prefix = mn & mask;
  int need = k;
  for (; b >= 0; b--) {
    const unsigned long long bit = 1ull << b;
    int c1 = 0, cm = 0;
    for (int i = lane; i < n; i += 32) {
      const unsigned long long key = keys[i];
      if ((key & mask) == prefix) {
        cm++;
        c1 += (key & bit) ? 1 : 0;
      }
    }
    cm = __reduce_add_sync(0xFFFFFFFFu, cm);
    c1 = __reduce_add_sync(0xFFFFFFFFu, c1);
    if (cm == need) break;  // every key under this prefix is kept
    if (c1 >= need) {
      prefix |= bit;
    } else {
      need -= c1;
    }
    mask |= bit;
  }
  unsigned long long kth = ~0ull;
  for (int i = lane; i < n; i += 32) {
    const unsigned long long key = keys[i];
    if ((key & mask) == prefix && key < kth) kth = key;
  }
  return warp_min_u64(kth);
}

// Moves the keys >= kth to the front of keys[0..n) in place, keeping their
// order; returns their number.  Warp-wide.
__device__ __noinline__ int warp_compact_ge(unsigned long long *keys, int n, unsigned long long kth) {
  const uint32_t lane = lane_id();
  int out = 0;
  for (int base = 0; base < n; base += 32) {
    const int i = base + static_cast<int>(lane);
    const unsigned long long key = i < n ? keys[i] : 0ull;
    const bool s = i < n && key >= kth;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, s);
    __syncwarp();
    if (s) keys[out + __popc(bal & lanemask_lt())] = key;
    out += __popc(bal);
    __syncwarp();
  }
  return out;
}

// Bitonic sort of a[0..n2) descending (n2 a power of two), one warp.
__device__ __noinline__ void warp_sort_desc(unsigned long long *a, int n2) {
  const int lane = static_cast<int>(lane_id());
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncwarp();
      for (int i = lane; i < (n2 >> 1); i += 32) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long x = a[lo], y = a[hi];
        if (desc ? (x < y) : (x > y)) {
          a[lo] = y;
          a[hi] = x;
        }
      }
    }
  }
  __syncwarp();
}

}  // namespace pz
