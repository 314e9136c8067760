// pz_warpsel.cuh — warp-level exact top-k over 64-bit ordered keys.
//
// Each warp filters its share of a slice against its own threshold and keeps
// the survivors in a warp-private shared-memory buffer (ballot appends, no
// atomics, no block barrier).  When the buffer fills, a bitwise radix select
// (counts by __reduce_add_sync) finds the exact k-th largest key, the buffer
// is compacted to the k best and the threshold rises.  Keys are unique per
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

// The j-th largest (1-based) of R keys per lane held in registers (32*R
// keys, duplicates allowed: ties count once per copy).  Warp-wide.
template <int R>
__device__ __forceinline__ unsigned long long warp_jth_reg(const unsigned long long (&v)[R], int j) {
  unsigned long long mn = ~0ull, mx = 0ull;
#pragma unroll
  for (int r = 0; r < R; r++) {
    mn = v[r] < mn ? v[r] : mn;
    mx = v[r] > mx ? v[r] : mx;
  }
  mn = warp_min_u64(mn);
  mx = warp_max_u64(mx);
  if (mn == mx) return mn;
  int b = 63 - __clzll(static_cast<long long>(mn ^ mx));
  unsigned long long mask = b == 63 ? 0ull : (~0ull << (b + 1));
  unsigned long long prefix = mn & mask;
  int need = j;
  for (; b >= 0; b--) {
    const unsigned long long bit = 1ull << b;
    int c1 = 0, cm = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const bool m = (v[r] & mask) == prefix;
      cm += m ? 1 : 0;
      c1 += (m && (v[r] & bit)) ? 1 : 0;
    }
    cm = __reduce_add_sync(0xFFFFFFFFu, cm);
    if (cm == need) break;  // all keys under this prefix are in: the j-th is their minimum
    c1 = __reduce_add_sync(0xFFFFFFFFu, c1);
    if (c1 >= need) {
      prefix |= bit;
    } else {
      need -= c1;
    }
    mask |= bit;
  }
  unsigned long long kth = ~0ull;
#pragma unroll
  for (int r = 0; r < R; r++)
    if ((v[r] & mask) == prefix && v[r] < kth) kth = v[r];
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

// Warp-private candidate buffer state (registers, warp-uniform).
struct WarpCand {
  unsigned long long *keys;  // shared memory, `cap` slots
  int cap;
  int n;
  unsigned long long tau;    // keys must be > tau to enter
  float tau_f;               // value part of tau: values below it never enter
  // Thresholds shared with the other warps of the block (shared memory) and
  // with the other slices of the row (global): each warp's k-th best key is
  // a lower bound on the row's k-th best, so the largest one is too.
  unsigned long long *block_tau;
  unsigned long long *row_tau;
};

// Adopts a higher threshold published by another warp or slice.
__device__ __forceinline__ void warp_adopt(WarpCand &w, unsigned long long t) {
  if (t > w.tau) {
    w.tau = t;
    w.tau_f = key_val(t);
  }
}

// Keeps the best k keys of a full buffer and raises its threshold.
__device__ __noinline__ void warp_make_room(WarpCand &w, int k) {
  const unsigned long long kth = warp_kth(w.keys, w.n, k);
  w.n = warp_compact_ge(w.keys, w.n, kth);
  if (kth > w.tau) {
    w.tau = kth;
    w.tau_f = key_val(kth);
  }
  if (lane_id() == 0) {
    if (w.block_tau) atomicMax(w.block_tau, w.tau);
    if (w.row_tau) atomicMax(w.row_tau, w.tau);
  }
  __syncwarp();
}

// Offers one key per lane (`q` = the lane has a key above tau).  Keeps the
// buffer exact: when the batch does not fit, selects the best k first.
__device__ __forceinline__ void warp_offer(WarpCand &w, int k, bool q, unsigned long long key) {
  uint32_t bal = __ballot_sync(0xFFFFFFFFu, q);
  if (bal == 0u) return;
  if (w.n + __popc(bal) > w.cap) {
    warp_make_room(w, k);
    q = q && key > w.tau;
    bal = __ballot_sync(0xFFFFFFFFu, q);
  }
  if (q) w.keys[w.n + __popc(bal & lanemask_lt())] = key;
  w.n += __popc(bal);
  __syncwarp();
}

// Reduces the buffer to its best k keys (unordered).
__device__ __forceinline__ void warp_finish(WarpCand &w, int k) {
  if (w.n > k) {
    const unsigned long long kth = warp_kth(w.keys, w.n, k);
    w.n = warp_compact_ge(w.keys, w.n, kth);
    if (kth > w.tau) {
      w.tau = kth;
      w.tau_f = key_val(kth);
    }
  }
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
