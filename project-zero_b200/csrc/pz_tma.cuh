// pz_tma.cuh — bulk asynchronous copies (TMA, untiled cp.async.bulk) from
// global into shared memory, completed on mbarriers, with bounded waits.
//
// Rules kept here: source and destination 16-byte aligned, sizes multiples
// of 16 bytes, no multicast, and every wait gives up after a clock budget so
// a copy that never lands cannot hang the GPU (the caller records an error
// and stops issuing).
#pragma once

#include <stdint.h>

namespace pz {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared accesses before later
// async-proxy (bulk copy) writes to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// global -> shared bulk copy; `bytes` a multiple of 16, both ends 16-byte aligned.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete; false after `budget` clock
// cycles without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    __nanosleep(64);  // leave the issue slots to warps with work
    if (clock64() - t0 > budget) return false;
  }
  return true;
}

// ~2 s at the B200's 1965 MHz boost clock.
constexpr long long kWaitBudget = 4000000000ll;
// shorter budget used while draining after a failure
constexpr long long kDrainBudget = 200000000ll;

}  // namespace pz

namespace pz {

// ---------------------------------------------------------------------------
// Per-thread asynchronous copies (cp.async, 16 bytes each) from global into
// shared memory.  A thread waits only for its own copies (wait_group), so a
// warp that reads back exactly the vectors its lanes copied needs no barrier
// and no spin-wait.  These travel the load path of ordinary global loads
// (about a microsecond of latency under full load), where a bulk copy
// completes only when all of its bytes have landed.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Waits until at most n (0..7) of this thread's copy groups are pending.
__device__ __forceinline__ void cp_async_wait_n(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}

}  // namespace pz
