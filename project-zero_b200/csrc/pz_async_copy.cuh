// pz_async_copy.cuh — per-thread asynchronous copies (cp.async, 16 bytes
// each) from global into shared memory.
//
// A thread waits only for its own copies (wait_group), so a warp that reads
// back exactly the vectors its lanes copied needs no barrier and no
// spin-wait.  These travel the load path of ordinary global loads (about a
// microsecond of latency under full load), where a bulk (TMA) copy
// completes only when all of its bytes have landed; for this stream, whose
// consumer is light, bulk copies measured no faster and would need waits on
// mbarriers.  Source and destination are 16-byte aligned.
#pragma once

#include <stdint.h>

namespace pz {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's copy groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace pz
