// pz_device.cuh — device-side building blocks of the B200 sampler.
//
// Everything numeric here reproduces the reference's float arithmetic bit
// for bit: explicit __f*_rn intrinsics (no FMA contraction), the
// reference's operation order, and the xorshift64* stream of
// reference src/sampling/rng.c:8-17.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pz_sampling.h"
#include "pz_kernels.cuh"

namespace pz {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Ordered keys.  A candidate is (value v, global id i).  The reference ranks
// by value descending and, among equal values, lower index first (strict
// `>` in reference src/sampling/top_k.c:37,40 and argmax.c:7; stable qsort in
// top_p.c:77).  IEEE equality treats -0 and +0 as equal, so -0 is folded
// into +0 before the value is mapped to an order-preserving uint32.  The
// 64-bit key (ord(v) << 32) | (~i) is then unique per element and its
// unsigned order is exactly the reference's ranking.  NaN never gets a key.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2ord(float v) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}
__device__ __forceinline__ uint64_t mkkey(float v, uint32_t idx) {
  return (static_cast<uint64_t>(f2ord(v)) << 32) | static_cast<uint32_t>(~idx);
}
__device__ __forceinline__ float key_val(uint64_t k) {
  return ord2f(static_cast<uint32_t>(k >> 32));
}
__device__ __forceinline__ int key_idx(uint64_t k) {
  return static_cast<int>(~static_cast<uint32_t>(k));
}
// Keys of values <= -1e30 can never enter a top-k list (the list starts as
// -1e30 and admission is strict `>`, top_k.c:30-37).
__device__ __forceinline__ uint64_t key_topk_floor() {
  return (static_cast<uint64_t>(f2ord(-1e30f)) << 32) | 0xFFFFFFFFull;
}

// ---------------------------------------------------------------------------
// RNG: xorshift64* of reference src/sampling/rng.c:8-17.  The 31-bit integer
// is converted with round-to-nearest (it can round up to 2^31, so the draw
// can be exactly 1.0f) and divided by 2^31 exactly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rng_next(unsigned long long &state) {
  unsigned long long s = state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  state = s;
  const uint32_t t = static_cast<uint32_t>((s * 0x2545F4914F6CDD1DULL) >> 33);
  return __fdiv_rn(__uint2float_rn(t), 2147483648.0f);
}

// ---------------------------------------------------------------------------
// exp for the softmax numerators.  The reference calls glibc's expf, which
// is correctly rounded except within ~1e-3 ulp of a rounding midpoint.  We
// evaluate exp in double (CUDA's exp(), <= 1 ulp of double) and round once
// to float, which is correctly rounded except within ~2^-29 ulp of a
// midpoint; the two agree on all but a few inputs in a thousand, and then
// differ by one ulp.  The function is monotone, so it never reorders
// candidates.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float cr_expf(float x) {
  return __double2float_rn(exp(static_cast<double>(x)));
}

// ---------------------------------------------------------------------------
// Row plan: how one row is sampled (reference src/transformer/generate.c:151-170
// plus the contract of include/pz_sampling.h).
// ---------------------------------------------------------------------------
enum RowMode : int {
  kModeGreedy = 0,       // argmax of the penalised logits, no draw
  kModeTopK = 1,         // selection + (top-p steps | top-k softmax) over the list
  kModeTopPFull = 2,     // sample_top_p over the whole row
  kModeSoftmaxFull = 3,  // softmax + CDF walk over the whole row
};

struct RowPlan {
  int mode;
  int keff;       // list length for kModeTopK
  int p_on;       // 0 < p < 1
  int pen_on;     // penalties change values
  int divide;     // temperature as x / T
  float T;
  float inv_T;    // 1.0f / T (temperature.c:12)
  float p;
  float rep, freq, pres;
};

__device__ __forceinline__ RowPlan plan_row(const pz_sampler_config &c, int V) {
  RowPlan P;
  P.T = c.temperature;
  P.p = c.top_p;
  P.rep = c.repetition_penalty;
  P.freq = c.frequency_penalty;
  P.pres = c.presence_penalty;
  P.pen_on = (P.rep != 1.0f || P.freq != 0.0f || P.pres != 0.0f);
  P.divide = (c.flags & PZ_CFG_TEMP_DIVIDE) ? 1 : 0;
  P.p_on = (P.p < 1.0f && P.p > 0.0f);
  const int k = c.top_k;
  if (c.flags & PZ_CFG_TOPK_LEGACY) {
    // sample_top_k's clamping (top_k.c:11-18); no nucleus step
    int kk = k > V ? V : k;
    if (kk <= 0) kk = 1;
    if (kk > PZ_TOP_K_MAX) kk = PZ_TOP_K_MAX;
    P.keff = kk;
    P.p_on = 0;
  } else {
    P.keff = (k <= 0 || k >= V) ? 0 : (k > PZ_TOP_K_MAX ? PZ_TOP_K_MAX : k);
  }
  if (c.flags & PZ_CFG_TOPP_ALWAYS) P.p_on = 1;
  P.inv_T = 1.0f;
  if (P.T <= 0.0f || P.T < 1e-6f) {
    P.mode = kModeGreedy;
  } else {
    P.inv_T = __fdiv_rn(1.0f, P.T);
    if (P.keff > 0)
      P.mode = kModeTopK;
    else
      P.mode = P.p_on ? kModeTopPFull : kModeSoftmaxFull;
  }
  return P;
}

// Penalty of the contract (A8) for an id seen `c` times.
__device__ __forceinline__ float penalize(float x, int c, const RowPlan &P) {
  float v = x;
  if (P.rep != 1.0f) v = (v > 0.0f) ? __fdiv_rn(v, P.rep) : __fmul_rn(v, P.rep);
  float pen = __fmul_rn(static_cast<float>(c), P.freq);
  pen = __fadd_rn(pen, P.pres);
  return __fsub_rn(v, pen);
}

// Temperature (A3): x * (1/T), or x / T with PZ_CFG_TEMP_DIVIDE.
__device__ __forceinline__ float temper(float x, const RowPlan &P) {
  return P.divide ? __fdiv_rn(x, P.T) : __fmul_rn(x, P.inv_T);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// ---------------------------------------------------------------------------
// Warp helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ int warp_incl_scan(int v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int w = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (static_cast<int>(lane_id()) >= o) v += w;
  }
  return v;
}

}  // namespace pz
