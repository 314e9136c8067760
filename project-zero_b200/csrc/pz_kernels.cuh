// pz_kernels.cuh — launch arguments of the sampler kernels (host + device).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pz_sampling.h"

// Config flags used only by the legacy single-row entry points.
// sample_top_k's own clamping (reference src/sampling/top_k.c:11-18):
// k > V -> V, k <= 0 -> 1, k > 1024 -> 1024; the list may cover the row.
#define PZ_CFG_TOPK_LEGACY 0x2u
// sample_top_p's steps whatever p is (reference src/sampling/top_p.c:30-108
// is called only for 0 < p < 1 by the generate loop, but the function itself
// accepts any p).
#define PZ_CFG_TOPP_ALWAYS 0x4u

namespace pz {

constexpr int kSliceThreads = 256;
constexpr int kFullThreads = 512;
constexpr int kFullCtasPerSm = 2;   // full_kernel rows in flight per SM
constexpr int kCapB = 1024;   // candidate buffer room above the list length
constexpr int kTQK = 64;      // lists up to this long: slice_kernel's coarse sketch
// Rows handed to full_kernel are filed in cost classes (class c at
// full_rows + c * full_stride, its count in n_full[c]); full_kernel's CTAs
// claim them one at a time through the counter n_full[kFullClasses],
// heaviest class first.
constexpr int kFullClasses = 8;
constexpr int kRowBits = 2;   // row_flags bits

struct SliceArgs {
  const void *logits;
  int64_t ld;           // elements between rows
  int V;                // columns held here (slice of the vocabulary when sharded)
  int V_global;         // vocabulary size the row's settings refer to
  int64_t v_offset;     // global id of column 0
  int B;
  const pz_sampler_config *cfg;
  const int32_t *hist;
  const int32_t *hist_off;
  int B1;               // rows [0, B1) are read by one CTA each
  int S;                // CTAs per row for the rows after B1 (split rows)
  int L;                // columns per CTA of a split row (multiple of 8)
  int kcap;             // power of two >= largest k_eff in the launch
  int kmax;             // declared largest k_eff (rows above it are rejected)
  int hcap;             // longest history a row may have (0: no history)
  int hts;              // history hash slots per CTA (power of two >= 2*hcap, or 0)
  int hshift;           // 32 - log2(hts)
  int nstages;          // bulk-copy ring slots per warp
  int mode_emit;        // 1: write the merged local list (vocab sharding), no draw
  int no_full_vocab;
  // The first wave's list-row CTAs start stagger_ns apart per CTA slot of
  // an SM (0: off); the first stagger_ctas CTAs are that wave.
  int stagger_ns;
  int stagger_ctas;
  int stagger_occ;      // CTAs in flight per SM
  // Batches with lists longer than kTQK, in two launches: slice_kernel
  // (kmax <= kTQK) files each row whose list is longer than kmax, up to
  // defer_kmax, in defer_rows instead of flagging it; slice_long_kernel
  // (deferred = 1) then takes row defer_rows[u] in CTA u < *n_defer.
  int defer_kmax;                  // 0: no deferring
  int deferred;
  int32_t *defer_rows;             // [B]
  int32_t *n_defer;                // [1] (zero before the first launch)
  // scratch
  unsigned long long *slice_keys;  // [(B-B1)*S][kcap] split rows' slice lists
  int32_t *slice_cnt;              // [(B-B1)*S]
  uint32_t *row_arrive;            // [B] slices of a split row done (0 between calls)
  uint32_t *row_flags;             // [B]
  unsigned long long *row_tau;     // [B] shared list threshold (0 between calls)
  unsigned long long *row_best;    // [B]
  int32_t *full_rows;              // [kFullClasses][full_stride]
  int32_t *n_full;                 // [kFullClasses + 1] (zero before the call)
  int full_stride;
  unsigned long long *emit_keys;   // [B][kcap+1] (mode_emit); slot kcap = count | flags
  // outputs
  unsigned long long *rng;
  int32_t *out;
  int32_t *cand_ids;
  float *cand_probs;
  int32_t *n_cand;
  int32_t *row_status;
  int cand_stride;
};

struct FullArgs {
  const void *logits;
  int64_t ld;
  int V;
  int B;
  const pz_sampler_config *cfg;
  const int32_t *hist;
  const int32_t *hist_off;
  int hcap;
  const unsigned long long *row_best;
  const uint32_t *row_flags;
  const int32_t *full_rows;       // [kFullClasses][full_stride]
  int32_t *n_full;                // [kFullClasses] counts, then the claim counter
  int full_stride;
  uint32_t *sort_a;     // [gridDim][2*maxV] (prob key, index) pairs
  uint32_t *sort_b;
  int64_t sort_stride;  // uint32 elements per CTA in sort_a/sort_b
  float *escr;          // [gridDim][e_stride] e values of the CTA's row
  int64_t e_stride;     // floats per CTA in escr (a multiple of 64)
  int smem_sort_cap;    // (key, value) entries an in-smem sort holds
  unsigned long long *rng;
  int32_t *out;
};

struct MergeArgs {               // vocab-sharded merge after the allgather
  const unsigned long long *gathered;  // [G][B][kcap+1]; slot kcap = count | flags
  int G;
  int B;
  int kcap;
  int kmax;
  int V_global;
  const pz_sampler_config *cfg;
  unsigned long long *rng;
  int32_t *out;
  int32_t *cand_ids;
  float *cand_probs;
  int32_t *n_cand;
  int32_t *row_status;
  int cand_stride;
};

struct LogprobArgs {              // logprob_kernel
  const void *logits;
  int64_t ld;
  int V;
  int B;
  const pz_sampler_config *cfg;
  const int32_t *hist;
  const int32_t *hist_off;
  int hcap;                      // longest history applied (a power of two >= it)
  const int32_t *tokens;
  const int32_t *cand_ids;
  const int32_t *n_cand;
  int cand_stride;
  float *token_logprob;
  float *cand_logprobs;
};

// Launchers (pz_kernels.cu).  Return cudaGetLastError() after the launch.
cudaError_t launch_logprob(const LogprobArgs &a, int dtype, cudaStream_t st);
cudaError_t launch_lm_head(const float *x, int B, int dim, const uint16_t *w, int V, float *logits,
                           int64_t ld, int num_sms, cudaStream_t st);
size_t logprob_smem_bytes(int V, int hcap);
cudaError_t launch_slice(const SliceArgs &a, int dtype, size_t smem,
                         cudaStream_t st);
size_t slice_smem_bytes(int kcap, int hts, int nstages, int V, int elem_bytes);
int slice_stages(int kcap, int hts);
int slice_ctas_per_sm_max(int kcap);
cudaError_t launch_full(const FullArgs &a, int dtype, int grid, size_t smem,
                        cudaStream_t st);
size_t full_smem_bytes(int V, int hcap);
__host__ __device__ size_t full_smem_fixed(int V, int hcap);
cudaError_t launch_merge(const MergeArgs &a, cudaStream_t st);
cudaError_t launch_temperature(float *x, int n, float T, cudaStream_t st);
cudaError_t launch_history_append(int32_t *ring, int B, int W, const int32_t *tokens,
                                  int32_t *counter, cudaStream_t st);
cudaError_t launch_rng_seed(unsigned long long *s, int B,
                            unsigned long long base,
                            const unsigned long long *seeds, cudaStream_t st);
cudaError_t set_kernel_attributes();
int max_dynamic_smem();

}  // namespace pz
