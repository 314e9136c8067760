// pz_capi.cu — the C ABI of include/pz_sampling.h: contexts, scratch, the
// reference's six legacy calls, the batched device API, and NCCL vocab
// sharding.  No torch types cross this boundary.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/pz_sampling.h"
#include "pz_kernels.cuh"

using pz::FullArgs;
using pz::MergeArgs;
using pz::SliceArgs;

namespace {

thread_local pz_status g_last_error = PZ_OK;
thread_local char g_detail[256] = "";

pz_status fail(pz_status s) {
  g_last_error = s;
  if (s == PZ_ERR_CUDA) {
    const cudaError_t e = cudaGetLastError();
    std::snprintf(g_detail, sizeof g_detail, "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  } else {
    std::snprintf(g_detail, sizeof g_detail, "%s", "");
  }
  return s;
}

// Records a failed CUDA call's error text and returns PZ_ERR_CUDA.
pz_status fail_cuda(cudaError_t e) {
  g_last_error = PZ_ERR_CUDA;
  std::snprintf(g_detail, sizeof g_detail, "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return PZ_ERR_CUDA;
}

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Restores the caller's current device on scope exit.
// (No device switch at all when the device is already current, so calls
// made during stream capture stay capture-safe.)
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  bool switched = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) return;
    if (prev == dev) {
      ok = true;
      return;
    }
    ok = switched = (cudaSetDevice(dev) == cudaSuccess);
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

// ---- kernel attributes, once per device ------------------------------------
// cudaFuncSetAttribute applies to the device that is current when it is
// called, so every device that runs the kernels needs its own call.
constexpr int kMaxDevices = 64;
std::mutex g_attr_mu;
bool g_attr_done[kMaxDevices];

cudaError_t ensure_kernel_attributes(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (g_attr_done[dev]) return cudaSuccess;
  const cudaError_t e = pz::set_kernel_attributes();
  if (e == cudaSuccess) g_attr_done[dev] = true;
  return e;
}

// ---- NCCL, loaded at run time (the process may already hold torch's) ----
struct NcclApi {
  bool loaded = false;
  void *h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
};
std::mutex g_nccl_mu;
NcclApi g_nccl;

bool load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.loaded) return true;
  const char *names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char *n : names) {
    g_nccl.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (g_nccl.h) break;
  }
  if (!g_nccl.h) return false;
#define PZ_SYM(field, name)                                                   \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(g_nccl.h, name)); \
  if (!g_nccl.field) return false;
  PZ_SYM(GetUniqueId, "ncclGetUniqueId")
  PZ_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
  PZ_SYM(AllGather, "ncclAllGather")
  PZ_SYM(CommFinalize, "ncclCommFinalize")
  PZ_SYM(CommDestroy, "ncclCommDestroy")
  PZ_SYM(CommAbort, "ncclCommAbort")
  PZ_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
  PZ_SYM(GroupStart, "ncclGroupStart")
  PZ_SYM(GroupEnd, "ncclGroupEnd")
#undef PZ_SYM
  g_nccl.loaded = true;
  return true;
}

}  // namespace

struct pz_sampler_ctx {
  int device = 0;
  int num_sms = 148;
  pz_ctx_limits lim{};
  int kcap_max = 1;
  int hcap_max = 0;
  int slices_cap = 0;
  size_t scratch = 0;
  std::vector<void *> allocs;
  unsigned long long *slice_keys = nullptr;
  int32_t *slice_cnt = nullptr;
  uint32_t *row_arrive = nullptr;
  uint32_t *row_flags = nullptr;
  unsigned long long *row_tau = nullptr;
  unsigned long long *row_best = nullptr;
  int32_t *full_rows = nullptr;
  int32_t *n_full = nullptr;      // [kFullClasses + 2]: full-row counts, claim counter, deferred rows
  int32_t *defer_rows = nullptr;  // [max_batch] rows for slice_long_kernel
  uint32_t *sort_a = nullptr;
  uint32_t *sort_b = nullptr;
  float *full_e = nullptr;
  int64_t sort_stride = 0;
  int64_t e_stride = 0;
  int full_grid = 0;
  // vocab sharding
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0;
  int nccl_timeout_ms = 60000;
  bool comm_failed = false;  // aborted after a timeout or an asynchronous error
  unsigned long long *emit = nullptr;
  unsigned long long *gathered = nullptr;
  // kernel timing: kProfEvents events per call, bracketing its phases
  // (slice_kernel, full_kernel, the allgather, merge_kernel)
  std::vector<cudaEvent_t> prof;
  std::vector<uint8_t> prof_short;  // per slot: only events 0 and 1 recorded
  int prof_used = 0;
  int prof_kernels = 0;

  template <typename T>
  bool alloc(T **p, size_t count) {
    void *q = nullptr;
    const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
    if (cudaMalloc(&q, bytes) != cudaSuccess) return false;
    if (cudaMemset(q, 0, bytes) != cudaSuccess) {
      cudaFree(q);
      return false;
    }
    allocs.push_back(q);
    scratch += bytes;
    *p = static_cast<T *>(q);
    return true;
  }
  void release() {
    for (void *q : allocs) cudaFree(q);
    allocs.clear();
    for (cudaEvent_t e : prof) cudaEventDestroy(e);
    prof.clear();
  }
};

namespace {

double now_ms() {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

// Aborts the context's communicator (it is unusable afterwards).
void abort_comm(pz_sampler_ctx *ctx) {
  if (ctx->comm && g_nccl.loaded) g_nccl.CommAbort(ctx->comm);
  ctx->comm = nullptr;
  ctx->comm_failed = true;
}

// Waits, by polling the communicator's asynchronous error, until a
// non-blocking NCCL call that returned `r` has finished.  Past the
// context's deadline the communicator is aborted and PZ_ERR_TIMEOUT comes
// back; an NCCL error aborts it too.
pz_status nccl_settle(pz_sampler_ctx *ctx, ncclResult_t r, double t0) {
  while (r == ncclInProgress) {
    if (now_ms() - t0 > ctx->nccl_timeout_ms) {
      abort_comm(ctx);
      g_last_error = PZ_ERR_TIMEOUT;
      std::snprintf(g_detail, sizeof g_detail, "NCCL call unfinished after %d ms; communicator aborted",
                    ctx->nccl_timeout_ms);
      return PZ_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (g_nccl.CommGetAsyncError(ctx->comm, &r) != ncclSuccess) r = ncclSystemError;
  }
  if (r != ncclSuccess) {
    abort_comm(ctx);
    g_last_error = PZ_ERR_NCCL;
    std::snprintf(g_detail, sizeof g_detail, "NCCL error %d; communicator aborted", static_cast<int>(r));
    return PZ_ERR_NCCL;
  }
  return PZ_OK;
}

}  // namespace

extern "C" {

const char *pz_status_str(pz_status s) {
  switch (s) {
    case PZ_OK: return "ok";
    case PZ_ERR_INVALID_ARGS: return "invalid arguments";
    case PZ_ERR_CUDA: return "CUDA runtime error";
    case PZ_ERR_OOM: return "out of memory";
    case PZ_ERR_NCCL: return "NCCL unavailable or failed";
    case PZ_ERR_TIMEOUT: return "timed out";
    case PZ_ERR_UNSUPPORTED: return "request beyond the context's limits";
    case PZ_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char *pz_version(void) { return "pz-sample-b200 0.1 (sm_100a)"; }

pz_status pz_last_error(void) { return g_last_error; }

const char *pz_last_error_detail(void) { return g_detail; }

pz_status pz_ctx_create(pz_sampler_ctx **out, int device,
                        const pz_ctx_limits *limits) {
  if (!out || !limits) return fail(PZ_ERR_INVALID_ARGS);
  *out = nullptr;
  const pz_ctx_limits L = *limits;
  if (L.max_batch <= 0 || L.max_vocab <= 0 || L.max_top_k < 0 ||
      L.max_top_k > PZ_TOP_K_MAX || L.max_history < 0 || L.max_history > 8192)
    return fail(PZ_ERR_INVALID_ARGS);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PZ_ERR_NO_DEVICE);
  if (device < 0 || device >= ndev) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  const cudaError_t attr_err = ensure_kernel_attributes(device);
  if (attr_err != cudaSuccess) return fail_cuda(attr_err);

  pz_sampler_ctx *c = new pz_sampler_ctx();
  c->device = device;
  c->lim = L;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  c->kcap_max = next_pow2(std::max(L.max_top_k, 1));
  c->hcap_max = L.max_history > 0 ? next_pow2(L.max_history) : 0;
  c->slices_cap = std::max(L.max_batch, 8192);
  // full_kernel: kFullCtasPerSm rows in flight per SM (no more CTAs than rows)
  c->full_grid = std::min(c->num_sms * pz::kFullCtasPerSm, L.max_batch);
  c->e_stride = (static_cast<int64_t>(L.max_vocab) + 63) / 64 * 64;
  c->sort_stride = 2 * static_cast<int64_t>(L.max_vocab);
  const int B = L.max_batch;
  bool ok = c->alloc(&c->slice_keys, static_cast<size_t>(c->slices_cap) * c->kcap_max) &&
            c->alloc(&c->slice_cnt, c->slices_cap) && c->alloc(&c->row_arrive, B) &&
            c->alloc(&c->row_flags, B) && c->alloc(&c->row_tau, B) && c->alloc(&c->row_best, B) &&
            c->alloc(&c->full_rows, static_cast<size_t>(B) * pz::kFullClasses) &&
            c->alloc(&c->n_full, pz::kFullClasses + 2) && c->alloc(&c->defer_rows, B) &&
            c->alloc(&c->sort_a, static_cast<size_t>(c->full_grid) * c->sort_stride) &&
            c->alloc(&c->sort_b, static_cast<size_t>(c->full_grid) * c->sort_stride) &&
            c->alloc(&c->full_e, static_cast<size_t>(c->full_grid) * c->e_stride);
  if (!ok) {
    c->release();
    delete c;
    return fail(PZ_ERR_OOM);
  }
  *out = c;
  return PZ_OK;
}

pz_status pz_ctx_destroy(pz_sampler_ctx *ctx) {
  if (!ctx) return PZ_OK;
  DeviceGuard g(ctx->device);
  if (ctx->comm && g_nccl.loaded) {
    // The communicator is non-blocking: finalize it (flushes its pending
    // collectives) within the deadline, else abort it; then free it.
    const double t0 = now_ms();
    ncclResult_t r = g_nccl.CommFinalize(ctx->comm);
    if (r == ncclSuccess || r == ncclInProgress) {
      if (nccl_settle(ctx, r, t0) == PZ_OK) g_nccl.CommDestroy(ctx->comm);
    } else {
      g_nccl.CommAbort(ctx->comm);
    }
    ctx->comm = nullptr;
  }
  cudaDeviceSynchronize();
  ctx->release();
  delete ctx;
  return PZ_OK;
}

size_t pz_ctx_scratch_bytes(const pz_sampler_ctx *ctx) { return ctx ? ctx->scratch : 0; }

void pz_row_shard(int B, int world, int rank, int *begin, int *count) {
  if (world <= 0 || rank < 0 || rank >= world || B < 0) {
    if (begin) *begin = 0;
    if (count) *count = 0;
    return;
  }
  const int base = B / world, rem = B % world;
  const int b = rank * base + std::min(rank, rem);
  if (begin) *begin = b;
  if (count) *count = base + (rank < rem ? 1 : 0);
}

// How rows are cut into CTAs.  With at least as many rows as the GPU has
// CTA slots (SMs x CTAs per SM at the kernel's occupancy), one CTA per row,
// and the CTA decides its row.  With fewer rows, every row is split into S
// slices, as many as fit the slots in one wave (B x S <= slots: a second,
// partial wave would cost a whole CTA life; config 2, 256 rows, ran 37.2 us
// at S = 3 and 33.4 us at S = 2): every slice pays a setup and an
// end-of-slice merge, and the last of a row's slices to finish merges the S
// lists and decides the row.  Launches of argmax rows only (list
// length 1) also split the rows of their last, partial wave (rows B1 on),
// so that this wave fills the GPU too; for list rows that was measured
// slower (a slice's short stream reaches a tight bound too late).  Slices
// of at least 128 KB of logits (every slice's setup, bound and list, and
// the last one's merge of S lists, cost more than its stream below that:
// one config-1 row drew in 47.4 us as 63 slices of 2048 columns and in
// 28.9 us as 4 slices of 32064), the split rows' lists within the context's
// scratch, and S lists of the launch's list length within the merge area
// (2048 keys).
// B200 HBM3e, bytes per ns (measured copy bandwidth), and the fraction of
// a CTA's life by which the slots of an SM are staggered.
constexpr double kHbmBytesPerNs = 6400.0;
constexpr double kStaggerFrac = 0.41;

// CTAs of slice_kernel per SM: its shared memory (dynamic, plus its static
// 1.3 KB and the 1 KB the hardware reserves per CTA) against the SM's 228 KB;
// its registers allow four (slice_long_kernel, for lists longer than 64: two).
static int slice_occupancy(size_t smem, int kcap) {
  const size_t per_sm = 228 * 1024;
  const int occ = static_cast<int>(per_sm / (smem + 2304));
  return std::max(1, std::min(occ, pz::slice_ctas_per_sm_max(kcap)));
}

static void choose_slices(const pz_sampler_ctx *c, int B, int V, int elem_bytes, int kcap,
                          size_t smem, int *B1_out, int *S_out, int *L_out) {
  const int occ = slice_occupancy(smem, kcap);
  const int slots = c->num_sms * occ;
  int B1 = 0, S = 1;
  if (B < slots) {
    S = slots / B;
  } else if (kcap == 1 && B % slots != 0) {
    B1 = B / slots * slots;
    S = slots / (B - B1);
  }
  // PZ_SLICES_PER_ROW: tuning override (every row in this many slices)
  static const int forced = [] {
    const char *e = std::getenv("PZ_SLICES_PER_ROW");
    return e ? std::atoi(e) : 0;
  }();
  if (forced > 0) {
    B1 = 0;
    S = forced;
  }
  const int min_cols = (128 * 1024) / elem_bytes;
  S = std::min(S, std::max(1, (V + min_cols - 1) / min_cols));
  S = std::min(S, std::max(1, c->slices_cap / std::max(B - B1, 1)));
  S = std::min(S, std::max(1, 2048 / std::max(kcap, 1)));
  S = std::max(S, 1);
  int L = (V + S - 1) / S;
  L = (L + 7) / 8 * 8;
  S = (V + L - 1) / L;
  if (S == 1) B1 = B;
  *B1_out = B1;
  *S_out = S;
  *L_out = L;
}

// Events per profiled call: start, after slice_kernel, after full_kernel,
// after the allgather, end (after merge_kernel).  Phases a call does not
// have are recorded back to back and time as zero.
constexpr int kProfEvents = 5;

// The next profiling slot of the context (nullptr when timing is off or
// its slots are used up).
static cudaEvent_t *next_prof_slot(pz_sampler_ctx *ctx, cudaStream_t st) {
  if ((ctx->prof_used + 1) * kProfEvents > static_cast<int>(ctx->prof.size())) return nullptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
    return nullptr;  // no timing events inside a captured graph
  cudaEvent_t *ev = &ctx->prof[ctx->prof_used * kProfEvents];
  ctx->prof_short[ctx->prof_used] = 0;
  ctx->prof_used++;
  return ev;
}

// ev_out: when not null, the call's profiling slot is handed back with its
// events 0..2 recorded and 3..4 left to the caller (vocab sharding records
// them around its allgather and merge).
static pz_status sample_impl(pz_sampler_ctx *ctx, const void *logits,
                             pz_dtype dtype, int B, int V, int64_t ld,
                             int64_t v_offset, int V_global,
                             const pz_sampler_config *cfg, const int32_t *hist,
                             const int32_t *hist_off,
                             unsigned long long *rng_state, int32_t *out,
                             const pz_batch_hints *hints,
                             const pz_batch_outputs *outputs, void *stream,
                             bool emit, cudaEvent_t **ev_out = nullptr) {
  if (ev_out) *ev_out = nullptr;
  if (!ctx || !logits || !cfg || B < 0 || V <= 0 || ld < V) return fail(PZ_ERR_INVALID_ARGS);
  if (dtype != PZ_DTYPE_F32 && dtype != PZ_DTYPE_BF16) return fail(PZ_ERR_INVALID_ARGS);
  if (!emit && (!rng_state || !out)) return fail(PZ_ERR_INVALID_ARGS);
  if ((hist == nullptr) != (hist_off == nullptr)) return fail(PZ_ERR_INVALID_ARGS);
  if (B == 0) return PZ_OK;
  if (B > ctx->lim.max_batch || V > ctx->lim.max_vocab) return fail(PZ_ERR_UNSUPPORTED);
  if (outputs && (outputs->cand_ids || outputs->cand_probs || outputs->cand_logprobs) &&
      outputs->cand_stride < 1)
    return fail(PZ_ERR_INVALID_ARGS);
  // list log-probabilities need the list: its ids and length
  if (outputs && outputs->cand_logprobs && (!outputs->cand_ids || !outputs->n_cand))
    return fail(PZ_ERR_INVALID_ARGS);
  int kmax = ctx->lim.max_top_k, hmax = ctx->lim.max_history, no_full = 0;
  if (hints) {
    if (hints->max_top_k > 0) kmax = std::min(kmax, hints->max_top_k);
    if (hints->max_history > 0) hmax = std::min(hmax, hints->max_history);
    no_full = hints->no_full_vocab ? 1 : 0;
  }
  if (outputs && (outputs->cand_ids || outputs->cand_probs) && outputs->cand_stride < kmax)
    return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  SliceArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.V = V;
  a.V_global = V_global;
  a.v_offset = v_offset;
  a.B = B;
  a.cfg = cfg;
  a.hist = hist;
  a.hist_off = hist_off;
  a.hcap = (hist != nullptr && hmax > 0) ? hmax : 0;
  a.hts = a.hcap > 0 ? next_pow2(2 * a.hcap) : 0;
  a.hshift = 32;
  for (int t = a.hts; t > 1; t >>= 1) a.hshift--;
  a.mode_emit = emit ? 1 : 0;
  a.no_full_vocab = no_full;
  a.slice_keys = ctx->slice_keys;
  a.slice_cnt = ctx->slice_cnt;
  a.row_arrive = ctx->row_arrive;
  a.row_flags = ctx->row_flags;
  a.row_tau = ctx->row_tau;
  a.row_best = ctx->row_best;
  a.full_rows = ctx->full_rows;
  a.n_full = ctx->n_full;
  a.full_stride = ctx->lim.max_batch;
  a.emit_keys = ctx->emit;
  a.rng = rng_state;
  a.out = out;
  if (outputs) {
    a.cand_ids = outputs->cand_ids;
    a.cand_probs = outputs->cand_probs;
    a.n_cand = outputs->n_cand;
    a.row_status = outputs->row_status;
    a.cand_stride = outputs->cand_stride;
  }
  // Sizes launch x for lists up to km: its list capacity, shared memory,
  // row split (whole: one CTA per row, no split) and first-wave stagger.
  auto size_launch = [&](pz::SliceArgs &x, int km, bool whole, size_t *smem_out) -> bool {
    x.kcap = next_pow2(std::max(km, 1));
    x.kmax = std::max(km, 1);
    x.nstages = pz::slice_stages(x.kcap, x.hts);
    const size_t sm = pz::slice_smem_bytes(x.kcap, x.hts, x.nstages, x.V, dtype == PZ_DTYPE_BF16 ? 2 : 4);
    if (whole) {
      x.B1 = B;
      x.S = 1;
      x.L = V;
    } else {
      choose_slices(ctx, B, V, dtype == PZ_DTYPE_BF16 ? 2 : 4, x.kcap, sm, &x.B1, &x.S, &x.L);
    }
    if (sm > static_cast<size_t>(pz::max_dynamic_smem())) return false;
    // Stagger of the first wave's list-row CTAs.  A wave's CTAs start
    // together, stream together and then all run their end-of-row work with
    // HBM idle; starting the CTA slots of an SM a fraction of a CTA's life
    // apart keeps some of them streaming at any time.  A CTA's life is about
    // its bytes at its share of HBM (CTAs in flight x bytes / bandwidth).
    const int occ = slice_occupancy(sm, x.kcap);
    const int slots = ctx->num_sms * occ;
    const double cta_bytes = static_cast<double>(x.S == 1 ? V : x.L) * (dtype == PZ_DTYPE_BF16 ? 2 : 4);
    // (measured best: the life at three CTAs per SM, shared by the slots)
    const double life_ns = cta_bytes * std::min(ctx->num_sms * 3, B * x.S) / kHbmBytesPerNs * 3.0 / occ;
    static const int forced = [] {
      const char *e = std::getenv("PZ_STAGGER_NS");  // tuning override
      return e ? std::atoi(e) : -1;
    }();
    x.stagger_ns = forced >= 0 ? forced : static_cast<int>(kStaggerFrac * life_ns);
    x.stagger_ctas = slots;
    x.stagger_occ = occ;
    *smem_out = sm;
    return true;
  };
  // A large batch whose lists may be longer than kTQK runs in two launches:
  // slice_kernel (up to four CTAs per SM) samples every row but those, which
  // it files for slice_long_kernel (two per SM, the fine sketch).
  const bool defer = !emit && kmax > pz::kTQK && B >= 4 * ctx->num_sms;
  size_t smem = 0, smem2 = 0;
  pz::SliceArgs a2{};
  if (defer) {
    a.defer_kmax = kmax;
    a.defer_rows = ctx->defer_rows;
    a.n_defer = ctx->n_full + pz::kFullClasses + 1;
    a2 = a;
    a2.defer_kmax = 0;
    a2.deferred = 1;
    if (!size_launch(a2, kmax, true, &smem2) || !size_launch(a, pz::kTQK, true, &smem))
      return fail(PZ_ERR_UNSUPPORTED);
  } else if (!size_launch(a, kmax, false, &smem)) {
    return fail(PZ_ERR_UNSUPPORTED);
  }
  const bool full_pass = !emit && !no_full;
  if ((full_pass || defer) &&
      cudaMemsetAsync(ctx->n_full, 0, sizeof(int32_t) * (pz::kFullClasses + 2), st) != cudaSuccess)
    return fail(PZ_ERR_CUDA);
  cudaEvent_t *ev = next_prof_slot(ctx, st);
  if (ev) cudaEventRecord(ev[0], st);
  cudaError_t ce = pz::launch_slice(a, dtype, smem, st);
  if (ce != cudaSuccess) return fail_cuda(ce);
  int kernels = 1;  // slice_kernel decides every row itself (but deferred ones)
  if (defer) {
    ce = pz::launch_slice(a2, dtype, smem2, st);
    if (ce != cudaSuccess) return fail_cuda(ce);
    kernels++;
  }
  if (ev) cudaEventRecord(ev[1], st);
  if (full_pass) {
    FullArgs f{};
    f.logits = logits;
    f.ld = ld;
    f.V = V;
    f.B = B;
    f.cfg = cfg;
    f.hist = hist;
    f.hist_off = hist_off;
    f.hcap = a.hcap > 0 ? next_pow2(a.hcap) : 0;
    f.row_best = ctx->row_best;
    f.row_flags = ctx->row_flags;
    f.full_rows = ctx->full_rows;
    f.n_full = ctx->n_full;
    f.full_stride = ctx->lim.max_batch;
    f.sort_a = ctx->sort_a;
    f.sort_b = ctx->sort_b;
    f.sort_stride = ctx->sort_stride;
    f.escr = ctx->full_e;
    f.e_stride = ctx->e_stride;
    f.rng = rng_state;
    f.out = out;
    const size_t fsmem = pz::full_smem_bytes(V, f.hcap);
    if (fsmem > static_cast<size_t>(pz::max_dynamic_smem())) return fail(PZ_ERR_UNSUPPORTED);
    const size_t fixed = (pz::full_smem_fixed(V, f.hcap) + 15) / 16 * 16;
    f.smem_sort_cap = static_cast<int>((fsmem - fixed) / 16);
    const int grid = std::min(ctx->full_grid, B);
    ce = pz::launch_full(f, dtype, grid, fsmem, st);
    if (ce != cudaSuccess) return fail_cuda(ce);
    kernels++;
  }
  if (!emit && outputs && (outputs->token_logprob || outputs->cand_logprobs)) {
    pz::LogprobArgs l{};
    l.logits = logits;
    l.ld = ld;
    l.V = V;
    l.B = B;
    l.cfg = cfg;
    l.hist = hist;
    l.hist_off = hist_off;
    l.hcap = a.hcap > 0 ? next_pow2(a.hcap) : 0;
    l.tokens = out;
    l.cand_ids = outputs->cand_ids;
    l.n_cand = outputs->n_cand;
    l.cand_stride = outputs->cand_stride;
    l.token_logprob = outputs->token_logprob;
    l.cand_logprobs = outputs->cand_logprobs;
    if (pz::logprob_smem_bytes(V, l.hcap) > static_cast<size_t>(pz::max_dynamic_smem()))
      return fail(PZ_ERR_UNSUPPORTED);
    ce = pz::launch_logprob(l, dtype, st);
    if (ce != cudaSuccess) return fail_cuda(ce);
    kernels++;
  }
  if (ev && kernels == 1 && !ev_out) {
    // slice_kernel alone: its two events are the call's only ones (fewer
    // commands between the launches of back-to-back calls)
    ctx->prof_short[(ev - ctx->prof.data()) / kProfEvents] = 1;
    ctx->prof_kernels += kernels;
  } else if (ev) {
    cudaEventRecord(ev[2], st);
    ctx->prof_kernels += kernels;
    if (ev_out) {
      *ev_out = ev;
    } else {
      cudaEventRecord(ev[3], st);
      cudaEventRecord(ev[4], st);
    }
  }
  return PZ_OK;
}

pz_status pz_sample_batch(pz_sampler_ctx *ctx, const void *logits,
                          pz_dtype dtype, int B, int V, int64_t ld,
                          const pz_sampler_config *cfg, const int32_t *hist,
                          const int32_t *hist_off,
                          unsigned long long *rng_state, int32_t *out_tokens,
                          const pz_batch_hints *hints,
                          const pz_batch_outputs *outputs, void *stream) {
  return sample_impl(ctx, logits, dtype, B, V, ld, 0, V, cfg, hist, hist_off,
                     rng_state, out_tokens, hints, outputs, stream, false);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// pz_sample_batch_static: the batched sampler with its scratch carved out of
// one fixed device array (per device, zero at module load) instead of a
// context's allocations.  Layout (bytes):
//   slice lists  kStaticSlices x PZ_STATIC_MAX_TOP_K u64   (split rows x S <= kStaticSlices)
//   slice counts kStaticSlices int32
//   row words    row_tau, row_best (u64), row_arrive, row_flags, full_rows
//                (32-bit), PZ_STATIC_MAX_BATCH each, then the n_full counter.
// Every word this path reads is written earlier in the same call (slice
// counts and lists by every slice CTA, row flags by slice 0), except the
// split rows' arrival counters, which start at zero with the array and are
// put back to zero by each row's last slice; the full-vocabulary counter,
// which must also start at zero, is never touched because such rows are
// refused.
// ---------------------------------------------------------------------------
namespace {

constexpr int kStaticSlices = 4096;
constexpr size_t kStaticOffCnt = sizeof(unsigned long long) * kStaticSlices * PZ_STATIC_MAX_TOP_K;
constexpr size_t kStaticOffTau = kStaticOffCnt + sizeof(int32_t) * kStaticSlices;
constexpr size_t kStaticOffBest = kStaticOffTau + sizeof(unsigned long long) * PZ_STATIC_MAX_BATCH;
constexpr size_t kStaticOffArrive = kStaticOffBest + sizeof(unsigned long long) * PZ_STATIC_MAX_BATCH;
constexpr size_t kStaticOffFlags = kStaticOffArrive + sizeof(uint32_t) * PZ_STATIC_MAX_BATCH;
constexpr size_t kStaticOffFull = kStaticOffFlags + sizeof(uint32_t) * PZ_STATIC_MAX_BATCH;
constexpr size_t kStaticOffNFull = kStaticOffFull + sizeof(int32_t) * PZ_STATIC_MAX_BATCH;
constexpr size_t kStaticBytes = kStaticOffNFull + 256;
static_assert(kStaticOffTau % 8 == 0 && kStaticOffArrive % 8 == 0, "u64 rows must stay aligned");

static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
std::atomic<unsigned char *> g_static_base[kStaticMaxDevices];
int g_static_sms[kStaticMaxDevices];

pz_status fail_detail(pz_status s, const char *msg) {
  g_last_error = s;
  std::snprintf(g_detail, sizeof g_detail, "%s", msg);
  return s;
}

// The array's address on device `dev` (the current device), looked up once.
pz_status static_scratch(int dev, unsigned char **base, int *num_sms) {
  unsigned char *p = g_static_base[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lk(g_static_mu);
    p = g_static_base[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void *q = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&q, g_static_scratch);
      if (e != cudaSuccess) return fail_cuda(e);
      e = ensure_kernel_attributes(dev);
      if (e != cudaSuccess) return fail_cuda(e);
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return fail_cuda(e);
      g_static_sms[dev] = sms;
      p = static_cast<unsigned char *>(q);
      g_static_base[dev].store(p, std::memory_order_release);
    }
  }
  *base = p;
  *num_sms = g_static_sms[dev];
  return PZ_OK;
}

}  // namespace

extern "C" {

pz_status pz_sample_batch_static(const void *logits, pz_dtype dtype, int B,
                                 int V, int64_t ld,
                                 const pz_sampler_config *cfg,
                                 const int32_t *hist, const int32_t *hist_off,
                                 unsigned long long *rng_state,
                                 int32_t *out_tokens,
                                 const pz_batch_outputs *outputs,
                                 void *stream) {
  if (B > PZ_STATIC_MAX_BATCH || V > PZ_STATIC_MAX_VOCAB) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "pz_sample_batch_static: B=%d V=%d beyond the static scratch's limits "
                  "(B <= %d, V <= %d)", B, V, PZ_STATIC_MAX_BATCH, PZ_STATIC_MAX_VOCAB);
    return fail_detail(PZ_ERR_UNSUPPORTED, msg);
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(PZ_ERR_NO_DEVICE);
  if (dev < 0 || dev >= kStaticMaxDevices) return fail(PZ_ERR_UNSUPPORTED);
  unsigned char *base = nullptr;
  int sms = 0;
  const pz_status s = static_scratch(dev, &base, &sms);
  if (s != PZ_OK) return s;
  // A context that owns nothing: its scratch pointers name the static array.
  pz_sampler_ctx view;
  view.device = dev;
  view.num_sms = sms;
  view.lim = pz_ctx_limits{PZ_STATIC_MAX_BATCH, PZ_STATIC_MAX_VOCAB, PZ_STATIC_MAX_TOP_K,
                           PZ_STATIC_MAX_HISTORY};
  view.kcap_max = PZ_STATIC_MAX_TOP_K;
  view.hcap_max = PZ_STATIC_MAX_HISTORY;
  view.slices_cap = kStaticSlices;
  view.slice_keys = reinterpret_cast<unsigned long long *>(base);
  view.slice_cnt = reinterpret_cast<int32_t *>(base + kStaticOffCnt);
  view.row_tau = reinterpret_cast<unsigned long long *>(base + kStaticOffTau);
  view.row_best = reinterpret_cast<unsigned long long *>(base + kStaticOffBest);
  view.row_arrive = reinterpret_cast<uint32_t *>(base + kStaticOffArrive);
  view.row_flags = reinterpret_cast<uint32_t *>(base + kStaticOffFlags);
  view.full_rows = reinterpret_cast<int32_t *>(base + kStaticOffFull);
  view.n_full = reinterpret_cast<int32_t *>(base + kStaticOffNFull);
  const pz_batch_hints h{PZ_STATIC_MAX_TOP_K, PZ_STATIC_MAX_HISTORY, 1, 0};
  return sample_impl(&view, logits, dtype, B, V, ld, 0, V, cfg, hist, hist_off, rng_state,
                     out_tokens, &h, outputs, stream, false);
}

pz_status pz_ctx_profile(pz_sampler_ctx *ctx, int n_calls) {
  if (!ctx || n_calls < 0) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  for (cudaEvent_t e : ctx->prof) cudaEventDestroy(e);
  ctx->prof.clear();
  ctx->prof_short.assign(static_cast<size_t>(n_calls), 0);
  ctx->prof_used = 0;
  ctx->prof_kernels = 0;
  for (int i = 0; i < kProfEvents * n_calls; i++) {
    cudaEvent_t e;
    const cudaError_t ce = cudaEventCreate(&e);
    if (ce != cudaSuccess) return fail_cuda(ce);
    ctx->prof.push_back(e);
  }
  return PZ_OK;
}

pz_status pz_ctx_profile_phases(pz_sampler_ctx *ctx, double *phase_ms, int *calls,
                                int *kernels) {
  if (!ctx) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  double sum[kProfEvents - 1] = {0.0, 0.0, 0.0, 0.0};
  for (int i = 0; i < ctx->prof_used; i++) {
    cudaEvent_t *ev = &ctx->prof[i * kProfEvents];
    const bool shrt = ctx->prof_short[i] != 0;
    cudaError_t ce = cudaEventSynchronize(ev[shrt ? 1 : kProfEvents - 1]);
    if (ce != cudaSuccess) return fail_cuda(ce);
    for (int j = 0; j + 1 < (shrt ? 2 : kProfEvents); j++) {
      float t = 0.0f;
      ce = cudaEventElapsedTime(&t, ev[j], ev[j + 1]);
      if (ce != cudaSuccess) return fail_cuda(ce);
      sum[j] += t;
    }
  }
  if (phase_ms)
    for (int j = 0; j + 1 < kProfEvents; j++) phase_ms[j] = sum[j];
  if (calls) *calls = ctx->prof_used;
  if (kernels) *kernels = ctx->prof_kernels;
  ctx->prof_used = 0;
  ctx->prof_kernels = 0;
  return PZ_OK;
}

pz_status pz_ctx_profile_read(pz_sampler_ctx *ctx, double *slice_ms, double *rest_ms,
                              int *calls, int *kernels) {
  double ph[kProfEvents - 1];
  const pz_status s = pz_ctx_profile_phases(ctx, ph, calls, kernels);
  if (s != PZ_OK) return s;
  if (slice_ms) *slice_ms = ph[0];
  if (rest_ms) *rest_ms = ph[1] + ph[2] + ph[3];
  return PZ_OK;
}

pz_status pz_rng_seed_batch(unsigned long long *rng_state, int B,
                            unsigned long long seed_base,
                            const unsigned long long *seeds, void *stream) {
  if (!rng_state || B < 0) return fail(PZ_ERR_INVALID_ARGS);
  if (B == 0) return PZ_OK;
  if (pz::launch_rng_seed(rng_state, B, seed_base, seeds,
                          static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return fail(PZ_ERR_CUDA);
  return PZ_OK;
}

pz_status pz_lm_head_logits(pz_sampler_ctx *ctx, const float *hidden, int B, int dim,
                            const uint16_t *w_cls, int V, float *logits, int64_t ld, void *stream) {
  if (!ctx || !hidden || !w_cls || !logits || B <= 0 || dim <= 0 || V <= 0 || ld < V || dim % 8 != 0)
    return fail(PZ_ERR_INVALID_ARGS);
  if (sizeof(float) * 8 * static_cast<size_t>(dim) > static_cast<size_t>(pz::max_dynamic_smem()))
    return fail(PZ_ERR_UNSUPPORTED);
  if ((reinterpret_cast<uintptr_t>(w_cls) & 15u) != 0 || (reinterpret_cast<uintptr_t>(hidden) & 15u) != 0)
    return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  const cudaError_t e = pz::launch_lm_head(hidden, B, dim, w_cls, V, logits, ld, ctx->num_sms,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PZ_OK : fail_cuda(e);
}

pz_status pz_sample_from_hidden(pz_sampler_ctx *ctx, const float *hidden, int B, int dim,
                                const uint16_t *w_cls, int V, float *logits, int64_t ld,
                                const pz_sampler_config *cfg, const int32_t *hist,
                                const int32_t *hist_off, unsigned long long *rng_state,
                                int32_t *out_tokens, const pz_batch_hints *hints,
                                const pz_batch_outputs *outputs, void *stream) {
  const pz_status s = pz_lm_head_logits(ctx, hidden, B, dim, w_cls, V, logits, ld, stream);
  if (s != PZ_OK) return s;
  return pz_sample_batch(ctx, logits, PZ_DTYPE_F32, B, V, ld, cfg, hist, hist_off, rng_state, out_tokens,
                         hints, outputs, stream);
}

pz_status pz_history_append(int32_t *hist_ring, int B, int W, const int32_t *tokens,
                            int32_t *counter, void *stream) {
  if (!hist_ring || !tokens || !counter || B < 0 || W <= 0) return fail(PZ_ERR_INVALID_ARGS);
  if (B == 0) return PZ_OK;
  const cudaError_t e =
      pz::launch_history_append(hist_ring, B, W, tokens, counter, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PZ_OK : fail_cuda(e);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The generate loop's sampling step as one CUDA graph (reference
// src/transformer/generate.c:137-170, per step: sample, then the sampled id
// joins the penalty window), with the RNG states and the window on the
// device from one step to the next.
// ---------------------------------------------------------------------------
struct pz_decode_step {
  pz_sampler_ctx *ctx = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int32_t *counter = nullptr;   // steps taken (device)
  int32_t *hist_off = nullptr;  // r * W (device)
};

namespace {
__global__ void ring_offsets_kernel(int32_t *off, int B, int W) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r <= B) off[r] = r * W;
}
void step_release(pz_decode_step *s) {
  if (s->exec) cudaGraphExecDestroy(s->exec);
  if (s->graph) cudaGraphDestroy(s->graph);
  if (s->counter) cudaFree(s->counter);
  if (s->hist_off) cudaFree(s->hist_off);
  delete s;
}
}  // namespace

extern "C" {

pz_status pz_decode_step_create(pz_sampler_ctx *ctx, const void *logits, pz_dtype dtype, int B, int V,
                                int64_t ld, const pz_sampler_config *cfg, int32_t *hist_ring, int W,
                                unsigned long long *rng_state, int32_t *out_tokens,
                                const pz_batch_hints *hints, pz_decode_step **step) {
  if (!ctx || !step || !logits || !cfg || !rng_state || !out_tokens || B <= 0 || V <= 0 ||
      (hist_ring != nullptr) != (W > 0) || W < 0)
    return fail(PZ_ERR_INVALID_ARGS);
  *step = nullptr;
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  pz_decode_step *s = new pz_decode_step();
  s->ctx = ctx;
  cudaStream_t cs = nullptr;
  cudaError_t e = cudaMalloc(&s->counter, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(s->counter, 0, sizeof(int32_t));
  if (e == cudaSuccess && hist_ring) {
    e = cudaMalloc(&s->hist_off, sizeof(int32_t) * (B + 1));
    if (e == cudaSuccess) {
      ring_offsets_kernel<<<(B + 256) / 256, 256>>>(s->hist_off, B, W);
      e = cudaGetLastError();
    }
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    step_release(s);
    return fail_cuda(e);
  }
  // one sampling call and the window update, recorded as a graph
  e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
  pz_status ps = PZ_OK;
  if (e == cudaSuccess) {
    ps = sample_impl(ctx, logits, dtype, B, V, ld, 0, V, cfg, hist_ring, s->hist_off, rng_state,
                     out_tokens, hints, nullptr, cs, false);
    if (ps == PZ_OK && hist_ring)
      e = pz::launch_history_append(hist_ring, B, W, out_tokens, s->counter, cs);
    else if (ps == PZ_OK)
      e = pz::launch_history_append(out_tokens, 0, 1, out_tokens, s->counter, cs);  // the step count only
    const cudaError_t e2 = cudaStreamEndCapture(cs, &s->graph);
    if (e == cudaSuccess) e = e2;
  }
  if (ps == PZ_OK && e == cudaSuccess) e = cudaGraphInstantiate(&s->exec, s->graph, 0);
  cudaStreamDestroy(cs);
  if (ps != PZ_OK || e != cudaSuccess) {
    step_release(s);
    return ps != PZ_OK ? ps : fail_cuda(e);
  }
  *step = s;
  return PZ_OK;
}

pz_status pz_decode_step_launch(pz_decode_step *step, void *stream) {
  if (!step) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(step->ctx->device);
  const cudaError_t e = cudaGraphLaunch(step->exec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PZ_OK : fail_cuda(e);
}

pz_status pz_decode_step_count(const pz_decode_step *step, int32_t *steps) {
  if (!step || !steps) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(step->ctx->device);
  const cudaError_t e = cudaMemcpy(steps, step->counter, sizeof(int32_t), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? PZ_OK : fail_cuda(e);
}

pz_status pz_decode_step_destroy(pz_decode_step *step) {
  if (!step) return PZ_OK;
  DeviceGuard g(step->ctx->device);
  cudaDeviceSynchronize();
  step_release(step);
  return PZ_OK;
}

// ---------------------------------------------------------------------------
// vocab sharding
// ---------------------------------------------------------------------------
pz_status pz_nccl_get_unique_id(void *id_out, size_t id_bytes) {
  if (!id_out || id_bytes < sizeof(ncclUniqueId)) return fail(PZ_ERR_INVALID_ARGS);
  if (!load_nccl()) return fail(PZ_ERR_NCCL);
  ncclUniqueId id;
  if (g_nccl.GetUniqueId(&id) != ncclSuccess) return fail(PZ_ERR_NCCL);
  std::memcpy(id_out, &id, sizeof id);
  return PZ_OK;
}

pz_status pz_ctx_init_nccl_timeout(pz_sampler_ctx *ctx, int world, int rank,
                                   const void *unique_id, size_t id_bytes,
                                   int timeout_ms) {
  if (!ctx || !unique_id || id_bytes < sizeof(ncclUniqueId) || world < 1 ||
      rank < 0 || rank >= world || timeout_ms <= 0 || ctx->comm)
    return fail(PZ_ERR_INVALID_ARGS);
  if (!load_nccl()) return fail(PZ_ERR_NCCL);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  const size_t per_rank = static_cast<size_t>(ctx->lim.max_batch) * (ctx->kcap_max + 1);
  if (!ctx->emit && !ctx->alloc(&ctx->emit, per_rank)) return fail(PZ_ERR_OOM);
  if (!ctx->gathered && !ctx->alloc(&ctx->gathered, per_rank * world)) return fail(PZ_ERR_OOM);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  // Non-blocking communicator: init and every collective return at once,
  // and their progress is polled against the deadline.
  ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
  conf.blocking = 0;
  ncclComm_t comm = nullptr;
  ctx->nccl_timeout_ms = timeout_ms;
  ctx->comm_failed = false;
  const double t0 = now_ms();
  const ncclResult_t r = g_nccl.CommInitRankConfig(&comm, world, id, rank, &conf);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) g_nccl.CommAbort(comm);
    return fail(PZ_ERR_NCCL);
  }
  ctx->comm = comm;
  const pz_status s = nccl_settle(ctx, r, t0);
  if (s != PZ_OK) return s;
  ctx->world = world;
  ctx->rank = rank;
  return PZ_OK;
}

pz_status pz_ctx_init_nccl(pz_sampler_ctx *ctx, int world, int rank,
                           const void *unique_id, size_t id_bytes) {
  return pz_ctx_init_nccl_timeout(ctx, world, rank, unique_id, id_bytes, 60000);
}

pz_status pz_ctx_wait(pz_sampler_ctx *ctx, void *stream, int timeout_ms) {
  if (!ctx || timeout_ms <= 0) return fail(PZ_ERR_INVALID_ARGS);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const double t0 = now_ms();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return PZ_OK;
    if (q != cudaErrorNotReady) return fail_cuda(q);
    if (ctx->comm) {
      ncclResult_t ar = ncclSuccess;
      if (g_nccl.CommGetAsyncError(ctx->comm, &ar) != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
        abort_comm(ctx);
        g_last_error = PZ_ERR_NCCL;
        std::snprintf(g_detail, sizeof g_detail, "NCCL asynchronous error %d; communicator aborted",
                      static_cast<int>(ar));
        return PZ_ERR_NCCL;
      }
    }
    if (now_ms() - t0 > timeout_ms) {
      // aborting the communicator ends its collectives still in flight
      if (ctx->comm) abort_comm(ctx);
      g_last_error = PZ_ERR_TIMEOUT;
      std::snprintf(g_detail, sizeof g_detail, "stream unfinished after %d ms", timeout_ms);
      return PZ_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

pz_status pz_ctx_abort_nccl(pz_sampler_ctx *ctx) {
  if (!ctx) return fail(PZ_ERR_INVALID_ARGS);
  if (ctx->comm) {
    DeviceGuard g(ctx->device);
    abort_comm(ctx);
  }
  return PZ_OK;
}

}  // extern "C"

namespace {

// The three steps of a vocab-sharded call.  (1) The local pass: this
// slice's lists, written to ctx->emit as [B][kcap+1] (counts in slot kcap).
pz_status vocab_check(const pz_sampler_ctx *ctx, int V_local, int64_t v_offset, int V_global,
                      unsigned long long *rng_state, int32_t *out_tokens,
                      const pz_batch_outputs *outputs) {
  if (!ctx || !rng_state || !out_tokens) return fail(PZ_ERR_INVALID_ARGS);
  if (!ctx->comm) return fail(ctx->comm_failed ? PZ_ERR_NCCL : PZ_ERR_INVALID_ARGS);
  if (outputs && (outputs->token_logprob || outputs->cand_logprobs)) return fail(PZ_ERR_UNSUPPORTED);
  if (outputs && (outputs->cand_ids || outputs->cand_probs) &&
      outputs->cand_stride < std::max(ctx->lim.max_top_k, 1))
    return fail(PZ_ERR_INVALID_ARGS);
  if (V_local <= 0 || V_global < V_local || v_offset < 0 || v_offset + V_local > V_global)
    return fail(PZ_ERR_INVALID_ARGS);
  return PZ_OK;
}

pz_status vocab_local(pz_sampler_ctx *ctx, const void *logits_slice, pz_dtype dtype, int B, int V_local,
                      int64_t ld, int64_t v_offset, int V_global, const pz_sampler_config *cfg,
                      const int32_t *hist, const int32_t *hist_off, void *stream, cudaEvent_t **ev) {
  pz_batch_hints h{};
  h.no_full_vocab = 1;
  return sample_impl(ctx, logits_slice, dtype, B, V_local, ld, v_offset, V_global, cfg, hist, hist_off,
                     nullptr, nullptr, &h, nullptr, stream, true, ev);
}

size_t vocab_block_words(const pz_sampler_ctx *ctx, int B) {
  return static_cast<size_t>(B) * (next_pow2(std::max(ctx->lim.max_top_k, 1)) + 1);
}

// (2) ONE allgather of every rank's list block (enqueued; in a group when
// one thread drives several communicators).
ncclResult_t vocab_allgather(pz_sampler_ctx *ctx, int B, void *stream) {
  return g_nccl.AllGather(ctx->emit, ctx->gathered, vocab_block_words(ctx, B), ncclUint64, ctx->comm,
                          static_cast<cudaStream_t>(stream));
}

// (3) The merge of the G blocks and the draw.
pz_status vocab_merge(pz_sampler_ctx *ctx, int B, int V_global, const pz_sampler_config *cfg,
                      unsigned long long *rng_state, int32_t *out_tokens, const pz_batch_outputs *outputs,
                      void *stream, cudaEvent_t *ev) {
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(PZ_ERR_CUDA);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (ev) cudaEventRecord(ev[3], st);
  MergeArgs m{};
  m.gathered = ctx->gathered;
  m.G = ctx->world;
  m.B = B;
  m.kcap = next_pow2(std::max(ctx->lim.max_top_k, 1));
  m.kmax = std::max(ctx->lim.max_top_k, 1);
  m.V_global = V_global;
  m.cfg = cfg;
  m.rng = rng_state;
  m.out = out_tokens;
  if (outputs) {
    m.cand_ids = outputs->cand_ids;
    m.cand_probs = outputs->cand_probs;
    m.n_cand = outputs->n_cand;
    m.row_status = outputs->row_status;
    m.cand_stride = outputs->cand_stride;
  }
  const cudaError_t ce = pz::launch_merge(m, st);
  if (ce != cudaSuccess) return fail_cuda(ce);
  if (ev) {
    cudaEventRecord(ev[4], st);
    ctx->prof_kernels += 1;
  }
  return PZ_OK;
}

}  // namespace

extern "C" {

pz_status pz_sample_batch_vocab_sharded(
    pz_sampler_ctx *ctx, const void *logits_slice, pz_dtype dtype, int B,
    int V_local, int64_t ld, int64_t v_offset, int V_global,
    const pz_sampler_config *cfg, const int32_t *hist, const int32_t *hist_off,
    unsigned long long *rng_state, int32_t *out_tokens,
    const pz_batch_outputs *outputs, void *stream) {
  pz_status s = vocab_check(ctx, V_local, v_offset, V_global, rng_state, out_tokens, outputs);
  if (s != PZ_OK) return s;
  cudaEvent_t *ev = nullptr;
  s = vocab_local(ctx, logits_slice, dtype, B, V_local, ld, v_offset, V_global, cfg, hist, hist_off, stream, &ev);
  if (s != PZ_OK) return s;
  {
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(PZ_ERR_CUDA);
    const double t0 = now_ms();
    const ncclResult_t r = vocab_allgather(ctx, B, stream);
    if (r != ncclSuccess && r != ncclInProgress) {
      abort_comm(ctx);
      return fail(PZ_ERR_NCCL);
    }
    s = nccl_settle(ctx, r, t0);  // the call is enqueued (not finished) when this returns
    if (s != PZ_OK) return s;
  }
  return vocab_merge(ctx, B, V_global, cfg, rng_state, out_tokens, outputs, stream, ev);
}

// ---------------------------------------------------------------------------
// Several devices from one host thread
// ---------------------------------------------------------------------------
pz_status pz_multi_init_nccl(pz_sampler_ctx *const *ctxs, int n, int timeout_ms) {
  if (!ctxs || n < 1 || n > kMaxDevices || timeout_ms <= 0) return fail(PZ_ERR_INVALID_ARGS);
  for (int i = 0; i < n; i++) {
    if (!ctxs[i] || ctxs[i]->comm) return fail(PZ_ERR_INVALID_ARGS);
    for (int j = 0; j < i; j++)
      if (ctxs[j]->device == ctxs[i]->device) return fail(PZ_ERR_INVALID_ARGS);
  }
  if (!load_nccl()) return fail(PZ_ERR_NCCL);
  ncclUniqueId id;
  if (g_nccl.GetUniqueId(&id) != ncclSuccess) return fail(PZ_ERR_NCCL);
  for (int i = 0; i < n; i++) {
    pz_sampler_ctx *c = ctxs[i];
    DeviceGuard g(c->device);
    if (!g.ok) return fail(PZ_ERR_CUDA);
    const size_t per_rank = static_cast<size_t>(c->lim.max_batch) * (c->kcap_max + 1);
    if (!c->emit && !c->alloc(&c->emit, per_rank)) return fail(PZ_ERR_OOM);
    if (!c->gathered && !c->alloc(&c->gathered, per_rank * n)) return fail(PZ_ERR_OOM);
    c->nccl_timeout_ms = timeout_ms;
    c->comm_failed = false;
  }
  // one thread creates every rank's communicator: a group, so that the
  // ranks' set-ups do not wait for one another
  const double t0 = now_ms();
  std::vector<ncclComm_t> comms(n, nullptr);
  ncclResult_t r = g_nccl.GroupStart();
  for (int i = 0; i < n && r == ncclSuccess; i++) {
    DeviceGuard g(ctxs[i]->device);
    ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
    conf.blocking = 0;
    const ncclResult_t ri = g_nccl.CommInitRankConfig(&comms[i], n, id, i, &conf);
    if (ri != ncclSuccess && ri != ncclInProgress) r = ri;
  }
  const ncclResult_t re = g_nccl.GroupEnd();
  if (r == ncclSuccess && re != ncclSuccess && re != ncclInProgress) r = re;
  if (r != ncclSuccess) {
    for (int i = 0; i < n; i++)
      if (comms[i]) g_nccl.CommAbort(comms[i]);
    return fail(PZ_ERR_NCCL);
  }
  pz_status s = PZ_OK;
  for (int i = 0; i < n; i++) {
    ctxs[i]->comm = comms[i];
    ctxs[i]->world = n;
    ctxs[i]->rank = i;
  }
  for (int i = 0; i < n && s == PZ_OK; i++) {
    DeviceGuard g(ctxs[i]->device);
    s = nccl_settle(ctxs[i], ncclInProgress, t0);
  }
  if (s != PZ_OK)
    for (int i = 0; i < n; i++)
      if (ctxs[i]->comm) abort_comm(ctxs[i]);
  return s;
}

pz_status pz_sample_batch_multi(int mode, int n, const pz_shard *shards, pz_dtype dtype, int V_global,
                                const pz_batch_hints *hints) {
  if (!shards || n < 1 || (mode != PZ_SHARD_ROWS && mode != PZ_SHARD_VOCAB)) return fail(PZ_ERR_INVALID_ARGS);
  for (int i = 0; i < n; i++)
    if (!shards[i].ctx) return fail(PZ_ERR_INVALID_ARGS);
  if (mode == PZ_SHARD_ROWS) {
    // independent shards: each queued as one pz_sample_batch on its device
    for (int i = 0; i < n; i++) {
      const pz_shard &h = shards[i];
      if (h.v_offset != 0 || h.V != V_global) return fail(PZ_ERR_INVALID_ARGS);
    }
    for (int i = 0; i < n; i++) {
      const pz_shard &h = shards[i];
      const pz_status s = sample_impl(h.ctx, h.logits, dtype, h.B, h.V, h.ld, 0, h.V, h.cfg, h.hist,
                                      h.hist_off, h.rng_state, h.out_tokens, hints, h.outputs, h.stream, false);
      if (s != PZ_OK) return s;
    }
    return PZ_OK;
  }
  // vocab sharding: every shard holds the same rows; shard i is rank i
  for (int i = 0; i < n; i++) {
    const pz_shard &h = shards[i];
    const pz_status s = vocab_check(h.ctx, h.V, h.v_offset, V_global, h.rng_state, h.out_tokens, h.outputs);
    if (s != PZ_OK) return s;
    if (h.ctx->world != n || h.ctx->rank != i || h.B != shards[0].B) return fail(PZ_ERR_INVALID_ARGS);
  }
  std::vector<cudaEvent_t *> ev(n, nullptr);
  for (int i = 0; i < n; i++) {
    const pz_shard &h = shards[i];
    const pz_status s = vocab_local(h.ctx, h.logits, dtype, h.B, h.V, h.ld, h.v_offset, V_global, h.cfg,
                                    h.hist, h.hist_off, h.stream, &ev[i]);
    if (s != PZ_OK) return s;
  }
  const double t0 = now_ms();
  ncclResult_t r = g_nccl.GroupStart();
  for (int i = 0; i < n && r == ncclSuccess; i++) {
    DeviceGuard g(shards[i].ctx->device);
    const ncclResult_t ri = vocab_allgather(shards[i].ctx, shards[i].B, shards[i].stream);
    if (ri != ncclSuccess && ri != ncclInProgress) r = ri;
  }
  const ncclResult_t re = g_nccl.GroupEnd();
  if (r == ncclSuccess && re != ncclSuccess && re != ncclInProgress) r = re;
  if (r != ncclSuccess) {
    for (int i = 0; i < n; i++) abort_comm(shards[i].ctx);
    return fail(PZ_ERR_NCCL);
  }
  for (int i = 0; i < n; i++) {
    DeviceGuard g(shards[i].ctx->device);
    const pz_status s = nccl_settle(shards[i].ctx, ncclInProgress, t0);
    if (s != PZ_OK) {
      for (int j = 0; j < n; j++)
        if (shards[j].ctx->comm) abort_comm(shards[j].ctx);
      return s;
    }
  }
  for (int i = 0; i < n; i++) {
    const pz_shard &h = shards[i];
    const pz_status s = vocab_merge(h.ctx, h.B, V_global, h.cfg, h.rng_state, h.out_tokens, h.outputs, h.stream,
                                    ev[i]);
    if (s != PZ_OK) return s;
  }
  return PZ_OK;
}

// ---------------------------------------------------------------------------
// Layer 1: the reference's six calls on host pointers.
// ---------------------------------------------------------------------------
namespace {
// One staging area per device: a single-row context, its stream and device
// buffers.  Calls on one device are serialised by its mutex (the
// reference's sample_top_p is not reentrant either).
struct LegacyState {
  std::mutex mu;
  pz_sampler_ctx *ctx = nullptr;
  int vocab = 0;
  cudaStream_t st = nullptr;
  float *d_logits = nullptr;
  pz_sampler_config *d_cfg = nullptr;
  unsigned long long *d_rng = nullptr;
  int32_t *d_out = nullptr;
};
LegacyState g_legacy[kMaxDevices];

void legacy_free(LegacyState &L) {
  if (L.d_logits) cudaFree(L.d_logits);
  if (L.d_cfg) cudaFree(L.d_cfg);
  if (L.d_rng) cudaFree(L.d_rng);
  if (L.d_out) cudaFree(L.d_out);
  L.d_logits = nullptr;
  L.d_cfg = nullptr;
  L.d_rng = nullptr;
  L.d_out = nullptr;
  if (L.ctx) pz_ctx_destroy(L.ctx);
  L.ctx = nullptr;
  L.vocab = 0;
}

// The current device's staging area, ready for V columns (its lock held by
// the caller through `lk`).
pz_status legacy_ready(int V, LegacyState **out, std::unique_lock<std::mutex> &lk) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PZ_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return PZ_ERR_UNSUPPORTED;
  LegacyState &L = g_legacy[dev];
  lk = std::unique_lock<std::mutex>(L.mu);
  *out = &L;
  if (L.ctx && L.vocab >= V) return PZ_OK;
  legacy_free(L);
  if (!L.st && cudaStreamCreateWithFlags(&L.st, cudaStreamNonBlocking) != cudaSuccess)
    return PZ_ERR_CUDA;
  pz_ctx_limits lim{};
  lim.max_batch = 1;
  lim.max_vocab = std::max(V, 1024);
  lim.max_top_k = PZ_TOP_K_MAX;
  lim.max_history = 0;
  pz_status s = pz_ctx_create(&L.ctx, dev, &lim);
  if (s != PZ_OK) return s;
  if (cudaMalloc(&L.d_logits, sizeof(float) * lim.max_vocab) != cudaSuccess ||
      cudaMalloc(&L.d_cfg, sizeof(pz_sampler_config)) != cudaSuccess ||
      cudaMalloc(&L.d_rng, sizeof(unsigned long long)) != cudaSuccess ||
      cudaMalloc(&L.d_out, sizeof(int32_t)) != cudaSuccess) {
    legacy_free(L);
    return PZ_ERR_OOM;
  }
  L.vocab = lim.max_vocab;
  return PZ_OK;
}

// One row through the batch pipeline with a legacy-shaped config.
int legacy_row(const float *logits, int V, const pz_sampler_config &cfg,
               unsigned long long *rng_state) {
  if (!logits || V <= 0) {
    g_last_error = PZ_ERR_INVALID_ARGS;
    return -1;
  }
  LegacyState *Lp = nullptr;
  std::unique_lock<std::mutex> lk;
  pz_status s = legacy_ready(V, &Lp, lk);
  if (s != PZ_OK) {
    g_last_error = s;
    return -1;
  }
  LegacyState &L = *Lp;
  cudaStream_t st = L.st;
  unsigned long long state = rng_state ? *rng_state : 1ull;
  int32_t tok = -1;
  if (cudaMemcpyAsync(L.d_logits, logits, sizeof(float) * V, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(L.d_cfg, &cfg, sizeof cfg, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(L.d_rng, &state, sizeof state, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    g_last_error = PZ_ERR_CUDA;
    return -1;
  }
  s = pz_sample_batch(L.ctx, L.d_logits, PZ_DTYPE_F32, 1, V, V, L.d_cfg, nullptr, nullptr, L.d_rng,
                      L.d_out, nullptr, nullptr, st);
  if (s != PZ_OK) {
    g_last_error = s;
    return -1;
  }
  if (cudaMemcpyAsync(&tok, L.d_out, sizeof tok, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&state, L.d_rng, sizeof state, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    g_last_error = PZ_ERR_CUDA;
    return -1;
  }
  if (rng_state) *rng_state = state;
  g_last_error = PZ_OK;
  return tok;
}

pz_sampler_config legacy_cfg() {
  pz_sampler_config c{};
  c.temperature = 1.0f;  // x * (1/1) leaves every value unchanged
  c.top_k = 0;
  c.top_p = 1.0f;
  c.repetition_penalty = 1.0f;
  return c;
}
}  // namespace

int pz_sample_argmax(const float *logits, int vocab_size) {
  pz_sampler_config c = legacy_cfg();
  c.temperature = 0.0f;
  return legacy_row(logits, vocab_size, c, nullptr);
}

void pz_apply_temperature(float *logits, int vocab_size, float temperature) {
  if (!logits || vocab_size <= 0) {
    g_last_error = PZ_ERR_INVALID_ARGS;
    return;
  }
  LegacyState *Lp = nullptr;
  std::unique_lock<std::mutex> lk;
  pz_status s = legacy_ready(vocab_size, &Lp, lk);
  if (s != PZ_OK) {
    g_last_error = s;
    return;
  }
  cudaStream_t st = Lp->st;
  float *d = Lp->d_logits;
  if (cudaMemcpyAsync(d, logits, sizeof(float) * vocab_size, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      pz::launch_temperature(d, vocab_size, temperature, st) != cudaSuccess ||
      cudaMemcpyAsync(logits, d, sizeof(float) * vocab_size, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    g_last_error = PZ_ERR_CUDA;
    return;
  }
  g_last_error = PZ_OK;
}

int pz_sample_top_p(float *logits, int vocab_size, float top_p,
                    unsigned long long *rng_state) {
  pz_sampler_config c = legacy_cfg();
  c.top_p = top_p;
  c.flags = PZ_CFG_TOPP_ALWAYS;
  return legacy_row(logits, vocab_size, c, rng_state);
}

int pz_sample_top_k(float *logits, int vocab_size, int k,
                    unsigned long long *rng_state) {
  pz_sampler_config c = legacy_cfg();
  c.top_k = k;
  c.flags = PZ_CFG_TOPK_LEGACY;
  return legacy_row(logits, vocab_size, c, rng_state);
}

int pz_sample_softmax(float *logits, int vocab_size,
                      unsigned long long *rng_state) {
  pz_sampler_config c = legacy_cfg();
  return legacy_row(logits, vocab_size, c, rng_state);
}

// The RNG word lives in host memory in the legacy API (a stack variable of
// the reference's generate loop, generate.c:125); these two run on the host,
// with the same arithmetic as the device draw.
void pz_rng_seed(unsigned long long *state, unsigned long long seed) {
  if (state) *state = (seed == 0) ? 1ull : seed;  // rng.c:3-6
}

float pz_rng_float(unsigned long long *state) {  // rng.c:8-17
  unsigned long long s = *state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  *state = s;
  return static_cast<float>((s * 0x2545F4914F6CDD1DULL) >> 33) / static_cast<float>(1u << 31);
}

int sample_argmax(const float *logits, int vocab_size) {
  return pz_sample_argmax(logits, vocab_size);
}
void apply_temperature(float *logits, int vocab_size, float temperature) {
  pz_apply_temperature(logits, vocab_size, temperature);
}
int sample_top_p(float *logits, int vocab_size, float top_p,
                 unsigned long long *rng_state) {
  return pz_sample_top_p(logits, vocab_size, top_p, rng_state);
}
int sample_top_k(float *logits, int vocab_size, int k,
                 unsigned long long *rng_state) {
  return pz_sample_top_k(logits, vocab_size, k, rng_state);
}
void rng_seed(unsigned long long *state, unsigned long long seed) {
  pz_rng_seed(state, seed);
}
float rng_float(unsigned long long *state) { return pz_rng_float(state); }

}  // extern "C"
