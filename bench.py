#!/usr/bin/env python
"""Benchmark of the B200 token sampler on BASELINE.json's workloads.

Headline (config 3): each GPU samples B=1024 rows of V=128256 fp32 logits
(N(0, 2.5^2) plus 8 boosted ids per row, +U(5,15)), each row with a
1024-token penalty history, T=0.7, top-k 50, top-p 0.9, repetition 1.1,
frequency 0.2, presence 0.1, RNG seed 1000+row.  Synthetic data, generated on
the device; a step is one pz_sample_batch call over the whole batch.  The
inputs (525 MB per GPU) are larger than L2 (126 MB), so no flush is needed.

Legs (extra keys of the same JSON line, each timed the same way):
  config2_greedy       B=256/GPU x V=151936 fp32, argmax only
  config4_hetero       B=8192 bf16 x V=151936 with per-row settings, the
                       global batch row-sharded over the N GPUs
  config5_vocab        B=4096 x V=262144 bf16, each GPU one vocabulary slice
                       of V/N columns, one NCCL allgather per step
  config1_sequential   one row, 500 dependent draws: through the device API
                       (CUDA graph, RNG state on the device) and through the
                       drop-in host calls apply_temperature + sample_top_p

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

--impl reference times the reference's own CPU sampler (oracle/_ref: the
reference's src/sampling sources compiled unmodified, driven through the
pipeline contract) on the host cores, on the same workload.  That arm loads
neither torch nor this repository's library.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))

METRIC = "sampled rows/s at B=1024,V=128256 full pipeline; % of B200 HBM peak"
W3 = dict(B=1024, V=128256, H=1024, T=0.7, k=50, p=0.9, rep=1.1, freq=0.2, pres=0.1, sd=2.5,
          nboost=8)
WORKLOAD = ("config3: B=1024 rows/GPU x V=128256 fp32, N(0,2.5^2)+8 boosts U(5,15), H=1024 history, "
            "T=0.7 top-k 50 top-p 0.9 rep 1.1 freq 0.2 pres 0.1, seeds 1000+row")
CFG_BYTES = 32

# pz_sampler_config (include/pz_sampling.h), 32 bytes: built here with numpy
# so that neither arm needs the product library to describe its inputs.
import numpy as np  # noqa: E402

CONFIG_DTYPE = np.dtype([
    ("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"),
    ("repetition_penalty", "<f4"), ("frequency_penalty", "<f4"),
    ("presence_penalty", "<f4"), ("flags", "<u4"), ("reserved", "<u4")])


def make_configs(B, temperature=1.0, top_k=0, top_p=1.0, rep=1.0, freq=0.0, pres=0.0):
    c = np.zeros(B, dtype=CONFIG_DTYPE)
    c["temperature"] = temperature
    c["top_k"] = top_k
    c["top_p"] = top_p
    c["repetition_penalty"] = rep
    c["frequency_penalty"] = freq
    c["presence_penalty"] = pres
    return c


def config3_configs(B):
    cfg = make_configs(B, W3["T"], W3["k"], W3["p"], W3["rep"], W3["freq"], W3["pres"])
    rng = (1000 + np.arange(B)).astype(np.uint64)
    return cfg, rng


def config4_configs(B, seed=4):
    """BASELINE config 4's per-row settings: T ~ U(0,1.5) with 10 % exactly
    0, k in {0,1,20,50,1024}, p ~ U(0.5,1), repetition ~ U(1,1.3), history
    length ~ U{0..2048}."""
    g = np.random.default_rng(seed)
    T = np.where(g.random(B) < 0.1, 0.0, 1.5 * g.random(B)).astype(np.float32)
    k = g.choice(np.array([0, 1, 20, 50, 1024]), B)
    p = (0.5 + 0.5 * g.random(B)).astype(np.float32)
    rep = (1.0 + 0.3 * g.random(B)).astype(np.float32)
    H = g.integers(0, 2049, B)
    return make_configs(B, T, k, p, rep), H


def config_line(world, B):
    """The `config` of both arms (identical for the same N)."""
    return {"workload": WORKLOAD, "global_batch": B * world, "rows_per_gpu": B, "V": W3["V"],
            "history": W3["H"], "parallelism": f"row-sharded x{world}, no communication",
            "l2": "inputs 525 MB/GPU > 126 MB L2; no flush"}


def algorithmic_bytes_per_row(V, H, esize):
    """Logits + history ids + token out + RNG word (read+write) + config."""
    return V * esize + H * 4 + 4 + 8 + 8 + CFG_BYTES


def hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def kernel_source_id():
    """First 12 hex digits of the SHA-1 of the kernels' source file."""
    import hashlib
    with open(os.path.join(REPO, "project-zero_b200", "csrc", "pz_kernels.cu"), "rb") as f:
        return hashlib.sha1(f.read()).hexdigest()[:12]


def profile_traffic():
    """dram bytes per launch of the slice kernel from the committed ncu
    summary, and the kernel source it was captured from ("build:
    pz_kernels.cu sha1 <12 hex>").  The traffic is dropped (None) when that
    source is not the one being benched."""
    p = os.path.join(REPO, "profiles", "slice_kernel_config3.md")
    t, build = None, None
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                t = float(line.split(":", 1)[1].strip())
            if line.startswith("build:"):
                build = line.split(":", 1)[1].strip()
    except OSError:
        pass
    live = "pz_kernels.cu sha1 " + kernel_source_id()
    if build != live:
        return None, f"stale (capture of {build}, benched {live})"
    return t, build


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons every 200 ms,
    one sampler per node (local rank 0) for the GPUs of this job."""
    Q = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids):
        self.bus = [b.lower() for b in bus_ids]
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                      text=True)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons, gpus = [], None, set(), set()
        rows = [[x.strip() for x in ln.split(",")] for ln in out.splitlines()]
        rows = [f for f in rows if len(f) >= 10]
        mine = [f for f in rows if any(b.endswith(f[1].lower()[-12:]) for b in self.bus)]
        for f in mine:
            gpus.add(f[1])
            try:
                sm.append(float(f[2]))
                mx = float(f[3])
            except ValueError:
                continue
            for name, col in (("hw_slowdown", 6), ("hw_thermal_slowdown", 7), ("sw_thermal_slowdown", 8),
                              ("sw_power_cap", 9)):
                if f[col].lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "gpus_sampled": len(gpus)}


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# CPU side (reference arm and cpu_baseline): the reference's compiled sampler
# ---------------------------------------------------------------------------
_W = {}


def _oracle_module():
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    return oracle


def _cpu_init(shm_names, shapes, kind):
    from multiprocessing import shared_memory
    oracle = _oracle_module()
    _W["shm"] = [shared_memory.SharedMemory(name=n) for n in shm_names]
    _W["arr"] = [np.ndarray(s, dtype=d, buffer=m.buf) for m, (s, d) in zip(_W["shm"], shapes)]
    _W["lib"] = oracle.Reference() if kind == "reference" else oracle.Oracle()


def _cpu_work(span):
    r0, r1 = span
    x, hist, hoff, cfg, rng = _W["arr"]
    lo, hi = int(hoff[r0]), int(hoff[r1])
    sub_off = (hoff[r0:r1 + 1] - lo).astype(np.int32)
    out = _W["lib"].sample_batch(x[r0:r1], cfg[r0:r1], rng[r0:r1], hist[lo:hi], sub_off)
    return out[0]


class CpuSampler:
    """Rows of one batch split over P worker processes (spawned; the
    reference's sample_top_p keeps a file-static buffer, so no threads)."""

    def __init__(self, x, hist, hoff, cfg, rng, procs, kind):
        import multiprocessing as mp
        from multiprocessing import shared_memory
        self.B = x.shape[0]
        self.shms, shapes = [], []
        for a in (x, hist, hoff, cfg, rng):
            a = np.ascontiguousarray(a)
            m = shared_memory.SharedMemory(create=True, size=max(a.nbytes, 1))
            np.ndarray(a.shape, dtype=a.dtype, buffer=m.buf)[...] = a
            self.shms.append(m)
            shapes.append((a.shape, a.dtype))
        self.procs = procs
        self.pool = mp.get_context("spawn").Pool(procs, initializer=_cpu_init,
                                                 initargs=([m.name for m in self.shms], shapes, kind))

    def run_rows(self, n=None):
        """The first n rows (all by default), split over the workers."""
        n = self.B if n is None else n
        step = math.ceil(n / self.procs)
        return self.pool.map(_cpu_work, [(i, min(n, i + step)) for i in range(0, n, step)])

    def close(self):
        self.pool.close()
        self.pool.join()
        for m in self.shms:
            m.close()
            m.unlink()


def time_cpu_rows(x, hist, hoff, cfg, rng, procs, kind, budget_s):
    """rows/s of the reference over the given rows, passes repeated for about
    budget_s seconds."""
    cs = CpuSampler(x, hist, hoff, cfg, rng, procs, kind)
    try:
        cs.run_rows()  # warm the workers
        t0 = time.perf_counter()
        n = 0
        while True:
            cs.run_rows()
            n += 1
            el = time.perf_counter() - t0
            if el >= budget_s:
                break
    finally:
        cs.close()
    return x.shape[0] * n / el, n, el


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_inputs_config3(B, seed=7):
    W = W3
    g = np.random.default_rng(seed)
    x = (g.standard_normal((B, W["V"]), dtype=np.float32) * np.float32(W["sd"]))
    for r in range(B):
        ids = g.choice(W["V"], W["nboost"], replace=False)
        x[r, ids] += g.uniform(5, 15, W["nboost"]).astype(np.float32)
    hist = g.integers(0, W["V"], B * W["H"], dtype=np.int32)
    hoff = (np.arange(B + 1) * W["H"]).astype(np.int32)
    return x, hist, hoff


def _bf16_bits(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)


def cpu_inputs_config4(B, V=151936, seed=11):
    g = np.random.default_rng(seed)
    x = g.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    for r in range(B):
        ids = g.choice(V, 256, replace=False)
        x[r, ids] += (10.0 * np.arange(1, 257, dtype=np.float64) ** -1.1).astype(np.float32)
    cfg, H = config4_configs(B)
    hoff = np.zeros(B + 1, dtype=np.int32)
    hoff[1:] = np.cumsum(H)
    hist = g.integers(0, V, int(hoff[-1]), dtype=np.int32)
    return _bf16_bits(x), hist, hoff, cfg, np.arange(1, B + 1, dtype=np.uint64)


def cpu_legs(procs, kind, budget_s):
    """The reference on host cores for the legs' workloads (bounded samples)."""
    legs = {}
    # config 2: argmax rows
    g = np.random.default_rng(3)
    B2, V2 = 64, 151936
    x = g.standard_normal((B2, V2), dtype=np.float32) * np.float32(3.0)
    x[np.arange(B2), g.integers(0, V2, B2)] += g.uniform(8, 20, B2).astype(np.float32)
    v, n, el = time_cpu_rows(x, np.zeros(0, np.int32), np.zeros(B2 + 1, np.int32), make_configs(B2, 0.0),
                             np.ones(B2, np.uint64), procs, kind, budget_s)
    legs["config2_greedy"] = {"rows_per_s": v, "cores": procs, "kind": kind,
                              "sample": f"{n} passes over {B2} config-2 rows"}
    # config 4: heterogeneous bf16 rows
    x, hist, hoff, cfg, rng = cpu_inputs_config4(128)
    v, n, el = time_cpu_rows(x, hist, hoff, cfg, rng, procs, kind, budget_s)
    legs["config4_hetero"] = {"rows_per_s": v, "cores": procs, "kind": kind,
                              "sample": f"{n} passes over 128 config-4 rows"}
    # config 1: one row at a time, as the reference engine runs it (one core)
    oracle = _oracle_module()
    lib = oracle.Reference() if kind == "reference" else oracle.Oracle()
    g = np.random.default_rng(42)
    V1 = 128256
    rows = g.standard_normal((16, V1), dtype=np.float32) * np.float32(2.5)
    for r in range(16):
        rows[r, g.choice(V1, 8, replace=False)] += g.uniform(5, 15, 8).astype(np.float32)
    s = lib.rng_seed(42)
    t0 = time.perf_counter()
    n = 0
    while True:
        y = lib.apply_temperature(rows[n % 16], 0.8)
        _, s = lib.sample_top_p(y, 0.95, s)
        n += 1
        if time.perf_counter() - t0 >= budget_s and n >= 4:
            break
    us_engine = (time.perf_counter() - t0) / n * 1e6
    cfg1 = make_configs(1, 0.8, 40, 0.95, 1.1)
    hist1 = g.integers(0, V1, 64, dtype=np.int32)
    hoff1 = np.array([0, 64], dtype=np.int32)
    t0 = time.perf_counter()
    m = 0
    rs = np.array([42], dtype=np.uint64)
    while True:
        _, rs = lib.sample_batch(rows[m % 16:m % 16 + 1], cfg1, rs, hist1, hoff1)[:2]
        m += 1
        if time.perf_counter() - t0 >= budget_s and m >= 4:
            break
    us_pipe = (time.perf_counter() - t0) / m * 1e6
    legs["config1_sequential"] = {
        "engine_us_per_draw": us_engine, "pipeline_us_per_draw": us_pipe, "cores": 1, "kind": kind,
        "sample": f"{n} draws of apply_temperature(0.8) + sample_top_p(0.95) (engine path, "
                  f"generate.c:154-156); {m} draws of the config-1 pipeline (T 0.8, top-k 40, "
                  f"top-p 0.95, rep 1.1, 64-id history)"}
    return legs


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    oracle = _oracle_module()
    kind = "reference" if oracle.reference_available() else "port"
    procs = host_cores()
    B = W3["B"]
    x, hist, hoff = cpu_inputs_config3(B)
    cfg, rng = config3_configs(B)
    cs = CpuSampler(x, hist, hoff, cfg, rng, procs, kind)
    try:
        cs.run_rows()  # warm the workers
        t0 = time.perf_counter()
        cs.run_rows()
        per_row = (time.perf_counter() - t0) / B
        # each step: a bounded sample of the batch, so that the K timed steps
        # take about two minutes of host time
        rows = min(B, max(procs, int(120.0 / max(args.steps, 1) / per_row)))
        for _ in range(max(args.warmup, 1)):
            cs.run_rows(rows)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cs.run_rows(rows)
        el = time.perf_counter() - t0
    finally:
        cs.close()
    value = rows * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (numpy N(0,2.5^2) + boosts, uniform histories)",
        "config": config_line(args.gpus, B),
        "host": {"cpu": cpu_model(), "processes": procs},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": procs, "kind": kind,
                         "sample": f"{args.steps} steps x {rows} of the {B} config-3 rows on {cpu_model()}"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_legs:
        line["legs"] = cpu_legs(procs, kind, budget_s=4.0)
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class Ctx:
    """Per-process GPU state: device, process group, library module."""

    def __init__(self):
        import torch
        sys.path.insert(0, os.path.join(REPO, "project-zero_b200"))
        import pz_sampling as pz
        self.torch, self.pz = torch, pz
        self.rank, self.world, self.local = dist_env()
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=self.dev)
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max_over_ranks(self, v):
        t = self.torch.tensor([float(v)], device=self.dev, dtype=self.torch.float64)
        if self.dist:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, v):
        if not self.dist:
            return [float(v)]
        t = self.torch.tensor([float(v)], device=self.dev, dtype=self.torch.float64)
        out = [self.torch.zeros_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [float(o.item()) for o in out]

    def bus_id(self, idx):
        p = self.torch.cuda.get_device_properties(idx)
        return f"{getattr(p, 'pci_domain_id', 0):08x}:{getattr(p, 'pci_bus_id', 0):02x}:" \
               f"{getattr(p, 'pci_device_id', 0):02x}.0"

    def timed(self, step, steps, warmup):
        """Device time of `steps` calls of step(), bracketed by a barrier and
        a synchronize; max over ranks (ms)."""
        torch = self.torch
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        self.barrier()
        return self.max_over_ranks(a.elapsed_time(b)), a.elapsed_time(b)


def make_device_inputs(torch, B, rank, device):
    W = W3
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    x = torch.randn(B, W["V"], generator=g, device=device, dtype=torch.float32).mul_(W["sd"])
    ids = torch.randint(0, W["V"], (B, W["nboost"]), generator=g, device=device)
    boost = torch.rand(B, W["nboost"], generator=g, device=device) * 10 + 5
    x.scatter_add_(1, ids, boost)
    hist = torch.randint(0, W["V"], (B * W["H"],), generator=g, device=device, dtype=torch.int32)
    hoff = torch.arange(B + 1, device=device, dtype=torch.int32) * W["H"]
    return x, hist, hoff


def headline(C, args, peak, peak_kind):
    torch, pz = C.torch, C.pz
    W = W3
    B, V, H = args.rows, W["V"], W["H"]
    x, hist, hoff = make_device_inputs(torch, B, C.rank, C.dev)
    cfg_np, _ = config3_configs(B)
    cfg = pz.configs_to_device(cfg_np, C.dev)
    rng = (1000 + C.rank * B + torch.arange(B, device=C.dev, dtype=torch.int64))
    out = torch.empty(B, dtype=torch.int32, device=C.dev)
    s = pz.Sampler(C.local, max_batch=B, max_vocab=V, max_top_k=W["k"], max_history=H)

    def step():
        s.sample(x, cfg, rng, out, hist, hoff, max_top_k=W["k"], max_history=H, no_full_vocab=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = None
    if C.local == 0:
        n_local = int(os.environ.get("LOCAL_WORLD_SIZE", C.world))
        clocks = Clocks([C.bus_id(i) for i in range(min(n_local, torch.cuda.device_count()))])
        clocks.start()
        time.sleep(0.5)
    # the timed region: one event before the first step and one after the
    # last (events between steps would add commands between the launches);
    # inside, the library's own two events bracket each call's kernel
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.profile(args.steps)
    C.barrier()
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    phases, n_prof, n_kernels = s.profile_phases()
    s.profile(0)
    C.barrier()
    my_ms = start.elapsed_time(end)
    per_rank = C.gather(my_ms / args.steps)
    total_ms = C.max_over_ranks(my_ms)
    clk = clocks.stop() if clocks else None
    value = C.world * B * args.steps / (total_ms / 1000.0)
    bpr = algorithmic_bytes_per_row(V, H, 4)
    launch_ms = phases["slice"] / max(n_prof, 1)
    achieved = bpr * B / (launch_ms / 1000.0) / 1e9
    traffic, traffic_build = profile_traffic()
    res = {
        "value": value, "ms_per_step": total_ms / args.steps, "per_rank_ms_per_step": per_rank,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_build": traffic_build,
                     "kernel": "slice_kernel<float>", "peak_kind": peak_kind,
                     "kernel_ms_per_step": {"slice_kernel": launch_ms,
                                            "rest": (phases["full"] + phases["merge"]) / max(n_prof, 1)},
                     "algorithmic_bytes_per_launch": bpr * B},
        "hbm_frac_of_peak_whole_step": (bpr * B / (total_ms / args.steps / 1000.0) / 1e9) / peak,
        "gpu_launches": n_kernels, "clocks": clk,
    }

    # end to end through the public API: pinned host inputs copied in, tokens read back
    x_h = x.cpu().pin_memory()
    hist_h = hist.cpu().pin_memory()
    hoff_h = hoff.cpu().pin_memory()
    cfg_h = cfg.cpu().pin_memory()
    out_h = torch.empty(B, dtype=torch.int32).pin_memory()
    ke = max(1, min(args.steps, 20))

    def e2e_step():
        x.copy_(x_h, non_blocking=True)
        hist.copy_(hist_h, non_blocking=True)
        hoff.copy_(hoff_h, non_blocking=True)
        cfg.copy_(cfg_h, non_blocking=True)
        step()
        out_h.copy_(out, non_blocking=True)

    te, _ = C.timed(e2e_step, ke, 1)
    res["e2e"] = {"value": C.world * B * ke / (te / 1000.0), "unit": "rows/s",
                  "h2d_bytes_per_step": x.numel() * 4 + hist.numel() * 4 + hoff.numel() * 4 + cfg.numel(),
                  "d2h_bytes_per_step": B * 4, "steps": ke}
    s.close()
    keep = (x, hist, hoff)
    return res, keep


def leg_config2(C, peak):
    """Greedy argmax: B=256 rows/GPU x V=151936 fp32 (weak scaling)."""
    torch, pz = C.torch, C.pz
    B, V = 256, 151936
    g = torch.Generator(device=C.dev)
    g.manual_seed(2000 + C.rank)
    x = torch.randn(B, V, generator=g, device=C.dev).mul_(3.0)
    spike = torch.randint(0, V, (B, 1), generator=g, device=C.dev)
    x.scatter_add_(1, spike, torch.rand(B, 1, generator=g, device=C.dev) * 12 + 8)
    cfg = pz.configs_to_device(make_configs(B, 0.0), C.dev)
    rng = torch.ones(B, dtype=torch.int64, device=C.dev)
    out = torch.empty(B, dtype=torch.int32, device=C.dev)
    s = pz.Sampler(C.local, max_batch=B, max_vocab=V, max_top_k=1, max_history=0)
    steps = 400

    def step():
        s.sample(x, cfg, rng, out, max_top_k=1, no_full_vocab=True)

    for _ in range(5):
        step()
    s.profile(steps)
    total, _ = C.timed(step, steps, 0)
    ph, n, kern = s.profile_phases()
    s.close()
    bpr = V * 4 + 4 + 16 + CFG_BYTES
    kms = ph["slice"] / max(n, 1)
    return {"workload": "B=256 rows/GPU x V=151936 fp32 N(0,3^2)+spike U(8,20), T=0 (argmax)",
            "rows_per_s": C.world * B * steps / (total / 1000.0), "ms_per_step": total / steps,
            "slice_kernel_ms": kms, "hbm_gbs": bpr * B / (kms / 1e3) / 1e9,
            "hbm_frac": bpr * B / (kms / 1e3) / 1e9 / peak, "gpu_launches": kern,
            "inputs": "156 MB/GPU > L2", "scaling": "weak"}


def leg_config4(C, peak, rows=8192):
    """Heterogeneous bf16 batch B=8192 x V=151936, row-sharded over the ranks
    (rows < 8192 only for profiling)."""
    torch, pz = C.torch, C.pz
    Bg, V = rows, 151936
    b0, B = pz.row_shard(Bg, C.world, C.rank)
    cfg_np, H = config4_configs(Bg)
    cfg_np, H = cfg_np[b0:b0 + B], H[b0:b0 + B]
    g = torch.Generator(device=C.dev)
    g.manual_seed(4000 + C.rank)
    xf = torch.randn(B, V, generator=g, device=C.dev).mul_(2.0)
    # Zipf(s=1.1) boosts over a random permutation: rank j of each row's
    # permutation gets 10 * j^-1.1 (the first 256 ranks carry all but a sliver)
    ids = torch.randint(0, V, (B, 256), generator=g, device=C.dev)
    zipf = 10.0 * torch.arange(1, 257, device=C.dev, dtype=torch.float32).pow(-1.1)
    xf.scatter_add_(1, ids, zipf.expand(B, 256).contiguous())
    x = xf.to(torch.bfloat16)
    del xf
    hoff_np = np.zeros(B + 1, dtype=np.int32)
    hoff_np[1:] = np.cumsum(H)
    hoff = torch.from_numpy(hoff_np).to(C.dev)
    hist = torch.randint(0, V, (max(int(hoff_np[-1]), 1),), generator=g, device=C.dev, dtype=torch.int32)
    cfg = pz.configs_to_device(cfg_np, C.dev)
    rng = torch.arange(1, B + 1, dtype=torch.int64, device=C.dev) + b0
    out = torch.empty(B, dtype=torch.int32, device=C.dev)
    s = pz.Sampler(C.local, max_batch=B, max_vocab=V, max_top_k=1024, max_history=2048)
    steps = 10

    def step():
        s.sample(x, cfg, rng, out, hist, hoff)

    for _ in range(3):
        step()
    s.profile(steps)
    total, _ = C.timed(step, steps, 0)
    ph, n, kern = s.profile_phases()
    s.close()
    keff = np.where((cfg_np["top_k"] <= 0) | (cfg_np["top_k"] >= V), 0, cfg_np["top_k"])
    n_full = int(((cfg_np["temperature"] >= 1e-6) & (keff == 0)).sum())
    bytes_rows = float((V * 2 + 4 * H + 4 + 16 + CFG_BYTES).sum())
    sms = ph["slice"] / max(n, 1)
    fms = ph["full"] / max(n, 1)
    return {"workload": "B=8192 bf16 x V=151936, N(0,2^2)+Zipf(1.1) boosts, per-row T/k/p/rep/H "
                        "(10% greedy, k in {0,1,20,50,1024}), row-sharded",
            "rows_per_s": Bg * steps / (total / 1000.0), "ms_per_step": total / steps,
            "rows_per_gpu": B, "full_vocab_rows_per_gpu": n_full,
            "slice_kernel_ms": sms, "full_kernel_ms": fms,
            "slice_kernel_hbm_gbs": bytes_rows / (sms / 1e3) / 1e9,
            "slice_kernel_hbm_frac": bytes_rows / (sms / 1e3) / 1e9 / peak,
            "whole_step_hbm_frac": bytes_rows / (total / steps / 1e3) / 1e9 / peak,
            "full_kernel_share": fms / max(sms + fms, 1e-9), "gpu_launches": kern,
            "scaling": "strong (8192 rows split over the GPUs)"}


def leg_config5(C, peak):
    """Vocab sharding: B=4096 x V=262144 bf16, V/N columns per GPU, one NCCL
    allgather of the per-GPU top-64 lists per step."""
    torch, pz = C.torch, C.pz
    B, Vg = 4096, 262144
    v0, Vl = pz.row_shard(Vg, C.world, C.rank)
    g = torch.Generator(device=C.dev)
    g.manual_seed(5000 + C.rank)
    xf = torch.randn(B, Vl, generator=g, device=C.dev).mul_(2.5)
    # 16 boosted global ids per row (same on every rank), applied where they fall
    gb = torch.Generator(device=C.dev)
    gb.manual_seed(5555)
    ids = torch.randint(0, Vg, (B, 16), generator=gb, device=C.dev)
    val = torch.rand(B, 16, generator=gb, device=C.dev) * 10 + 5
    mine = (ids >= v0) & (ids < v0 + Vl)
    xf.scatter_add_(1, torch.where(mine, ids - v0, 0), torch.where(mine, val, 0.0))
    x = xf.to(torch.bfloat16)
    del xf
    cfg = pz.configs_to_device(make_configs(B, 1.0, 64, 0.95), C.dev)
    rng = torch.arange(1, B + 1, dtype=torch.int64, device=C.dev)
    out = torch.empty(B, dtype=torch.int32, device=C.dev)
    s = pz.Sampler(C.local, max_batch=B, max_vocab=Vl, max_top_k=64, max_history=0)
    uid = pz.Sampler.nccl_unique_id() if C.rank == 0 else bytes(128)
    if C.dist:
        obj = [uid]
        C.dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    s.init_nccl(C.world, C.rank, uid, timeout_ms=120000)
    steps = 50

    def step():
        s.sample_vocab_sharded(x, v0, Vg, cfg, rng, out)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    s.profile(steps)
    total, _ = C.timed(step, steps, 0)
    ph, n, kern = s.profile_phases()
    s.close()
    n = max(n, 1)
    bytes_slice = B * (Vl * 2 + 16 + CFG_BYTES)
    sms = ph["slice"] / n
    return {"workload": f"B=4096 x V=262144 bf16 N(0,2.5^2)+16 boosts U(5,15), T 1.0 top-k 64 top-p 0.95; "
                        f"{C.world} vocab slice(s) of {Vl} columns",
            "shards": C.world, "rows_per_s": B * steps / (total / 1000.0), "ms_per_step": total / steps,
            "slice_kernel_ms": sms, "allgather_ms": ph["allgather"] / n, "merge_kernel_ms": ph["merge"] / n,
            "allgather_share": ph["allgather"] / max(ph["slice"] + ph["allgather"] + ph["merge"], 1e-9),
            "allgather_bytes_per_rank": B * 65 * 8,
            "slice_kernel_hbm_frac": bytes_slice / (sms / 1e3) / 1e9 / peak, "gpu_launches": kern,
            "scaling": "strong (the vocabulary split over the GPUs)"}


def leg_config1(C):
    """One row, 500 dependent draws, fresh logits each step."""
    torch, pz = C.torch, C.pz
    V, N = 128256, 500
    g = torch.Generator(device=C.dev)
    g.manual_seed(42 + C.rank)
    xs = torch.randn(N, V, generator=g, device=C.dev).mul_(2.5)
    ids = torch.randint(0, V, (N, 8), generator=g, device=C.dev)
    xs.scatter_add_(1, ids, torch.rand(N, 8, generator=g, device=C.dev) * 10 + 5)
    hist = torch.randint(0, V, (64,), generator=g, device=C.dev, dtype=torch.int32)
    hoff = torch.tensor([0, 64], dtype=torch.int32, device=C.dev)
    res = {"workload": "1 row x V=128256 fp32 N(0,2.5^2)+8 boosts U(5,15), 500 sequential draws, "
                       "fresh logits per step (device-resident, written before the timed region)"}
    s = pz.Sampler(C.local, max_batch=1, max_vocab=V, max_top_k=64, max_history=64)
    for name, cfg_np, k, use_hist in (
            ("pipeline", make_configs(1, 0.8, 40, 0.95, 1.1), 40, True),
            ("engine", make_configs(1, 0.8, 0, 0.95), 0, False)):
        cfg = pz.configs_to_device(cfg_np, C.dev)
        rng = torch.tensor([42], dtype=torch.int64, device=C.dev)
        out = torch.empty(N, dtype=torch.int32, device=C.dev)

        def draws():
            for i in range(N):
                s.sample(xs[i:i + 1], cfg, rng, out[i:i + 1], hist if use_hist else None,
                         hoff if use_hist else None, max_top_k=max(k, 1), max_history=64 if use_hist else 0,
                         no_full_vocab=k > 0)
                if use_hist:
                    hist[i % 64:i % 64 + 1].copy_(out[i:i + 1])  # the history window slides

        draws()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            draws()
        tot, _ = C.timed(graph.replay, 3, 1)
        res[f"{name}_device_graph_us_per_draw"] = tot / 3 / N * 1000.0
        del graph
    # the library's own decode step (pz_decode_step_*): fresh logits copied
    # into the fixed buffer, then the step graph (sample, window append)
    buf = torch.empty(1, V, device=C.dev)
    cfg = pz.configs_to_device(make_configs(1, 0.8, 40, 0.95, 1.1), C.dev)
    rng = torch.tensor([42], dtype=torch.int64, device=C.dev)
    out1 = torch.empty(1, dtype=torch.int32, device=C.dev)
    ring = hist.view(1, 64)
    step = pz.DecodeStep(s, buf, cfg, rng, out1, ring, max_top_k=40, max_history=64, no_full_vocab=True)
    it = [0]

    def one():
        buf.copy_(xs[it[0] % N:it[0] % N + 1])
        step.launch()
        it[0] += 1

    tot, _ = C.timed(one, N, 5)
    res["pipeline_decode_step_us_per_draw"] = tot / N * 1000.0
    step.close()
    s.close()
    # the drop-in host calls of the reference's generate loop (generate.c:154-156)
    xh = xs[:16].cpu().numpy()
    st = pz.rng_seed(42)
    for i in range(3):
        y = pz.apply_temperature(xh[i].copy(), 0.8)
        _, st = pz.sample_top_p(y, 0.95, st)
    t0 = time.perf_counter()
    n = 0
    while n < 200 and (n < 20 or time.perf_counter() - t0 < 2.0):
        y = pz.apply_temperature(xh[n % 16].copy(), 0.8)
        _, st = pz.sample_top_p(y, 0.95, st)
        n += 1
    res["engine_host_dropin_us_per_draw"] = (time.perf_counter() - t0) / n * 1e6
    res["host_dropin_draws"] = n
    return res


def run_ours(args):
    C = Ctx()
    torch = C.torch
    peak, peak_kind = hbm_peak()
    if args.only_leg:
        # one leg alone (profiling): its JSON object, no headline line
        fn = {"config2_greedy": lambda: leg_config2(C, peak),
              "config4_hetero": lambda: leg_config4(C, peak, args.c4_rows),
              "config5_vocab": lambda: leg_config5(C, peak),
              "config1_sequential": lambda: leg_config1(C)}[args.only_leg]
        r = fn()
        if C.rank == 0:
            print(json.dumps({"leg": args.only_leg, **r}), flush=True)
        if C.dist:
            C.barrier()
            C.dist.destroy_process_group()
        return 0
    res, keep = headline(C, args, peak, peak_kind)
    B = args.rows
    legs = {}
    if not args.no_legs:
        del keep
        torch.cuda.empty_cache()
        legs["config2_greedy"] = leg_config2(C, peak)
        legs["config4_hetero"] = leg_config4(C, peak)
        torch.cuda.empty_cache()
        legs["config5_vocab"] = leg_config5(C, peak)
        torch.cuda.empty_cache()
        legs["config1_sequential"] = leg_config1(C)

    cpu = cpu_leg = None
    if C.rank == 0 and C.world == 1 and not args.no_cpu:
        oracle = _oracle_module()
        kind = "reference" if oracle.reference_available() else "port"
        procs = host_cores()
        nb = 256
        x, hist, hoff = cpu_inputs_config3(nb, seed=9)
        cfg, rng = config3_configs(nb)
        v, n, el = time_cpu_rows(x, hist, hoff, cfg, rng, procs, kind, budget_s=args.cpu_seconds)
        cpu = {"value": v, "unit": "rows/s", "cores": procs, "kind": kind,
               "sample": f"{n} passes over {nb} config-3 rows ({el:.1f} s wall, {cpu_model()})"}
        if not args.no_legs:
            cpu_leg = cpu_legs(procs, kind, budget_s=3.0)
            for name, v in cpu_leg.items():
                if name in legs:
                    legs[name]["cpu_reference"] = v

    if C.rank == 0:
        line = {
            "metric": METRIC, "value": res["value"], "unit": "rows/s", "n_gpus": C.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch.randn N(0,2.5^2) + 8 boosts U(5,15), uniform 1024-id histories)",
            "config": config_line(C.world, B),
            "per_rank_ms_per_step": res["per_rank_ms_per_step"],
            "roofline": res["roofline"],
            "hbm_frac_of_peak_whole_step": res["hbm_frac_of_peak_whole_step"],
            "e2e": res["e2e"],
            "gpu_launches": res["gpu_launches"],  # counted by the library over the timed calls
            "clocks": res["clocks"],
            "cpu_baseline": cpu,
        }
        if legs:
            line["legs"] = legs
        print(json.dumps(line), flush=True)
    if C.dist:
        C.barrier()
        C.dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline legs")
    ap.add_argument("--no-legs", action="store_true", help="headline config 3 only")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--only-leg", default="", choices=["", "config2_greedy", "config4_hetero",
                                                        "config5_vocab", "config1_sequential"],
                    help="run one leg alone (profiling)")
    ap.add_argument("--c4-rows", type=int, default=8192, help="config-4 rows (profiling a smaller case)")
    ap.add_argument("--rows", type=int, default=W3["B"],
                    help="rows per GPU (profiling a smaller case; the bench line is quoted at 1024)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
