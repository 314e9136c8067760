#!/usr/bin/env python
"""Benchmark of the B200 token sampler on BASELINE.json's headline workload.

Workload (config 3): each GPU samples B=1024 rows of V=128256 fp32 logits
(N(0, 2.5^2) plus 8 boosted ids per row, +U(5,15)), each row with a
1024-token penalty history, T=0.7, top-k 50, top-p 0.9, repetition 1.1,
frequency 0.2, presence 0.1, RNG seed 1000+row.  Synthetic data, generated on
the device; a step is one pz_sample_batch call over the whole batch.  The
inputs (525 MB per GPU) are larger than L2 (126 MB), so no flush is needed.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (row sharding, weak)

--impl reference times the reference's own CPU sampler (oracle/_ref: the
reference's src/sampling sources compiled unmodified, driven through the
pipeline contract) on the host cores, on the same workload.
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
sys.path.insert(0, os.path.join(REPO, "project-zero_b200"))

METRIC = "sampled rows/s at B=1024,V=128256 full pipeline; % of B200 HBM peak"
W3 = dict(B=1024, V=128256, H=1024, T=0.7, k=50, p=0.9, rep=1.1, freq=0.2, pres=0.1, sd=2.5,
          nboost=8)
WORKLOAD = ("config3: B=1024 rows/GPU x V=128256 fp32, N(0,2.5^2)+8 boosts U(5,15), H=1024 history, "
            "T=0.7 top-k 50 top-p 0.9 rep 1.1 freq 0.2 pres 0.1, seeds 1000+row")
CFG_BYTES = 32


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


def profile_traffic():
    """dram bytes per launch of the slice kernel from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", "slice_kernel_config3.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons (200 ms)."""
    Q = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id, index):
        self.bus = bus_id.lower()
        self.index = str(index)
        self.p = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                      text=True)
        except OSError:
            self.p = None

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        rows = [[x.strip() for x in ln.split(",")] for ln in out.splitlines()]
        rows = [f for f in rows if len(f) >= 10]
        mine = [f for f in rows if self.bus.endswith(f[1].lower()[-12:])]
        if not mine:
            mine = [f for f in rows if f[0] == self.index]
        for f in mine:
            f = f[1:]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, col in (("hw_slowdown", 5), ("hw_thermal_slowdown", 6), ("sw_thermal_slowdown", 7),
                              ("sw_power_cap", 8)):
                if f[col].lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# CPU side (reference arm and cpu_baseline): the reference's compiled sampler
# ---------------------------------------------------------------------------
_W = {}


def _cpu_init(shm_names, shapes, kind):
    import numpy as np
    from multiprocessing import shared_memory
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    _W["shm"] = [shared_memory.SharedMemory(name=n) for n in shm_names]
    _W["arr"] = [np.ndarray(s, dtype=d, buffer=m.buf) for m, (s, d) in zip(_W["shm"], shapes)]
    _W["lib"] = oracle.Reference() if kind == "reference" else oracle.Oracle()


def _cpu_work(span):
    import numpy as np
    r0, r1 = span
    x, hist, hoff, cfg, rng = _W["arr"]
    lo, hi = int(hoff[r0]), int(hoff[r1])
    sub_off = (hoff[r0:r1 + 1] - lo).astype(np.int32)
    lib = _W["lib"]
    out = lib.sample_batch(x[r0:r1], cfg[r0:r1], rng[r0:r1], hist[lo:hi], sub_off)
    return out[0]


class CpuSampler:
    """Rows of one batch split over P worker processes (spawned; the
    reference's sample_top_p keeps a file-static buffer, so no threads)."""

    def __init__(self, x, hist, hoff, cfg, rng, procs, kind):
        import multiprocessing as mp
        import numpy as np
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
        ctx = mp.get_context("spawn")
        self.pool = ctx.Pool(procs, initializer=_cpu_init,
                             initargs=([m.name for m in self.shms], shapes, kind))
        step = math.ceil(self.B / procs)
        self.spans = [(i, min(self.B, i + step)) for i in range(0, self.B, step)]

    def run(self):
        return self.pool.map(_cpu_work, self.spans)

    def run_rows(self, n):
        """The first n rows, split over the workers."""
        step = math.ceil(n / self.procs)
        return self.pool.map(_cpu_work, [(i, min(n, i + step)) for i in range(0, n, step)])

    def close(self):
        self.pool.close()
        self.pool.join()
        for m in self.shms:
            m.close()
            m.unlink()


def cpu_inputs_numpy(B, seed=7):
    import numpy as np
    W = W3
    g = np.random.default_rng(seed)
    x = (g.standard_normal((B, W["V"]), dtype=np.float32) * np.float32(W["sd"]))
    for r in range(B):
        ids = g.choice(W["V"], W["nboost"], replace=False)
        x[r, ids] += g.uniform(5, 15, W["nboost"]).astype(np.float32)
    hist = g.integers(0, W["V"], B * W["H"], dtype=np.int32)
    hoff = (np.arange(B + 1) * W["H"]).astype(np.int32)
    return x, hist, hoff


def cpu_configs(B):
    import numpy as np
    from pz_sampling import make_configs
    cfg = make_configs(B, W3["T"], W3["k"], W3["p"], W3["rep"], W3["freq"], W3["pres"])
    rng = (1000 + np.arange(B)).astype(np.uint64)
    return cfg, rng


def time_cpu(x, hist, hoff, procs, kind, budget_s, min_steps=1, max_steps=None):
    cfg, rng = cpu_configs(x.shape[0])
    cs = CpuSampler(x, hist, hoff, cfg, rng, procs, kind)
    try:
        cs.run()  # warm the workers
        t0 = time.perf_counter()
        n = 0
        while True:
            cs.run()
            n += 1
            el = time.perf_counter() - t0
            if (n >= min_steps and el >= budget_s) or (max_steps and n >= max_steps):
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


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    kind = "reference" if oracle.reference_available() else "port"
    procs = host_cores()
    B = W3["B"]
    x, hist, hoff = cpu_inputs_numpy(B)
    cfg, rng = cpu_configs(B)
    cs = CpuSampler(x, hist, hoff, cfg, rng, procs, kind)
    try:
        cs.run()  # warm the workers
        t0 = time.perf_counter()
        cs.run()
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
        "config": {"workload": WORKLOAD, "global_batch": B, "parallelism": f"{procs} host processes",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": procs, "kind": kind,
                         "sample": f"{args.steps} steps x {rows} of the {B} config-3 rows on {cpu_model()}"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
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


def run_ours(args):
    import numpy as np
    import torch
    import pz_sampling as pz

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)
    W = W3
    B, V, H = args.rows, W["V"], W["H"]
    x, hist, hoff = make_device_inputs(torch, B, rank, dev)
    cfg_np, _ = cpu_configs(B)
    cfg = pz.configs_to_device(cfg_np, dev)
    rng = (1000 + rank * B + torch.arange(B, device=dev, dtype=torch.int64))
    out = torch.empty(B, dtype=torch.int32, device=dev)
    s = pz.Sampler(local, max_batch=B, max_vocab=V, max_top_k=W["k"], max_history=H)

    def step():
        s.sample(x, cfg, rng, out, hist, hoff, max_top_k=W["k"], max_history=H, no_full_vocab=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(dev)
    bus = f"{getattr(props, 'pci_domain_id', 0):08x}:{getattr(props, 'pci_bus_id', 0):02x}:" \
          f"{getattr(props, 'pci_device_id', 0):02x}.0"
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = vis.split(",")[local] if vis and len(vis.split(",")) > local else str(local)
    clocks = Clocks(bus, phys)
    clocks.start()
    time.sleep(0.5)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    s.profile(args.steps)  # CUDA events around the kernels of each timed call
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    slice_ms, rest_ms, n_prof, n_kernels = s.profile_read()
    s.profile(0)
    if dist:
        dist.barrier()
    total_ms = starts[0].elapsed_time(ends[-1])
    per = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    clk = clocks.stop()
    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = world * B * args.steps / (total_ms / 1000.0)

    # roofline of the dominant kernel: slice_kernel, one launch per step,
    # timed with CUDA events on the launching stream inside the timed region
    peak, peak_kind = hbm_peak()
    bpr = algorithmic_bytes_per_row(V, H, 4)
    launch_ms = slice_ms / max(n_prof, 1)
    achieved = bpr * B / (launch_ms / 1000.0) / 1e9
    traffic = profile_traffic()

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

    e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(ke):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * B * ke / (float(te.item()) / 1000.0)
    h2d = x.numel() * 4 + hist.numel() * 4 + hoff.numel() * 4 + cfg.numel()
    d2h = B * 4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle
        kind = "reference" if oracle.reference_available() else "port"
        procs = host_cores()
        nb = min(B, 256)
        xs = x[:nb].cpu().numpy()
        hs = hist[: nb * H].cpu().numpy()
        ho = hoff[: nb + 1].cpu().numpy()
        v, n, el = time_cpu(xs, hs, ho, procs, kind, budget_s=args.cpu_seconds)
        cpu = {"value": v, "unit": "rows/s", "cores": procs, "kind": kind,
               "sample": f"{n} passes over {nb} rows of the same config-3 inputs ({el:.1f} s wall, "
                         f"{cpu_model()})"}

    s.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch.randn N(0,2.5^2) + 8 boosts U(5,15), uniform 1024-id histories)",
            "config": {"workload": WORKLOAD, "global_batch": B * world, "rows_per_gpu": B, "V": V,
                       "history": H, "parallelism": f"row-sharded x{world}, no communication",
                       "l2": "inputs 525 MB/GPU > 126 MB L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "slice_kernel<float>", "peak_kind": peak_kind,
                         "kernel_ms_per_step": {"slice_kernel": launch_ms,
                                                "rest": rest_ms / max(n_prof, 1)},
                         "algorithmic_bytes_per_launch": bpr * B},
            "hbm_frac_of_peak_whole_step": (bpr * B / (total_ms / args.steps / 1000.0) / 1e9) / peak,
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": ke},
            "gpu_launches": n_kernels,  # counted by the library over the timed calls
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
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
