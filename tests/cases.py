"""Builds sampler inputs from small JSON-able specs (BASELINE.json's five
configs at reduced batch, plus edge cases).  The same spec gives the same
bits everywhere (tests/synth.py), so golden fixtures store specs + outputs."""
from __future__ import annotations

import numpy as np

import synth

CONFIG_DTYPE = np.dtype([
    ("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"),
    ("repetition_penalty", "<f4"), ("frequency_penalty", "<f4"),
    ("presence_penalty", "<f4"), ("flags", "<u4"), ("reserved", "<u4")])


def configs(B, temperature=1.0, top_k=0, top_p=1.0, rep=1.0, freq=0.0, pres=0.0, flags=0):
    c = np.zeros(B, dtype=CONFIG_DTYPE)
    c["temperature"] = temperature
    c["top_k"] = top_k
    c["top_p"] = top_p
    c["repetition_penalty"] = rep
    c["frequency_penalty"] = freq
    c["presence_penalty"] = pres
    c["flags"] = flags
    return c


def build(spec):
    """spec -> dict(logits [B,V] f32 or u16 bf16 bits, cfg, rng [B] u64,
    hist, hist_off).  Keys of spec:
      seed, B, V, sd, row0 (default 0), dtype 'f32'|'bf16',
      boosts: [n, lo, hi] | zipf: [n, scale] | spike: [lo, hi],
      hist_len: int | 'hetero', cfg: dict of scalars | 'hetero',
      rng_base (default 1000): rng[r] = rng_base + row0 + r (0 -> 1)."""
    seed, B, V = spec["seed"], spec["B"], spec["V"]
    row0 = spec.get("row0", 0)
    x = synth.logits_normal(seed, B, V, spec["sd"], row0=row0)
    if "boosts" in spec:
        n, lo, hi = spec["boosts"]
        synth.add_boosts(x, seed, n, lo, hi, row0=row0)
    if "spike" in spec:
        lo, hi = spec["spike"]
        synth.add_boosts(x, seed, 1, lo, hi, row0=row0)
    if "zipf" in spec:
        n, scale = spec["zipf"]
        synth.add_zipf_boosts(x, seed, n, scale, row0=row0)
    if spec.get("cfg") == "hetero":
        u = [synth.param_uniform(seed, B, j, row0=row0) for j in range(7)]
        T = np.where(u[0] < 0.1, 0.0, 1.5 * u[1]).astype(np.float32)
        ks = np.array([0, 1, 20, 50, 1024])[np.minimum((u[2] * 5).astype(int), 4)]
        p = (0.5 + 0.5 * u[3]).astype(np.float32)
        rep = (1.0 + 0.3 * u[4]).astype(np.float32)
        cfg = configs(B, T, ks, p, rep)
        H = np.floor(u[5] * 2049).astype(np.int64)
    else:
        cfg = configs(B, **spec.get("cfg", {}))
        H = np.full(B, int(spec.get("hist_len", 0)), dtype=np.int64)
    hist = hist_off = None
    if spec.get("hist_len", 0) != 0 or spec.get("cfg") == "hetero":
        hist, hist_off = synth.history(seed + 7, H, V, row0=row0)
    base = spec.get("rng_base", 1000)
    rng = np.array([(base + row0 + r) or 1 for r in range(B)], dtype=np.uint64)
    if spec.get("dtype", "f32") == "bf16":
        x = synth.to_bf16_bits(x)
    return dict(logits=x, cfg=cfg, rng=rng, hist=hist, hist_off=hist_off)


# BASELINE.json configs at reduced batch (the oracle must finish in seconds).
PIPELINE_SPECS = {
    "c1_k40_p95": dict(seed=42, B=6, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=64,
                       cfg=dict(temperature=0.8, top_k=40, top_p=0.95, rep=1.1), rng_base=42),
    "c1_engine_p95": dict(seed=43, B=4, V=128256, sd=2.5, boosts=[8, 5.0, 15.0],
                          cfg=dict(temperature=0.8, top_k=0, top_p=0.95), rng_base=42),
    "c2_greedy": dict(seed=2, B=8, V=151936, sd=3.0, spike=[8.0, 20.0], cfg=dict(temperature=0.0)),
    "c3_full": dict(seed=3, B=8, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=1024,
                    cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1)),
    "c4_hetero": dict(seed=4, B=24, V=151936, sd=2.0, zipf=[256, 10.0], dtype="bf16", cfg="hetero"),
    "c5_vocab": dict(seed=5, B=6, V=262144, sd=2.5, boosts=[16, 5.0, 15.0], dtype="bf16",
                     cfg=dict(temperature=1.0, top_k=64, top_p=0.95)),
    "softmax_full": dict(seed=6, B=3, V=32000, sd=2.0, boosts=[4, 3.0, 6.0],
                         cfg=dict(temperature=0.9, top_k=0, top_p=1.0)),
    "topk_only": dict(seed=7, B=4, V=50000, sd=2.0, hist_len=200,
                      cfg=dict(temperature=1.2, top_k=100, top_p=1.0, rep=1.3, pres=0.5)),
    "topk1024_p": dict(seed=8, B=3, V=65536, sd=1.0, dtype="bf16",
                       cfg=dict(temperature=1.4, top_k=1024, top_p=0.99)),
    "greedy_pen": dict(seed=9, B=4, V=20000, sd=2.0, boosts=[2, 1.0, 2.0], hist_len=500,
                       cfg=dict(temperature=0.0, rep=1.5, freq=0.3, pres=0.4)),
    "bf16_topp_full": dict(seed=10, B=3, V=151936, sd=2.0, zipf=[64, 8.0], dtype="bf16",
                           cfg=dict(temperature=1.3, top_k=0, top_p=0.8)),
    "topp_big_vocab_argmax": dict(seed=11, B=2, V=262144, sd=2.0, dtype="bf16",
                                  cfg=dict(temperature=0.9, top_k=0, top_p=0.7)),
    "small_v": dict(seed=12, B=16, V=7, sd=1.0, cfg=dict(temperature=0.5, top_k=3, top_p=0.8)),
    "small_v_full": dict(seed=13, B=16, V=100, sd=0.5, cfg=dict(temperature=0.5, top_k=0, top_p=0.9)),
}


def edge_rows():
    """Hand-built rows: ties, -inf, -1e30, single element, k > V, p edges.
    Returns list of (name, logits f32 [1,V], cfg, rng)."""
    out = []
    inf = np.float32(np.inf)

    def row(name, vals, **cfg):
        x = np.array([vals], dtype=np.float32)
        out.append((name, x, configs(1, **cfg), np.array([42], dtype=np.uint64)))

    row("ties_greedy", [1, 3, 3, 2, 3], temperature=0.0)
    row("ties_topk2", [1, 3, 3, 2, 3], temperature=1.0, top_k=2, top_p=1.0)
    row("ties_topk2_p", [1, 3, 3, 2, 3], temperature=1.0, top_k=2, top_p=0.5)
    row("neg_inf", [-inf, -inf, 2.0, -inf, 1.0], temperature=0.7, top_k=3, top_p=1.0)
    row("all_minus_1e30", [-1e30, -1e30, -1e30], temperature=1.0, top_k=2, top_p=1.0)
    row("below_floor", [-2e30, -1e31, -3e30, -1e30], temperature=1.0, top_k=2, top_p=0.9)
    row("single", [42.0], temperature=0.8, top_k=0, top_p=0.9)
    row("single_softmax", [42.0], temperature=0.8)
    row("zero_signs", [-0.0, 0.0, -0.0, 0.0], temperature=0.0)
    row("zero_signs_topk", [-0.0, 0.0, -0.0, 0.0], temperature=1.0, top_k=3, top_p=1.0)
    row("peak_p_half", [-100.0, 100.0, -100.0, -100.0], temperature=1.0, top_p=0.5)
    row("uniform4_softmax", [0.0, 0.0, 0.0, 0.0], temperature=1.0)
    row("tiny_T", [1.0, 5.0, 3.0], temperature=1e-6, top_k=2, top_p=1.0)
    row("below_tiny_T", [1.0, 5.0, 3.0], temperature=9e-7, top_k=2)
    row("k_eq_V_minus1", [0.5, 0.1, 0.9, 0.3], temperature=1.0, top_k=3, top_p=1.0)
    row("k_ge_V_softmax", [0.5, 0.1, 0.9, 0.3], temperature=1.0, top_k=4, top_p=1.0)
    row("neg_k_topp", [0.5, 0.1, 0.9, 0.3], temperature=1.0, top_k=-5, top_p=0.7)
    row("divide_flag", [0.1, 0.2, 0.3, 0.4, 0.5], temperature=0.3, top_k=4, top_p=0.95, flags=1)
    row("nan_first_greedy", [np.nan, 1.0, 2.0], temperature=0.0)
    row("nan_mid_greedy", [1.0, np.nan, 2.0, 2.0], temperature=0.0)
    row("nan_mid_topk", [1.0, np.nan, 2.0, 0.5], temperature=1.0, top_k=2, top_p=0.9)
    row("nan_first_topp", [np.nan, 1.0, 2.0], temperature=1.0, top_p=0.9)
    return out
