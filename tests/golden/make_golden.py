"""Generates tests/golden/golden.json by running the REFERENCE's own sampler
(Project Zero src/sampling/*.c + src/math/softmax*.c, compiled unmodified into
oracle/_ref by oracle/Makefile) on seeded synthetic inputs.

Run in the container that holds the reference tree:
    make -C oracle all && python tests/golden/make_golden.py

The fixture stores each input as a generator spec (tests/cases.py rebuilds
the same bits anywhere) plus the reference's outputs: sampled ids and final
RNG words.  The CPU restatement (oracle/) is checked against the same
outputs here before anything is written.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))

import cases  # noqa: E402
import oracle  # noqa: E402

M = 0x2545F4914F6CDD1D
MASK = (1 << 64) - 1


def _inv_xorshift_right(y, k):
    x = y
    for _ in range(64 // k + 1):
        x = y ^ (x >> k)
    return x & MASK


def _inv_xorshift_left(y, k):
    x = y
    for _ in range(64 // k + 1):
        x = (y ^ (x << k)) & MASK
    return x


def state_before(s_after):
    """Inverse of the xorshift step of reference rng.c:11-13."""
    s = _inv_xorshift_right(s_after, 27)
    s = _inv_xorshift_left(s, 25)
    return _inv_xorshift_right(s, 12)


def state_drawing(t31):
    """A state whose next rng_float converts the 31-bit integer t31."""
    minv = pow(M, -1, 1 << 64)
    s_after = ((t31 << 33) * minv) & MASK
    return state_before(s_after)


def main():
    R = oracle.Reference()
    O = oracle.Oracle()
    out = {"reference_build": {"avx512": R.avx512, "softmax_kernel": R.softmax_kernel},
           "pipeline": [], "edge": [], "legacy": {}}

    for name, spec in cases.PIPELINE_SPECS.items():
        d = cases.build(spec)
        tok, rng = R.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        otok, orng, *_ = O.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        assert (tok == otok).all() and (rng == orng).all(), f"oracle disagrees with reference on {name}"
        out["pipeline"].append({"name": name, "spec": spec, "tokens": tok.tolist(),
                                "rng_out": [int(v) for v in rng]})
        print(f"{name}: {tok.tolist()}")

    for name, x, cfg, rng0 in cases.edge_rows():
        tok, rng = R.sample_batch(x, cfg, rng0)
        otok, orng, *_ = O.sample_batch(x, cfg, rng0)
        assert (tok == otok).all() and (rng == orng).all(), f"oracle disagrees with reference on {name}"
        out["edge"].append({"name": name, "tokens": tok.tolist(), "rng_out": [int(v) for v in rng]})

    # the six calls, known answers
    L = out["legacy"]
    L["rng"] = {}
    for seed in [42, 12345, 0, 111, 222, (1 << 63) + 5]:
        s = R.rng_seed(seed)
        vals = []
        for _ in range(16):
            v, s = R.rng_float(s)
            vals.append(int(np.float32(v).view(np.uint32)))
        L["rng"][str(seed)] = {"float_bits": vals, "final": s}
    s1 = state_drawing((1 << 31) - 1)
    v, _ = R.rng_float(s1)
    assert v == 1.0, v
    L["rng_one_state"] = s1
    L["argmax"] = [[[1.0, 3.0, 2.0, 0.5], R.sample_argmax([1.0, 3.0, 2.0, 0.5])],
                   [[10.0, 3.0, 2.0, 0.5], R.sample_argmax([10.0, 3.0, 2.0, 0.5])],
                   [[1.0, 2.0, 3.0, 100.0], R.sample_argmax([1.0, 2.0, 3.0, 100.0])],
                   [[-5.0, -1.0, -3.0, -2.0], R.sample_argmax([-5.0, -1.0, -3.0, -2.0])],
                   [[42.0], R.sample_argmax([42.0])]]
    topk = []
    for vals, k, seed, n in [([1.0, 5.0, 3.0, 2.0], 1, 42, 20),
                             ([1, 2, 3, 4, 5, 6, 7, 8], 3, 42, 100),
                             ([1.0, 10.0, 100.0, 0.1], 2, 42, 50),
                             ([1.0, 2.0], 100, 42, 1),
                             (list(range(32)), 5000, 42, 1),
                             ([float(i % 100) for i in range(2048)], 1024, 99, 1),
                             ([(i % 50) * 0.1 for i in range(4096)], 2000, 7, 1),
                             ([1, 2, 3, 4, 5, 6, 7, 8], 0, 1, 1),
                             ([1, 2, 3, 4, 5, 6, 7, 8], -5, 1, 1),
                             ([0.3, 0.1, 0.2, 0.25, 0.05], 4, 5, 40)]:
        s = R.rng_seed(seed)
        res = []
        for _ in range(n):
            t, s = R.sample_top_k(vals, k, s)
            res.append(t)
        topk.append({"logits": [float(v) for v in vals], "k": k, "seed": seed, "tokens": res, "final": s})
    L["top_k"] = topk
    topp = []
    for vals, p, seed, n in [([-100.0, 100.0, -100.0, -100.0], 0.5, 42, 20),
                             ([0.0, 0.0, 0.0, 0.0], 1.0, 42, 200),
                             ([0.5, 1.5, -0.5, 2.5, 0.0, 1.0], 0.7, 9, 60),
                             ([0.5, 1.5, -0.5, 2.5, 0.0, 1.0], 0.0, 9, 5),
                             ([0.5, 1.5, -0.5, 2.5, 0.0, 1.0], 1.5, 9, 5)]:
        s = R.rng_seed(seed)
        res = []
        for _ in range(n):
            t, s = R.sample_top_p(vals, p, s)
            res.append(t)
        topp.append({"logits": [float(v) for v in vals], "p": p, "seed": seed, "tokens": res, "final": s})
    L["top_p"] = topp
    # draw of exactly 1.0: the fallbacks (top_k.c:72, top_p.c:98, generate.c:161)
    ones = []
    for vals, kind, arg in [([0.3, 0.1, 0.9, 0.2], "top_k", 3), ([0.3, 0.1, 0.9, 0.2], "top_p", 0.9),
                            ([0.3, 0.1, 0.9, 0.2], "softmax", None)]:
        if kind == "top_k":
            t, s = R.sample_top_k(vals, arg, s1)
        elif kind == "top_p":
            t, s = R.sample_top_p(vals, arg, s1)
        else:
            t, s, _ = R.sample_softmax(vals, s1)
        ones.append({"logits": vals, "kind": kind, "arg": arg, "token": t, "final": s})
    L["draw_one"] = ones
    T = []
    for vals, temp in [([2.0, 4.0, 6.0, 8.0], 2.0), ([1.0, 2.0, 3.0], 1.0), ([1.0, 2.0, 3.0], 0.5),
                       ([1.0, 5.0, 3.0, 2.0], 0.7), ([0.1, -0.3, 7.25, 1e-3], 0.3), ([3.0, -3.0], 1e-9)]:
        y = R.apply_temperature(vals, temp)
        T.append({"logits": vals, "T": temp, "bits": [int(b) for b in np.asarray(y, np.float32).view(np.uint32)]})
    L["temperature"] = T

    path = os.path.join(HERE, "golden.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
