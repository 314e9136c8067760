"""The C restatement (oracle/libpzoracle.so) run over a large batch by spawned
worker processes, rows split evenly (TEST INFRASTRUCTURE).

Spawned, not forked: the tests that use it have already initialised CUDA in
the parent, and a process forked after that hangs.  The inputs are shared
with the workers through shared memory, not pickled.
"""
from __future__ import annotations

import math
import multiprocessing as mp
import os
from multiprocessing import shared_memory

import numpy as np

_W = {}
TESTS = os.path.dirname(os.path.abspath(__file__))


def _init(names, shapes):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(TESTS), "oracle"))
    import oracle
    _W["shm"] = [shared_memory.SharedMemory(name=n) for n in names]
    _W["arr"] = [np.ndarray(s, dtype=t, buffer=m.buf) for m, (s, t) in zip(_W["shm"], shapes)]
    _W["lib"] = oracle.Oracle()


def _work(job):
    r0, r1, stride = job
    x, cfg, rng, hist, hoff = _W["arr"]
    lo, hi = int(hoff[r0]), int(hoff[r1])
    sub = (hoff[r0:r1 + 1] - lo).astype(np.int32)
    return _W["lib"].sample_batch(x[r0:r1], cfg[r0:r1], rng[r0:r1], hist[lo:hi], sub, cand_stride=stride)


def sample_batch(x, cfg, rng, hist=None, hist_off=None, cand_stride=0, procs=None):
    """Oracle.sample_batch over [B, V] rows, in parallel.  Same return value:
    (tokens, new_rng, cand_ids, cand_probs, n_cand)."""
    B = x.shape[0]
    if hist is None:
        hist = np.zeros(0, np.int32)
        hist_off = np.zeros(B + 1, np.int32)
    procs = procs or max(1, min(len(os.sched_getaffinity(0)), 32))
    shms, shapes = [], []
    try:
        for a in (x, cfg, rng, hist, hist_off):
            a = np.ascontiguousarray(a)
            m = shared_memory.SharedMemory(create=True, size=max(a.nbytes, 1))
            np.ndarray(a.shape, dtype=a.dtype, buffer=m.buf)[...] = a
            shms.append(m)
            shapes.append((a.shape, a.dtype))
        step = math.ceil(B / (4 * procs))
        jobs = [(i, min(B, i + step), cand_stride) for i in range(0, B, step)]
        with mp.get_context("spawn").Pool(procs, initializer=_init,
                                          initargs=([m.name for m in shms], shapes)) as pool:
            parts = pool.map(_work, jobs)
    finally:
        for m in shms:
            m.close()
            m.unlink()
    tok = np.concatenate([p[0] for p in parts])
    rng_out = np.concatenate([p[1] for p in parts])
    if not cand_stride:
        return tok, rng_out, None, None, None
    return (tok, rng_out, np.concatenate([p[2] for p in parts]), np.concatenate([p[3] for p in parts]),
            np.concatenate([p[4] for p in parts]))
