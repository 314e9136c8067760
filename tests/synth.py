"""Seeded synthetic sampler inputs whose bits are reproducible on any IEEE host.

Every value comes from a counter-based hash (the splitmix64 finaliser) and a
fixed sequence of IEEE double operations followed by one round-to-nearest
conversion to float32, so the same call gives the same bits in this container
and on the GPU box.  That lets the golden fixtures store only the generator
arguments and the expected outputs.

Shapes follow BASELINE.json's configs: logits ~ N(0, sd^2) (Irwin-Hall(10)
approximation, tails to +-5.5 sd), plus boosted "hot" ids, plus penalty
histories of uniform ids.
"""
from __future__ import annotations

import math

import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)
_G = np.uint64(0x9E3779B97F4A7C15)
_C = np.uint64(0xD1B54A32D192ED03)

# counter bases for the independent streams of one row
_NORMAL, _BOOST, _HIST, _PARAM = 0, 1 << 40, 2 << 40, 3 << 40


def _mix64(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def hash3(seed, stream, ctr):
    """64-bit hash of (seed, stream, counter); arrays broadcast."""
    seed = np.asarray(seed, dtype=np.uint64)
    stream = np.asarray(stream, dtype=np.uint64)
    ctr = np.asarray(ctr, dtype=np.uint64)
    with np.errstate(over="ignore"):
        a = _mix64(seed ^ (stream * _G))
        return _mix64(a + ctr * _C)


def logits_normal(seed, B, V, sd, row0=0):
    """[B, V] float32, ~N(0, sd^2): Irwin-Hall of ten 16-bit uniforms plus a
    32-bit dither, scaled by one double multiply."""
    out = np.empty((B, V), dtype=np.float32)
    K = float(sd) / (65536.0 * math.sqrt(10.0 / 12.0))
    idx = np.arange(V, dtype=np.uint64)
    for r in range(B):
        s = np.uint64(row0 + r)
        h0 = hash3(seed, s, _NORMAL + 3 * idx)
        h1 = hash3(seed, s, _NORMAL + 3 * idx + 1)
        h2 = hash3(seed, s, _NORMAL + 3 * idx + 2)
        S = np.zeros(V, dtype=np.int64)
        for h in (h0, h1):
            for sh in (0, 16, 32, 48):
                S += ((h >> np.uint64(sh)) & np.uint64(0xFFFF)).astype(np.int64)
        for sh in (0, 16):
            S += ((h2 >> np.uint64(sh)) & np.uint64(0xFFFF)).astype(np.int64)
        d = (h2 >> np.uint64(32)).astype(np.float64)
        U = S.astype(np.float64) + d * (1.0 / 4294967296.0)
        out[r] = ((U - 327675.0) * K).astype(np.float32)
    return out


def _distinct_ids(seed, row, n, V, base):
    ids, seen, c = [], set(), 0
    n = min(n, V)
    while len(ids) < n:
        t = int(hash3(seed, row, base + c) % np.uint64(V))
        c += 1
        if t not in seen:
            seen.add(t)
            ids.append(t)
    return ids


def _unit(seed, row, ctr):
    """uniform double in [0, 1) with 53 bits."""
    return float(int(hash3(seed, row, ctr)) >> 11) * (1.0 / 9007199254740992.0)


def add_boosts(x, seed, n, lo, hi, row0=0):
    """Adds U(lo, hi) to n distinct random ids of every row, in place."""
    B, V = x.shape
    for r in range(B):
        ids = _distinct_ids(seed, row0 + r, n, V, _BOOST)
        for j, t in enumerate(ids):
            b = lo + (hi - lo) * _unit(seed, row0 + r, _BOOST + (1 << 20) + j)
            x[r, t] = np.float32(float(x[r, t]) + b)
    return x


def add_zipf_boosts(x, seed, n, scale, s=1.1, row0=0):
    """Adds scale * rank^-s to n distinct random ids (a random permutation's
    first n ranks), in place."""
    B, V = x.shape
    for r in range(B):
        ids = _distinct_ids(seed, row0 + r, n, V, _BOOST)
        for j, t in enumerate(ids):
            x[r, t] = np.float32(float(x[r, t]) + scale * math.pow(j + 1, -s))
    return x


def history(seed, lengths, V, row0=0):
    """CSR history: ids uniform over [0, V).  lengths: int per row."""
    lengths = np.asarray(lengths, dtype=np.int64)
    off = np.zeros(len(lengths) + 1, dtype=np.int32)
    off[1:] = np.cumsum(lengths)
    hist = np.empty(int(off[-1]), dtype=np.int32)
    for r, H in enumerate(lengths):
        if H:
            j = np.arange(H, dtype=np.uint64)
            hist[off[r]:off[r + 1]] = (hash3(seed, row0 + r, _HIST + j) % np.uint64(V)).astype(np.int32)
    return hist, off


def to_bf16_bits(x):
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def param_uniform(seed, B, which, row0=0):
    """[B] doubles in [0,1) for per-row parameter `which`."""
    return np.array([_unit(seed, row0 + r, _PARAM + which) for r in range(B)])
