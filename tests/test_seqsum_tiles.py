"""The exact sequential-sum replay of full_kernel, restated on the CPU.

full_kernel reproduces the reference's sequential float sums (the top-p and
softmax normalisers, top_p.c:57-65 and softmax.c:12-16; the cumulative
cutoff and the draw, top_p.c:80-105; the softmax CDF walk,
generate.c:159-167) bit for bit, in parallel (pz_seqsum.cuh):

- inside a binade of the running sum s (grid u = 2^eu), adding x >= 0 is the
  map N -> N + a[N & 1] on the integer grid; the increment is rint(x/u)
  except at an exact half, where the parity of N decides;
- on a normal grid the increment is computed in float arithmetic
  (seq_elem_fast: y = x * 2^-eu, rint by adding 2^23, the half test from
  rint(y) - y), elsewhere from the bits (seq_elem);
- terms are cut into tiles of 256; a tile's composite map on the grid of
  the sum at its start is applied with one add, and since N only grows, a
  tile leaves the binade (or meets a target) iff its end does; only such
  tiles are replayed term by term, the binade-leaving term with a real add.

This checks the arithmetic and the tile walk against numpy's float32
addition on random, tied, subnormal and binade-crossing sequences.  It tests
the algorithm, not the CUDA code (the -m gpu parity tests do that)."""
import numpy as np
import pytest

F32 = np.float32
LIMIT = 1 << 24
CLAMP = 1 << 30
TILE = 256


def grid_exp(s):
    ex = (int(F32(s).view(np.uint32)) >> 23) & 0xFF
    return (1 if ex == 0 else ex) - 150


def seq_n(s):
    b = int(F32(s).view(np.uint32))
    ex, m = (b >> 23) & 0xFF, b & 0x7FFFFF
    return m if ex == 0 else m | 0x800000


def seq_float(n, eu):
    return np.uint32(((eu + 149) << 23) + n).view(F32)


def elem_exact(x, eu):
    """seq_elem: the increments (even N, odd N) from the bits of x."""
    b = int(F32(x).view(np.uint32))
    ex, M = (b >> 23) & 0xFF, b & 0x7FFFFF
    if ex == 0:
        e2 = -149
    else:
        M |= 0x800000
        e2 = ex - 150
    m, tie = 0, False
    if M:
        sh = e2 - eu
        if sh >= 0:
            m = CLAMP if sh >= 7 else min(M << sh, CLAMP)
        elif -sh < 26:
            q = -sh
            m = M >> q
            rem, half = M & ((1 << q) - 1), 1 << (q - 1)
            if rem > half:
                m += 1
            elif rem == half:
                tie = True
    if not tie:
        return m, m
    return (m + 1, m) if m & 1 else (m, m + 1)


def elem_fast(x, eu):
    """seq_elem_fast: the same increments in float arithmetic (-126 <= eu)."""
    sc = np.uint32((127 - eu) << 23).view(F32)
    with np.errstate(over="ignore", invalid="ignore"):
        y = F32(x) * sc
        r = y + F32(8388608.0)
        m = int(r.view(np.uint32)) - 0x4B000000
        d = (r - F32(8388608.0)) - y
    tie = abs(float(d)) == 0.5
    if not (y < F32(8388608.0)):
        return LIMIT, LIMIT
    if not tie:
        return m, m
    return m, (m + 1 if d < 0 else m - 1)


def compose(f, g):
    fe, fo = f
    ge, go = g
    return (min(fe + (go if fe & 1 else ge), CLAMP), min(fo + (ge if fo & 1 else go), CLAMP))


def apply(f, n):
    return n + (f[1] if n & 1 else f[0])


def seq_sum(xs, s=F32(0.0)):
    """The reference's loop: s = fl(s + x) in order."""
    out = []
    for x in xs:
        s = F32(s + F32(x))
        out.append(s)
    return out


def tile_exact(xs, s, j0=0, kind=None, target=0.0):
    """Term-by-term replay inside one tile (the device does it with a warp
    scan of the exact maps; each binade-leaving term is a real add).
    Returns (s, first j meeting the target or -1)."""
    for i, x in enumerate(xs):
        if not np.isfinite(s):
            s = F32(s + F32(x))
        else:
            eu = grid_exp(s)
            n = apply(elem_exact(x, eu), seq_n(s))
            s = F32(s + F32(x)) if n >= LIMIT else seq_float(n, eu)
        if meets(s, kind, target):
            return s, j0 + i
    return s, -1


def meets(s, kind, target):
    return (kind == "ge" and s >= target) or (kind == "gt" and s > target)


def thr_n(kind, target, eu):
    if kind is None:
        return 1 << 32
    q = float(target) * 2.0 ** -eu
    return max(0, int(np.ceil(q))) if kind == "ge" else max(0, int(np.floor(q)) + 1)


def tile_walk(xs, head=1024, kind=None, target=0.0):
    """seq_scan: the head in order; then tile sums, a prefix from the head's
    exact sum that predicts each tile's grid, maps on the predicted grids,
    and the walk (a tile whose prediction is the current grid costs one add
    unless its end leaves the binade or meets the target; any other tile is
    replayed exactly).  Returns (s, hit, stats)."""
    s, hit = F32(0.0), -1
    for j, x in enumerate(xs[:head]):
        s = F32(s + F32(x))
        if meets(s, kind, target):
            return s, j, {"tiles": 0, "replayed": 0}
    starts = list(range(head, len(xs), TILE))
    tsum = [float(np.sum(xs[t:t + TILE], dtype=F32)) for t in starts]
    pre = float(s) + np.concatenate([[0.0], np.cumsum(tsum)[:-1]]) if starts else []
    pred = [grid_exp(F32(p)) for p in pre]
    stats = {"tiles": len(starts), "replayed": 0}
    for t, j0 in enumerate(starts):
        tile = xs[j0:j0 + TILE]
        if not np.isfinite(s):
            if meets(s, kind, target):
                return s, j0, stats
            s = F32(s + F32(np.sum(tile)))  # stays NaN or inf
            continue
        eu = grid_exp(s)
        if pred[t] == eu:
            f = (0, 0)
            for x in tile:
                f = compose(f, elem_fast(x, eu) if eu >= -126 else elem_exact(x, eu))
            n = apply(f, seq_n(s))
            if n < LIMIT and n < thr_n(kind, target, eu):
                s = seq_float(n, eu)
                continue
        stats["replayed"] += 1
        s, hit = tile_exact(tile, s, j0, kind, target)
        if hit >= 0:
            return s, hit, stats
    return s, -1, stats


def first_hit(xs, kind, target):
    s = F32(0.0)
    for j, x in enumerate(xs):
        s = F32(s + F32(x))
        if meets(s, kind, target):
            return s, j
    return s, -1


def test_fast_map_equals_exact_map_and_float_addition():
    rng = np.random.default_rng(11)
    checked = ties = 0
    for _ in range(4000):
        s = F32(np.exp2(rng.uniform(-100, 20)) * rng.uniform(1, 2))
        eu = grid_exp(s)
        u = 2.0 ** eu
        cands = [F32(u * rng.uniform(0, 3)), F32(u * (rng.integers(0, 40) + 0.5)),
                 F32(u * 0.5), F32(u * rng.uniform(0, 1e-3)), F32(s * rng.uniform(0, 2)),
                 F32(u * rng.integers(1, 1000)), F32(0.0), F32(u * 2.0 ** 23 * rng.uniform(0.9, 1.1))]
        for x in cands:
            fe, fo = elem_exact(x, eu)
            ge, go = elem_fast(x, eu)
            if fe < (1 << 23):
                assert (fe, fo) == (ge, go), (s, x, eu)
            else:
                assert ge >= (1 << 23)  # the fast map reports "leaves the binade"
            n = seq_n(s)
            n2 = apply((ge, go), n)
            if n2 < LIMIT:
                assert seq_float(n2, eu) == F32(s + x), (s, x)
                checked += 1
            else:  # reported as leaving the binade: it does
                assert grid_exp(F32(s + x)) > eu, (s, x)
            ties += fe != fo
    assert checked > 20000 and ties > 3000


def _seq(kind, rng, n):
    if kind == "exp":  # softmax numerators of N(0, 2^2) logits
        v = rng.normal(0, 2, n).astype(F32)
        return np.exp((v - v.max()).astype(np.float64)).astype(F32)
    if kind == "ties":  # terms on a coarse grid: many exact halves
        return (rng.integers(0, 64, n) * 2.0 ** -12).astype(F32)
    if kind == "sorted":  # sorted probabilities (the cutoff and draw sums)
        p = rng.dirichlet(np.full(n, 0.3)).astype(F32)
        return np.sort(p)[::-1].copy()
    if kind == "tiny":  # subnormal and tiny terms, then large ones
        a = (rng.uniform(0, 1, n) * 2.0 ** -140).astype(F32)
        a[n // 2:] = rng.uniform(0, 1, n - n // 2).astype(F32)
        return a
    if kind == "zeros_then_one":
        a = np.zeros(n, F32)
        a[-300] = 1.0
        a[-299:] = F32(2.0 ** -25)
        return a
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["exp", "ties", "sorted", "tiny", "zeros_then_one"])
def test_tile_walk_equals_sequential_sum(kind):
    rng = np.random.default_rng(sum(map(ord, kind)))
    for n in (1000, 1024, 1300, 9000, 40000):
        xs = _seq(kind, rng, n)
        want = seq_sum(xs)[-1]
        got, _, st = tile_walk(xs)
        assert got.view(np.uint32) == want.view(np.uint32), (kind, n, got, want)
        if n > 1024 + TILE:
            assert st["tiles"] > st["replayed"]
        # after the head the sum leaves its binade a few times at most
        assert st["replayed"] <= 12 or kind == "tiny", st


def test_tile_walk_nan_and_inf():
    xs = np.ones(3000, F32)
    xs[2000] = np.nan
    assert np.isnan(tile_walk(xs)[0])
    xs = np.full(3000, F32(3e38))
    assert tile_walk(xs)[0] == np.inf


@pytest.mark.parametrize("kind", ["exp", "ties", "sorted"])
def test_tile_walk_first_hit(kind):
    """Targets: the cutoff (s >= p), the draws (s > r); the hit and the sum
    at the hit are the reference loop's."""
    rng = np.random.default_rng(7 + len(kind))
    for n in (5000, 30000):
        xs = _seq(kind, rng, n)
        total = float(seq_sum(xs)[-1])
        for frac in (0.001, 0.3, 0.9, 0.999999, 1.0, 1.5):
            for k in ("ge", "gt"):
                target = F32(total * frac)
                want_s, want_j = first_hit(xs, k, target)
                got_s, got_j, _ = tile_walk(xs, kind=k, target=target)
                assert got_j == want_j, (kind, n, frac, k)
                assert got_s.view(np.uint32) == want_s.view(np.uint32)
