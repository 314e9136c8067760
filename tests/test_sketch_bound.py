"""The list path's exactness argument, restated on the CPU.

For list rows (k <= 64) slice_kernel keeps only a sketch of the stream: per
group of 4 lanes' vectors (64 f32 elements: 16 contiguous columns at each of
4 places 128 columns apart in a 512-column chunk; 128 bf16 elements in a
1024-column chunk) the top 16 bits of the
ordered value of the group's largest raw logit.  The bound is the k-th
largest sketch value (k + 8 in a first pass when the row has history ids);
`tb`, its tempered floor.  Candidates are the elements at or above `tb` of
the groups whose largest value can temper to `tb` or above, with penalties
applied only to values that reach `tb` unpenalised (penalties that can only
lower a value), or every history id scored apart (other penalties); a
second pass bounds with the groups holding no history id when the first
finds fewer than k candidates.

Lists longer than 64 (slice_long_kernel) keep a finer sketch: one entry per
lane and 16 elements of a chunk (a lane's four f32 vectors, or two of its
four bf16 vectors), up to 4096 candidate entries and 2048 candidates; the
rest of the argument is the same (`fine=True` below).

This restatement checks, on random and adversarial rows, that the exact
top-k of the row (the reference's ranking: value descending, lower index
first) is always among the candidates, which is what makes the device's
list exact.  It tests the algorithm, not the CUDA code (the -m gpu parity
tests do that)."""
import numpy as np
import pytest

F32 = np.float32
ORD_NEG_INF = 0x007FFFFF


def f2ord(v):
    u = np.asarray(v, dtype=F32).view(np.uint32).copy()
    u[u == 0x80000000] = 0
    neg = (u & 0x80000000) != 0
    return np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def ord2f(o):
    o = np.asarray(o, dtype=np.uint32)
    u = np.where((o & 0x80000000) != 0, o & np.uint32(0x7FFFFFFF), ~o).astype(np.uint32)
    return u.view(F32)


def temper(x, T, divide):
    x = np.asarray(x, dtype=F32)
    if divide:
        return (x / F32(T)).astype(F32)
    return (x * (F32(1.0) / F32(T))).astype(F32)


def penalize(x, c, rep, freq, pres):
    v = np.asarray(x, dtype=F32)
    if rep != 1.0:
        v = np.where(v > 0, v / F32(rep), v * F32(rep)).astype(F32)
    pen = (F32(c) * F32(freq)).astype(F32) + F32(pres)
    return (v - F32(pen)).astype(F32)


def groups_of(V, vec=4, fine=False):
    """Column lists of the sketch groups of a row starting 16-byte aligned
    (vec = 4 f32 or 8 bf16 values per 16-byte vector; a chunk is 2 KB).
    fine: one group per lane and 16 elements (entry j of lane l holds the
    lane's vectors j*vpe .. j*vpe+vpe-1, vector u of lane l being the
    chunk's vector u*32+l)."""
    out = []
    per_chunk = 2048 // (16 // vec)
    if fine:
        vpe = 16 // vec
        for c in range((V + per_chunk - 1) // per_chunk):
            for lane in range(32):
                for j in range(4 // vpe):
                    cols = []
                    for u in range(j * vpe, (j + 1) * vpe):
                        base = c * per_chunk + (u * 32 + lane) * vec
                        cols.extend(range(base, base + vec))
                    cols = [q for q in cols if q < V]
                    out.append(np.array(cols, dtype=np.int64))
        return out
    for c in range((V + per_chunk - 1) // per_chunk):
        for p in range(8):
            cols = []
            for u in range(4):
                base = c * per_chunk + (u * 32 + 4 * p) * vec
                cols.extend(range(base, base + 4 * vec))
            cols = [j for j in cols if j < V]
            out.append(np.array(cols, dtype=np.int64))
    return out


def kth_largest(vals, k):
    vals = np.sort(np.asarray(vals, dtype=np.int64))[::-1]
    return int(vals[k - 1]) if len(vals) >= k else 0


def candidates(x, k, hist, T, divide, rep, freq, pres, vec=4, fine=False):
    """The list path's candidate columns for one row (None: overflow, the
    device redoes the slice exactly)."""
    V = len(x)
    grp = groups_of(V, vec, fine)
    gcap, ccap = (4096, 2048) if fine else (1024, 2048)
    counts = {}
    for h in hist:
        counts[int(h)] = counts.get(int(h), 0) + 1
    hist_on = len(counts) > 0
    pen_dec = rep >= 1.0 and freq >= 0.0 and pres >= 0.0
    sk = []
    for cols in grp:
        vals = x[cols]
        vals = vals[~np.isnan(vals)]
        sk.append(int(f2ord(vals.max())) >> 16 if len(vals) else 0)
    sk = np.array(sk, dtype=np.int64)
    hgroup = np.array([any(int(j) in counts for j in cols) for cols in grp])
    ord_inf = int(f2ord(np.float32(np.inf)))
    for pas in (0, 1):
        elig = (sk != 0) if pas == 0 else ((sk != 0) & ~hgroup)
        kb = k + 8 if (pas == 0 and hist_on) else k
        b16 = kth_largest(sk[elig], kb)
        bord = b16 << 16
        tb = temper(ord2f(bord), T, divide) if bord > ORD_NEG_INF else F32(-np.inf)
        up = np.minimum((sk << 16) | 0xFFFF, ord_inf)
        sel = (sk != 0) & ~(temper(ord2f(up), T, divide) < tb)
        if sel.sum() > gcap:
            return None
        cand = set()
        for g in np.nonzero(sel)[0]:
            for j in grp[g]:
                v = temper(x[j], T, divide)
                if not (v >= tb):
                    continue
                if int(j) in counts:
                    if not pen_dec:
                        continue
                    v = temper(penalize(x[j], counts[int(j)], rep, freq, pres), T, divide)
                    if not (v >= tb):
                        continue
                cand.add(int(j))
        if hist_on and not pen_dec:
            for j, c in counts.items():
                v = temper(penalize(x[j], c, rep, freq, pres), T, divide)
                if v >= tb:
                    cand.add(j)
        if len(cand) > ccap:
            return None
        if len(cand) >= k or not hist_on or b16 == 0:
            return cand
    return cand


def exact_topk(x, k, hist, T, divide, rep, freq, pres):
    counts = {}
    for h in hist:
        counts[int(h)] = counts.get(int(h), 0) + 1
    v = x.astype(F32).copy()
    for j, c in counts.items():
        v[j] = penalize(x[j], c, rep, freq, pres)
    v = temper(v, T, divide)
    idx = np.nonzero(~np.isnan(v))[0]
    order = sorted(idx.tolist(), key=lambda j: (-float(v[j]), j))
    return set(order[:k])


def make_row(rs, V, kind):
    x = (rs.standard_normal(V) * 2.5).astype(F32)
    if kind == "boosted":
        pos = rs.choice(V, 8, replace=False)
        x[pos] += rs.uniform(5, 15, 8).astype(F32)
    elif kind == "ties":
        x = (np.round(x * 2) / 2).astype(F32)
    elif kind == "negative":
        x = (-np.abs(x) - 1).astype(F32)
    elif kind == "nan":
        x[rs.choice(V, 200, replace=False)] = np.nan
    elif kind == "crowded":
        # the large values all in the same lanes of every chunk
        for c in range(V // 512):
            x[c * 512 + np.arange(4) * 128 + 3] = F32(9.0 + 0.01 * c)
    return x


KINDS = ["plain", "boosted", "ties", "negative", "nan", "crowded"]


def to_bf16_values(x):
    """bf16 logits as the kernel widens them (round to nearest even)."""
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(np.isnan(x), 0x7FC0, r).astype(np.uint32)
    return (r << 16).astype(np.uint32).view(F32)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("kind", KINDS)
def test_exact_list_is_among_candidates(kind, dtype):
    rs = np.random.default_rng(100 + KINDS.index(kind) + (50 if dtype == "bf16" else 0))
    V = 5000
    vec = 4 if dtype == "f32" else 8
    for trial in range(12):
        x = make_row(rs, V, kind)
        if dtype == "bf16":
            x = to_bf16_values(x)
        k = int(rs.choice([2, 8, 50, 64]))
        T = float(rs.choice([0.3, 0.7, 1.5]))
        divide = bool(trial % 2)
        mode = trial % 3
        if mode == 0:
            hist, rep, freq, pres = [], 1.0, 0.0, 0.0
        else:
            top = np.argsort(-np.nan_to_num(x, nan=-np.inf))[:80]
            hist = list(rs.choice(V, 60)) + list(top[: 40 if mode == 1 else 10])
            rep, freq, pres = (3.0, 0.5, 0.2) if mode == 1 else (0.8, 0.0, -0.5)
        cand = candidates(x, k, hist, T, divide, rep, freq, pres, vec)
        if cand is None:
            continue  # overflow: the device redoes the slice exactly
        want = exact_topk(x, k, hist, T, divide, rep, freq, pres)
        assert want <= cand, (kind, trial, sorted(want - cand)[:5])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("kind", KINDS)
def test_exact_long_list_is_among_candidates(kind, dtype):
    """Lists of 65 to 1024 entries through the fine sketch."""
    rs = np.random.default_rng(300 + KINDS.index(kind) + (50 if dtype == "bf16" else 0))
    vec = 4 if dtype == "f32" else 8
    n_checked = 0
    for trial in range(6):
        k = int(rs.choice([65, 200, 1024]))
        V = 60000 if k == 1024 else (20000 if trial % 2 else 6000)
        x = make_row(rs, V, kind)
        if dtype == "bf16":
            x = to_bf16_values(x)
        T = float(rs.choice([0.3, 0.7, 1.5]))
        divide = bool(trial % 2)
        mode = trial % 3
        if mode == 0:
            hist, rep, freq, pres = [], 1.0, 0.0, 0.0
        else:
            top = np.argsort(-np.nan_to_num(x, nan=-np.inf))[:1200]
            hist = list(rs.choice(V, 300)) + list(top[: 600 if mode == 1 else 100])
            rep, freq, pres = (3.0, 0.5, 0.2) if mode == 1 else (0.8, 0.0, -0.5)
        cand = candidates(x, k, hist, T, divide, rep, freq, pres, vec, fine=True)
        if cand is None:
            continue  # overflow: the device redoes the slice exactly
        n_checked += 1
        want = exact_topk(x, k, hist, T, divide, rep, freq, pres)
        assert want <= cand, (kind, trial, sorted(want - cand)[:5])
    assert n_checked > 0
