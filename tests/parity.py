"""Boundary-case proof for sampled ids that differ from the oracle.

north_star: sampled ids must be identical except where the uniform draw
falls within 1e-6 of a CDF boundary, and such cases are counted.  For a row
whose GPU token differs from the oracle's, the oracle's traced walk
(pzo_row_trace: the ids in walk order, the running float CDF the reference
compares the draw with, the draw as compared) shows where each token sits;
the mismatch is a boundary case when every CDF edge between the two walk
positions lies within 1e-6 (relative to the walk's total mass) of the draw.
Anything else is a wrong token.
"""
from __future__ import annotations

import numpy as np

DRAW_RTOL = 1e-6


def walk_position(cdf, r):
    """Walk position the draw r selects: the first j with r < cdf[j], or
    len(cdf) (the fallback) when r reaches past the last edge."""
    hit = np.nonzero(r < cdf)[0]
    return int(hit[0]) if hit.size else len(cdf)


def is_boundary(order, cdf, r, fallback, tok_gpu, rtol=DRAW_RTOL):
    """True when tok_gpu sits at a walk position that the oracle's draw r
    reaches by crossing only CDF edges within rtol * total of r."""
    n = len(cdf)
    if n == 0:
        return False  # no draw (argmax): ids must match exactly
    total = float(cdf[-1])
    po = walk_position(cdf, r)
    cands = [int(j) for j in np.nonzero(order == tok_gpu)[0]]
    if tok_gpu == fallback:
        cands.append(n)
    for pg in cands:
        lo, hi = min(po, pg), max(po, pg)
        edges = cdf[lo:hi].astype(np.float64)
        if np.all(np.abs(float(r) - edges) <= rtol * total):
            return True
    return False


def row_inputs(d, row):
    """(logits row, config, rng state, history ids) of one row of a case dict."""
    h = None
    if d.get("hist") is not None:
        h = d["hist"][d["hist_off"][row]:d["hist_off"][row + 1]]
    return d["logits"][row], d["cfg"][row], int(d["rng"][row]), h


def boundary_rows(oracle_lib, d, tok_oracle, tok_gpu, rows=None):
    """Checks every mismatching row; returns (n_boundary, wrong) where wrong
    lists the rows whose mismatch is not a boundary case."""
    rows = np.nonzero(tok_oracle != tok_gpu)[0] if rows is None else rows
    wrong = []
    for r in rows:
        x, cfg, rng, h = row_inputs(d, int(r))
        tok, draw, order, cdf, fb = oracle_lib.row_trace(x, cfg, rng, h)
        assert tok == int(tok_oracle[r]), f"trace of row {r} disagrees with the batch oracle"
        if not is_boundary(order, cdf, draw, fb, int(tok_gpu[r])):
            wrong.append(int(r))
    return len(rows) - len(wrong), wrong
