"""The boundary-case proof of tests/parity.py, on the CPU: the oracle's traced
walk agrees with its batch result, a token one walk position away from the
draw is accepted only when the draw sits within 1e-6 of the edge between
them, and any other token is rejected."""
import numpy as np

import cases
from parity import DRAW_RTOL, boundary_rows, is_boundary, row_inputs, walk_position


def test_walk_positions_and_synthetic_edges():
    order = np.array([5, 9, 2, 7], dtype=np.int32)
    cdf = np.array([0.4, 0.7, 0.9, 1.0], dtype=np.float32)
    assert walk_position(cdf, np.float32(0.1)) == 0
    assert walk_position(cdf, np.float32(0.4)) == 1   # r < cdf is strict
    assert walk_position(cdf, np.float32(1.0)) == 4   # past the end: fallback
    r = np.float32(0.7) - np.float32(2e-7)            # just below the edge 0.7
    assert is_boundary(order, cdf, r, 5, 2)            # next position: one edge within 1e-6
    assert not is_boundary(order, cdf, r, 5, 7)        # two positions away: edge 0.9 is far
    assert not is_boundary(order, cdf, np.float32(0.55), 5, 2)
    assert not is_boundary(order, cdf, r, 5, 123)      # not in the walk at all
    # the fallback (id 5 = walk position 0 and past-the-end) next to the last edge
    assert is_boundary(order, cdf, np.float32(1.0), 5, 7)
    assert is_boundary(order, cdf, np.float32(0.99999994), 5, 5)
    assert not is_boundary(np.zeros(0, np.int32), np.zeros(0, np.float32), 0.0, -1, 3)


def _case(name):
    return cases.build(cases.PIPELINE_SPECS[name])


def test_trace_agrees_with_the_batch_oracle(oracle_lib):
    for name in ("c1_k40_p95", "c3_full", "c4_hetero", "softmax_full", "topk_only", "small_v_full"):
        d = _case(name)
        tok, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        for r in range(len(tok)):
            x, cfg, rng, h = row_inputs(d, r)
            t, draw, order, cdf, fb = oracle_lib.row_trace(x, cfg, rng, h)
            assert t == tok[r], (name, r)
            if len(cdf):
                pos = walk_position(cdf, draw)
                assert (order[pos] if pos < len(order) else fb) == t, (name, r)


def test_planted_wrong_tokens_are_rejected(oracle_lib):
    """A planted mistake (the oracle's token swapped for a neighbour in the
    walk, or for an id outside it) is caught unless the draw really sits on
    the edge between them."""
    d = _case("c3_full")
    tok, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
    planted = tok.copy()
    checked = 0
    for r in range(len(tok)):
        x, cfg, rng, h = row_inputs(d, r)
        t, draw, order, cdf, fb = oracle_lib.row_trace(x, cfg, rng, h)
        pos = walk_position(cdf, draw)
        nb = pos + 1 if pos + 1 < len(order) else pos - 1
        if nb < 0:
            continue
        edge = cdf[min(pos, nb)]
        near = abs(float(draw) - float(edge)) <= DRAW_RTOL * float(cdf[-1])
        assert is_boundary(order, cdf, draw, fb, int(order[nb])) == near
        planted[r] = order[nb]
        checked += 1
    assert checked > 0
    n_ok, wrong = boundary_rows(oracle_lib, d, tok, planted)
    assert len(wrong) == checked - n_ok and len(wrong) > 0
    planted = tok.copy()
    planted[0] = -5
    assert boundary_rows(oracle_lib, d, tok, planted)[1] == [0]
