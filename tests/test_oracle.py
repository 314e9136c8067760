"""The CPU checker itself, pinned before anything is compared against it:
restatement == golden vectors produced by the reference's own compiled
sampler; the reference's unit/property tests (tests/test_sampling.c,
tests/test_bugfixes.c) replayed on it; the penalty contract by hand."""
import math

import numpy as np
import pytest

import cases
import oracle
import synth


def test_pipeline_golden(oracle_lib, golden):
    for case in golden["pipeline"]:
        d = cases.build(case["spec"])
        tok, rng, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        assert tok.tolist() == case["tokens"], case["name"]
        assert [int(v) for v in rng] == case["rng_out"], case["name"]


def test_edge_golden(oracle_lib, golden):
    want = {c["name"]: c for c in golden["edge"]}
    for name, x, cfg, rng in cases.edge_rows():
        tok, r, *_ = oracle_lib.sample_batch(x, cfg, rng)
        assert tok.tolist() == want[name]["tokens"], name
        assert [int(v) for v in r] == want[name]["rng_out"], name


def test_legacy_known_answers(oracle_lib, golden):
    L = golden["legacy"]
    for seed, rec in L["rng"].items():
        s = oracle_lib.rng_seed(int(seed))
        for bits in rec["float_bits"]:
            v, s = oracle_lib.rng_float(s)
            assert int(np.float32(v).view(np.uint32)) == bits
        assert s == rec["final"]
    for vals, want in L["argmax"]:
        assert oracle_lib.sample_argmax(vals) == want
    for rec in L["top_k"]:
        s = oracle_lib.rng_seed(rec["seed"])
        got = []
        for _ in rec["tokens"]:
            t, s = oracle_lib.sample_top_k(rec["logits"], rec["k"], s)
            got.append(t)
        assert got == rec["tokens"] and s == rec["final"]
    for rec in L["top_p"]:
        s = oracle_lib.rng_seed(rec["seed"])
        got = []
        for _ in rec["tokens"]:
            t, s = oracle_lib.sample_top_p(rec["logits"], rec["p"], s)
            got.append(t)
        assert got == rec["tokens"] and s == rec["final"]
    for rec in L["temperature"]:
        y = oracle_lib.apply_temperature(rec["logits"], rec["T"])
        assert [int(b) for b in y.view(np.uint32)] == rec["bits"]


def test_rng_can_return_exactly_one(oracle_lib, golden):
    # rng.c:16 converts a 31-bit integer with rounding: 2^31-1 rounds to 2^31
    s = golden["legacy"]["rng_one_state"]
    v, _ = oracle_lib.rng_float(s)
    assert v == 1.0
    for rec in golden["legacy"]["draw_one"]:
        vals = rec["logits"]
        if rec["kind"] == "top_k":
            t, s2 = oracle_lib.sample_top_k(vals, rec["arg"], s)
        elif rec["kind"] == "top_p":
            t, s2 = oracle_lib.sample_top_p(vals, rec["arg"], s)
        else:
            t, s2, _ = oracle_lib.sample_softmax(vals, s)
        assert (t, s2) == (rec["token"], rec["final"]), rec["kind"]


# ---- the reference's own tests (tests/test_sampling.c:24-245) -------------
def test_ref_rng_properties(oracle_lib):
    s = oracle_lib.rng_seed(42)
    for _ in range(1000):
        v, s = oracle_lib.rng_float(s)
        assert 0.0 <= v < 1.0
    a = oracle_lib.rng_seed(12345)
    b = oracle_lib.rng_seed(12345)
    for _ in range(100):
        va, a = oracle_lib.rng_float(a)
        vb, b = oracle_lib.rng_float(b)
        assert va == vb
    a, b = oracle_lib.rng_seed(111), oracle_lib.rng_seed(222)
    diff = False
    for _ in range(10):
        va, a = oracle_lib.rng_float(a)
        vb, b = oracle_lib.rng_float(b)
        diff |= abs(va - vb) > 1e-9
    assert diff
    v, _ = oracle_lib.rng_float(oracle_lib.rng_seed(0))
    assert 0.0 <= v < 1.0


def test_ref_argmax_and_temperature(oracle_lib):
    assert oracle_lib.sample_argmax([1.0, 3.0, 2.0, 0.5]) == 1
    assert oracle_lib.sample_argmax([10.0, 3.0, 2.0, 0.5]) == 0
    assert oracle_lib.sample_argmax([1.0, 2.0, 3.0, 100.0]) == 3
    assert oracle_lib.sample_argmax([-5.0, -1.0, -3.0, -2.0]) == 1
    assert oracle_lib.sample_argmax([42.0]) == 0
    np.testing.assert_allclose(oracle_lib.apply_temperature([2, 4, 6, 8], 2.0), [1, 2, 3, 4], atol=1e-6)
    np.testing.assert_allclose(oracle_lib.apply_temperature([1, 2, 3], 1.0), [1, 2, 3], atol=1e-6)
    np.testing.assert_allclose(oracle_lib.apply_temperature([1, 2, 3], 0.5), [2, 4, 6], atol=1e-6)
    assert oracle_lib.sample_argmax(oracle_lib.apply_temperature([1, 5, 3, 2], 0.7)) == 1


def test_ref_top_p_and_top_k_properties(oracle_lib):
    s = oracle_lib.rng_seed(42)
    for _ in range(20):
        t, s = oracle_lib.sample_top_p([-100.0, 100.0, -100.0, -100.0], 0.5, s)
        assert t == 1
    s = oracle_lib.rng_seed(42)
    seen = set()
    for _ in range(200):
        t, s = oracle_lib.sample_top_p([0.0] * 4, 1.0, s)
        assert 0 <= t < 4
        seen.add(t)
    assert len(seen) >= 3
    s = oracle_lib.rng_seed(42)
    for _ in range(20):
        t, s = oracle_lib.sample_top_k([1.0, 5.0, 3.0, 2.0], 1, s)
        assert t == 1
    for _ in range(50):
        t, s = oracle_lib.sample_top_k([1.0, 10.0, 100.0, 0.1], 2, s)
        assert t in (1, 2)
    t, s = oracle_lib.sample_top_k([1.0, 2.0], 100, s)
    assert 0 <= t < 2
    # tests/test_bugfixes.c:35-92 (QA-BUG-001)
    for vals, k in [(list(range(32)), 5000), ([i % 100 for i in range(2048)], 1024),
                    ([(i % 50) * 0.1 for i in range(4096)], 2000), (list(range(1, 9)), 0),
                    (list(range(1, 9)), -5)]:
        t, _ = oracle_lib.sample_top_k([float(v) for v in vals], k, oracle_lib.rng_seed(1))
        assert 0 <= t < len(vals)


# ---- pipeline contract pieces --------------------------------------------
def test_penalty_contract(oracle_lib):
    x = np.array([2.0, -2.0, 0.5, 3.0, -0.0], dtype=np.float32)
    y = oracle_lib.apply_penalties(x, [0, 1, 1, 3, 3, 3, 7, -1, 4], 1.25, 0.5, 0.25)
    f = np.float32
    assert y[0] == f(f(f(2.0) / f(1.25)) - f(f(1 * f(0.5)) + f(0.25)))
    assert y[1] == f(f(f(-2.0) * f(1.25)) - f(f(2 * f(0.5)) + f(0.25)))
    assert y[2] == x[2]
    assert y[3] == f(f(f(3.0) / f(1.25)) - f(f(3 * f(0.5)) + f(0.25)))
    assert y[4] == f(f(f(-0.0) * f(1.25)) - f(f(1 * f(0.5)) + f(0.25)))
    # no penalty settings: identity
    assert (oracle_lib.apply_penalties(x, [0, 1, 2], 1.0, 0.0, 0.0).view(np.uint32) == x.view(np.uint32)).all()


def test_pipeline_reduces_to_reference_sequence(oracle_lib):
    """k=0, no history, fp32: the pipeline IS generate.c:151-170."""
    x = synth.logits_normal(99, 3, 5000, 2.0)
    for T, p in [(0.8, 0.9), (1.1, 1.0), (0.0, 0.9)]:
        cfg = cases.configs(3, temperature=T, top_p=p)
        rng = np.array([5, 6, 7], dtype=np.uint64)
        tok, r, *_ = oracle_lib.sample_batch(x, cfg, rng)
        for i in range(3):
            if T == 0.0:
                assert tok[i] == oracle_lib.sample_argmax(x[i])
                assert r[i] == rng[i]
                continue
            y = oracle_lib.apply_temperature(x[i], T)
            if p < 1.0:
                t, s = oracle_lib.sample_top_p(y, p, int(rng[i]))
            else:
                t, s, _ = oracle_lib.sample_softmax(y, int(rng[i]))
            assert (tok[i], int(r[i])) == (t, s)


def test_bf16_widening_is_exact(oracle_lib):
    x = synth.logits_normal(5, 2, 3000, 2.0)
    b = synth.to_bf16_bits(x)
    w = synth.bf16_bits_to_f32(b)
    cfg = cases.configs(2, temperature=0.9, top_k=30, top_p=0.9)
    rng = np.array([1, 2], dtype=np.uint64)
    a = oracle_lib.sample_batch(b, cfg, rng, cand_stride=32)
    c = oracle_lib.sample_batch(w, cfg, rng, cand_stride=32)
    assert (a[0] == c[0]).all() and (a[2] == c[2]).all()


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")
def test_restatement_matches_reference_random(oracle_lib):
    R = oracle.Reference()
    rs = np.random.default_rng(3)
    for trial in range(30):
        V = int(rs.integers(1, 3000))
        B = 4
        spec = dict(seed=100 + trial, B=B, V=V, sd=float(rs.uniform(0.3, 4.0)),
                    boosts=[min(4, V), 1.0, 8.0], hist_len=int(rs.integers(0, 50)),
                    cfg=dict(temperature=float(rs.choice([0.0, 0.3, 0.9, 1.7])),
                             top_k=int(rs.choice([0, 1, 5, 40, V, V + 3, -1])),
                             top_p=float(rs.choice([0.3, 0.9, 1.0, 0.0])),
                             rep=float(rs.choice([1.0, 1.2])), freq=float(rs.choice([0.0, 0.3])),
                             pres=float(rs.choice([0.0, 0.2]))),
                    dtype=str(rs.choice(["f32", "bf16"])))
        d = cases.build(spec)
        a = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        b = R.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
        assert (a[0] == b[0]).all() and (a[1] == b[1]).all(), spec


def test_reference_probability_error_is_as_surveyed(oracle_lib):
    """The reference's sequential float normaliser is off by ~1e-4 relative
    on full-vocab rows; the kernels therefore replay it exactly instead of
    reducing in a tree."""
    x = synth.logits_normal(1, 1, 128256, 2.5)[0] / np.float32(0.8)
    m = x.max()
    e = np.exp((x - m).astype(np.float32)).astype(np.float32)
    s32 = np.float32(0)
    for v in e[:20000]:
        s32 = np.float32(s32 + v)
    s64 = float(np.sum(e[:20000].astype(np.float64)))
    assert abs(float(s32) - s64) / s64 > 1e-7
    assert math.isfinite(s64)
