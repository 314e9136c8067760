"""Parity of the CUDA sampler (through the C ABI) with the reference.

Bar: greedy ids and top-k id sets bit-exact;
post-penalty probabilities within 1e-6 relative; sampled ids identical
except draws within 1e-6 of a CDF boundary (counted; the golden cases and
the full-size config-3 batch must have none)."""
import numpy as np
import pytest

import cases
import synth
from gpu_helpers import compare_with_oracle, run_gpu

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6


@pytest.mark.parametrize("name", list(cases.PIPELINE_SPECS))
def test_golden_pipeline(cuda, pz, golden, oracle_lib, name):
    case = next(c for c in golden["pipeline"] if c["name"] == name)
    d = cases.build(case["spec"])
    g = run_gpu(cuda, pz, d)
    assert g["tokens"].tolist() == case["tokens"]
    assert [int(v) for v in g["rng"]] == case["rng_out"]
    assert (g["status"] == 0).all()
    mism, _, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label=f"golden {name}")
    assert mism == 0


def test_edge_rows(cuda, pz, golden):
    want = {c["name"]: c for c in golden["edge"]}
    s = pz.Sampler(0, max_batch=4, max_vocab=64, max_top_k=1024, max_history=0)
    for name, x, cfg, rng in cases.edge_rows():
        g = run_gpu(cuda, pz, dict(logits=x, cfg=cfg, rng=rng, hist=None, hist_off=None), sampler=s)
        assert g["tokens"].tolist() == want[name]["tokens"], name
        assert [int(v) for v in g["rng"]] == want[name]["rng_out"], name
    s.close()


def test_legacy_six_calls(cuda, pz, golden):
    L = golden["legacy"]
    for vals, want in L["argmax"]:
        assert pz.sample_argmax(vals) == want
    for rec in L["top_k"]:
        s = pz.rng_seed(rec["seed"])
        got = []
        for _ in rec["tokens"]:
            t, s = pz.sample_top_k(rec["logits"], rec["k"], s)
            got.append(t)
        assert got == rec["tokens"] and s == rec["final"], rec["k"]
    for rec in L["top_p"]:
        s = pz.rng_seed(rec["seed"])
        got = []
        for _ in rec["tokens"]:
            t, s = pz.sample_top_p(rec["logits"], rec["p"], s)
            got.append(t)
        assert got == rec["tokens"] and s == rec["final"], rec["p"]
    for rec in L["temperature"]:
        y = pz.apply_temperature(np.array(rec["logits"], dtype=np.float32), rec["T"])
        assert [int(b) for b in y.view(np.uint32)] == rec["bits"]


def test_draw_of_exactly_one(cuda, pz, golden):
    s1 = golden["legacy"]["rng_one_state"]
    for rec in golden["legacy"]["draw_one"]:
        if rec["kind"] == "top_k":
            t, s = pz.sample_top_k(rec["logits"], rec["arg"], s1)
        elif rec["kind"] == "top_p":
            t, s = pz.sample_top_p(rec["logits"], rec["arg"], s1)
        else:
            t, s = pz.sample_softmax(rec["logits"], s1)
        assert (t, s) == (rec["token"], rec["final"]), rec["kind"]


def test_config3_full_size(cuda, pz, oracle_lib):
    """BASELINE config 3 at its full size, every row against the oracle."""
    spec = dict(seed=31, B=1024, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=1024,
                cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1))
    d = cases.build(spec)
    g = run_gpu(cuda, pz, d, max_top_k=50, max_history=1024, no_full_vocab=True)
    mism, n, maxrel = compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label="config3 B=1024")
    print(f"config3: {mism} boundary mismatches in {n} rows, max prob rel err {maxrel:.2e}")
    assert mism == 0
    # and against the reference's own compiled sampler (oracle/_ref)
    import oracle
    if not oracle.reference_available():
        pytest.skip("the reference build (oracle/_ref) is not present")
    tok_ref, rng_ref = oracle.Reference().sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"],
                                                       d["hist_off"])
    assert (g["tokens"] == tok_ref).all()
    assert (g["rng"] == rng_ref).all()


def test_config2_full_size_greedy(cuda, pz, oracle_lib):
    spec = dict(seed=21, B=256, V=151936, sd=3.0, spike=[8.0, 20.0], cfg=dict(temperature=0.0))
    d = cases.build(spec)
    g = run_gpu(cuda, pz, d, max_top_k=1, no_full_vocab=True)
    tok, rng, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"])
    assert (g["tokens"] == tok).all()
    assert (g["rng"] == d["rng"]).all()  # greedy rows draw nothing


def test_config4_heterogeneous(cuda, pz, oracle_lib):
    spec = dict(seed=41, B=256, V=151936, sd=2.0, zipf=[256, 10.0], dtype="bf16", cfg="hetero")
    d = cases.build(spec)
    g = run_gpu(cuda, pz, d)
    mism, n, maxrel = compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label="config4 B=256")
    print(f"config4: {mism} boundary cases in {n} rows, max prob rel err {maxrel:.2e}")


def test_full_vocab_rows_exact(cuda, pz, oracle_lib):
    """k = 0 rows: top-p over the whole row and the softmax CDF walk replay
    the reference's sequential float sums exactly."""
    for spec in [dict(seed=51, B=16, V=128256, sd=2.5, boosts=[8, 5.0, 15.0],
                      cfg=dict(temperature=0.8, top_k=0, top_p=0.95)),
                 dict(seed=52, B=8, V=151936, sd=2.0, zipf=[128, 8.0], dtype="bf16",
                      cfg=dict(temperature=1.4, top_k=0, top_p=0.99)),
                 dict(seed=53, B=8, V=128256, sd=2.5, hist_len=300,
                      cfg=dict(temperature=1.0, top_k=0, top_p=1.0, rep=1.2))]:
        d = cases.build(spec)
        g = run_gpu(cuda, pz, d)
        # every mismatch is proved to be a boundary case inside; the sums
        # replay the reference's exactly, so only an expf ulp can move an edge
        compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label=f"full-vocab seed {spec['seed']}")


def test_strided_and_unaligned_rows(cuda, pz, oracle_lib):
    """Row stride > V and a base that is not 16-byte aligned exercise the
    scalar head/tail paths."""
    torch = cuda
    B, V, ld = 6, 3001, 3013
    wide = synth.logits_normal(61, B, ld, 2.0)
    cfg = cases.configs(B, temperature=0.9, top_k=17, top_p=0.9)
    rng = np.arange(1, B + 1, dtype=np.uint64)
    full = torch.from_numpy(wide).cuda()
    x = full[:, 1:1 + V]  # base offset by 4 bytes, row stride 3013
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=32, max_history=0)
    out = torch.zeros(B, dtype=torch.int32, device="cuda")
    r = torch.from_numpy(rng.view(np.int64).copy()).cuda()
    c = torch.from_numpy(np.ascontiguousarray(cfg).view(np.uint8).copy()).cuda()
    s.sample(x, c, r, out)
    torch.cuda.synchronize()
    tok, rr, *_ = oracle_lib.sample_batch(np.ascontiguousarray(wide[:, 1:1 + V]), cfg, rng)
    assert (out.cpu().numpy() == tok).all()
    assert (r.cpu().numpy().view(np.uint64) == rr).all()
    s.close()


def test_repeat_calls_are_identical(cuda, pz):
    spec = dict(seed=71, B=64, V=50000, sd=2.0, hist_len=100,
                cfg=dict(temperature=0.8, top_k=30, top_p=0.9, rep=1.2))
    d = cases.build(spec)
    s = pz.Sampler(0, max_batch=64, max_vocab=50000, max_top_k=64, max_history=128)
    a = run_gpu(cuda, pz, d, sampler=s)
    b = run_gpu(cuda, pz, d, sampler=s)
    assert (a["tokens"] == b["tokens"]).all() and (a["rng"] == b["rng"]).all()
    s.close()


def test_hint_and_limit_violations_fail_loudly(cuda, pz):
    spec = dict(seed=81, B=4, V=5000, sd=2.0, hist_len=300,
                cfg=dict(temperature=0.8, top_k=0, top_p=0.9, rep=1.2))
    d = cases.build(spec)
    g = run_gpu(cuda, pz, d, no_full_vocab=True)
    assert (g["tokens"] == -1).all() and (g["status"] == pz.PZ_ROW_HINT_VIOLATED).all()
    g = run_gpu(cuda, pz, d, max_history=128)
    assert (g["tokens"] == -1).all() and (g["status"] == pz.PZ_ROW_HISTORY_TOO_LONG).all()
    d["cfg"]["top_k"] = 100
    g = run_gpu(cuda, pz, d, max_top_k=64)
    assert (g["tokens"] == -1).all() and (g["status"] == pz.PZ_ROW_HINT_VIOLATED).all()


def test_vocab_sharded_single_rank(cuda, pz, golden):
    """The vocab-sharded path (emit -> NCCL allgather -> merge) with one rank
    gives the golden tokens of config 5."""
    torch = cuda
    case = next(c for c in golden["pipeline"] if c["name"] == "c5_vocab")
    d = cases.build(case["spec"])
    from gpu_helpers import to_device
    x, cfg, rng, hist, hist_off = to_device(torch, d)
    B, V = x.shape
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=64, max_history=0)
    s.init_nccl(1, 0, pz.Sampler.nccl_unique_id())
    out = torch.zeros(B, dtype=torch.int32, device="cuda")
    s.sample_vocab_sharded(x, 0, V, cfg, rng, out)
    torch.cuda.synchronize()
    assert out.cpu().tolist() == case["tokens"]
    assert [int(v) for v in rng.cpu().numpy().view(np.uint64)] == case["rng_out"]
    s.close()


def test_list_values_crowded_in_few_lanes(cuda, pz, oracle_lib):
    """The list's values at positions that all fall to the same lanes of
    every chunk (one sketch group per chunk holds several of them): the
    group maxima alone undercount the list, and the re-read of the groups
    at or above the bound must still find every value of the exact list."""
    rs = np.random.default_rng(5)
    for dtype, period in [("f32", 1024), ("bf16", 2048)]:
        B, V = 4, 65536
        x = (rs.standard_normal((B, V)) * 0.5).astype(np.float32)
        for r in range(B):
            for i in range(60):
                x[r, (i * period + (i % 4)) % V] = np.float32(8.0 + 0.01 * i + r)
        logits = synth.to_bf16_bits(x) if dtype == "bf16" else x
        for k, p in [(50, 0.9), (8, 1.0), (64, 0.5)]:
            cfg = cases.configs(B, temperature=0.9, top_k=k, top_p=p)
            d = dict(logits=logits, cfg=cfg, rng=np.arange(7, 7 + B, dtype=np.uint64), hist=None,
                     hist_off=None)
            g = run_gpu(cuda, pz, d, max_top_k=64, no_full_vocab=True)
            mism, _, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL)
            assert mism == 0, (dtype, k)


def test_penalised_maximum_gives_way(cuda, pz, oracle_lib):
    """A row's largest logits are history ids whose penalty pushes them below
    their neighbours in the same 16-byte vector: the neighbours must win
    (greedy) or enter the list (top-k)."""
    rs = np.random.default_rng(11)
    B, V = 8, 8192
    for dtype in ("f32", "bf16"):
        x = (rs.standard_normal((B, V)) * 0.5).astype(np.float32)
        hist, off = [], [0]
        for r in range(B):
            p = 64 * (r + 1) + (r % 3)
            x[r, p], x[r, p + 1], x[r, 4000 + r] = 20.0, 10.0, 9.0
            ids = [p, 4000 + r] if r % 2 else [p]
            hist += ids
            off.append(len(hist))
        logits = synth.to_bf16_bits(x) if dtype == "bf16" else x
        for temp, k, p_ in [(0.0, 0, 1.0), (0.8, 3, 0.9), (0.8, 1, 1.0)]:
            cfg = cases.configs(B, temperature=temp, top_k=k, top_p=p_, rep=100.0)
            d = dict(logits=logits, cfg=cfg, rng=np.arange(3, 3 + B, dtype=np.uint64),
                     hist=np.array(hist, dtype=np.int32), hist_off=np.array(off, dtype=np.int32))
            g = run_gpu(cuda, pz, d, max_top_k=8, max_history=8)
            tok, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
            assert (g["tokens"] == tok).all(), (dtype, temp, k)
            mism, _, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL)
            assert mism == 0, (dtype, temp, k)


def test_penalties_that_raise_values(cuda, pz, oracle_lib):
    """rep < 1 and a negative presence penalty raise history logits (the
    history ids are then scored in their own round, not in the stream);
    rep >= 1 with non-negative freq/pres lower them (scored in the stream)."""
    for seed, cfg in [(91, dict(temperature=0.8, top_k=40, top_p=0.9, rep=0.7, freq=0.0, pres=-1.5)),
                      (92, dict(temperature=0.8, top_k=50, top_p=1.0, rep=1.0, freq=-0.4, pres=0.0)),
                      (93, dict(temperature=0.8, top_k=50, top_p=0.9, rep=1.3, freq=0.5, pres=0.2))]:
        for dtype in ("f32", "bf16"):
            spec = dict(seed=seed, B=64, V=50000, sd=2.0, boosts=[8, 3.0, 6.0], hist_len=400,
                        dtype=dtype, cfg=cfg)
            d = cases.build(spec)
            g = run_gpu(cuda, pz, d, max_top_k=64, max_history=512)
            mism, _, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL)
            assert mism == 0, (seed, dtype)


@pytest.mark.parametrize("B", [100, 148 + 21, 296 + 30, 444 + 30, 592 + 30, 592 + 3])
def test_last_wave_rows_split(cuda, pz, oracle_lib, B):
    """Batches on either side of the GPU's CTA slots (148 SMs x 2 to 4 CTAs):
    at half the slots or fewer, every row is split over several CTAs (slices
    of at least 128 KB, as many as fit one wave) and decided by the slice
    that finishes last; above, one CTA per row, except that argmax-only
    launches split the rows of their last, partial wave.  Mixed settings
    (greedy, top-k, top-p, k = 1024, history) cover every kind of row; a
    second call checks that the arrival counters start again."""
    spec = dict(seed=91 + B, B=B, V=50000, sd=2.0, zipf=[64, 6.0], cfg="hetero")
    d = cases.build(spec)
    s = pz.Sampler(0, max_batch=B, max_vocab=50000, max_top_k=1024, max_history=2048)
    g = run_gpu(cuda, pz, d, sampler=s)
    compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label=f"last wave B={B} hetero")
    again = run_gpu(cuda, pz, d, sampler=s)
    assert (again["tokens"] == g["tokens"]).all() and (again["rng"] == g["rng"]).all()
    spec = dict(seed=92 + B, B=B, V=50000, sd=2.0, boosts=[8, 3.0, 6.0], hist_len=200,
                cfg=dict(temperature=0.0, rep=1.3))
    d = cases.build(spec)
    g = run_gpu(cuda, pz, d, sampler=s, max_top_k=1, max_history=256)
    mism, n, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL, label=f"last wave B={B} greedy")
    assert mism == 0, (B, mism)
    again = run_gpu(cuda, pz, d, sampler=s, max_top_k=1, max_history=256)
    assert (again["tokens"] == g["tokens"]).all()
    s.close()


def test_sketch_bound_second_pass_and_overflow(cuda, pz, oracle_lib):
    """The list path's fallbacks.  Rows whose largest logits are all history
    ids under a strong penalty: the first bound, taken over every group's
    maximum, is too high once those maxima are penalised, and the second
    pass (groups without history ids only) must find the list.  Rows of
    equal values: every group reaches the bound, the candidates overflow,
    and the slice is redone exactly with the block-wide buffer."""
    rs = np.random.default_rng(23)
    B, V, n_top = 8, 50000, 80
    for dtype in ("f32", "bf16"):
        x = (rs.standard_normal((B, V)) * 1.0).astype(np.float32)
        hist, off = [], [0]
        for r in range(B):
            if r < 4:
                top = rs.choice(V, n_top, replace=False)
                x[r, top] = 12.0 + rs.random(n_top).astype(np.float32)
                hist += [int(t) for t in top]
            else:
                x[r, :] = np.float32(0.5) if r % 2 else np.float32(-1.25)
                hist += [7, 11]
            off.append(len(hist))
        logits = synth.to_bf16_bits(x) if dtype == "bf16" else x
        for k, p_ in [(50, 0.9), (8, 1.0)]:
            cfg = cases.configs(B, temperature=0.9, top_k=k, top_p=p_, rep=4.0, freq=0.5)
            d = dict(logits=logits, cfg=cfg, rng=np.arange(5, 5 + B, dtype=np.uint64),
                     hist=np.array(hist, dtype=np.int32), hist_off=np.array(off, dtype=np.int32))
            g = run_gpu(cuda, pz, d, max_top_k=64, max_history=128)
            tok, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
            assert (g["tokens"] == tok).all(), (dtype, k)
            mism, _, _ = compare_with_oracle(oracle_lib, d, g, PROB_RTOL)
            assert mism == 0, (dtype, k)
