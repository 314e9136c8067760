"""Vocab sharding across two GPUs: each rank holds half of every row's
columns, the ranks exchange their local lists with one NCCL allgather, and
every rank returns the tokens (and RNG states) of the single-GPU sampler and
of the oracle.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cases

pytestmark = pytest.mark.gpu

TESTS = os.path.dirname(os.path.abspath(__file__))
SPEC = dict(seed=61, B=64, V=65536, sd=2.5, boosts=[16, 5.0, 15.0], dtype="bf16",
            cfg=dict(temperature=1.0, top_k=64, top_p=0.95))


def _worker(rank, world, uid_path, q):
    import sys
    for p in (TESTS, os.path.join(os.path.dirname(TESTS), "oracle"),
              os.path.join(os.path.dirname(TESTS), "project-zero_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import time
        import pz_sampling as pz
        from gpu_helpers import to_device
        torch.cuda.set_device(rank)
        d = cases.build(SPEC)
        B, V = SPEC["B"], SPEC["V"]
        begin, count = pz.row_shard(V, world, rank)  # this rank's column slice
        if rank == 0:
            uid = pz.Sampler.nccl_unique_id()
            with open(uid_path + ".tmp", "wb") as f:
                f.write(uid)
            os.rename(uid_path + ".tmp", uid_path)
        else:
            for _ in range(600):
                if os.path.exists(uid_path):
                    break
                time.sleep(0.05)
        with open(uid_path, "rb") as f:
            uid = f.read()
        x, cfg, rng, _, _ = to_device(torch, d, device=f"cuda:{rank}")
        xs = x[:, begin:begin + count]
        s = pz.Sampler(rank, max_batch=B, max_vocab=count, max_top_k=64, max_history=0)
        s.init_nccl(world, rank, uid)
        out = torch.full((B,), -7, dtype=torch.int32, device=f"cuda:{rank}")
        s.sample_vocab_sharded(xs, begin, V, cfg, rng, out)
        torch.cuda.synchronize()
        q.put((rank, "ok", out.cpu().tolist(), [int(v) for v in rng.cpu().numpy().view(np.uint64)]))
        s.close()
    except Exception as e:
        q.put((rank, "err", repr(e), None))


def test_vocab_sharded_two_gpus(tmp_path, oracle_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    uid_path = str(tmp_path / "nccl_uid")
    procs = [ctx.Process(target=_worker, args=(r, world, uid_path, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, status, tok, rng = q.get(timeout=240)
        assert status == "ok", tok
        res[rank] = (tok, rng)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]  # every rank draws the same tokens
    d = cases.build(SPEC)
    tok, rng, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"])
    assert res[0][0] == tok.tolist()
    assert res[0][1] == [int(v) for v in rng]


def test_contexts_on_two_devices_in_one_process(oracle_lib):
    """Kernel attributes (the opt-in to large dynamic shared memory) are set
    per device: contexts on cuda:0 and cuda:1 in one process both sample a
    config-3 batch exactly."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import pz_sampling as pz
    from gpu_helpers import compare_with_oracle
    spec = dict(seed=62, B=64, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=1024,
                cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1))
    d = cases.build(spec)
    torch.cuda.set_device(0)
    for dev in (1, 0):
        x = torch.from_numpy(d["logits"]).to(f"cuda:{dev}")
        cfg = torch.from_numpy(np.ascontiguousarray(d["cfg"]).view(np.uint8).copy()).to(f"cuda:{dev}")
        rng = torch.from_numpy(d["rng"].view(np.int64).copy()).to(f"cuda:{dev}")
        hist = torch.from_numpy(d["hist"]).to(f"cuda:{dev}")
        hoff = torch.from_numpy(d["hist_off"]).to(f"cuda:{dev}")
        s = pz.Sampler(dev, max_batch=64, max_vocab=128256, max_top_k=64, max_history=1024)
        out = torch.full((64,), -7, dtype=torch.int32, device=f"cuda:{dev}")
        cid = torch.full((64, 64), -9, dtype=torch.int32, device=f"cuda:{dev}")
        cpr = torch.full((64, 64), -9.0, dtype=torch.float32, device=f"cuda:{dev}")
        ncd = torch.full((64,), -9, dtype=torch.int32, device=f"cuda:{dev}")
        with torch.cuda.device(dev):
            s.sample(x, cfg, rng, out, hist, hoff, max_top_k=64, max_history=1024, no_full_vocab=True,
                     cand_ids=cid, cand_probs=cpr, n_cand=ncd)
        torch.cuda.synchronize(dev)
        g = dict(tokens=out.cpu().numpy(), rng=rng.cpu().numpy().view(np.uint64), cand_ids=cid.cpu().numpy(),
                 cand_probs=cpr.cpu().numpy(), n_cand=ncd.cpu().numpy())
        s.close()
        mism, _, _ = compare_with_oracle(oracle_lib, d, g, 1e-6, label=f"context on cuda:{dev}")
        assert mism == 0
        # the legacy single-row calls keep one staging area per device
        with torch.cuda.device(dev):
            t = pz.sample_argmax(d["logits"][0])
        assert t == int(np.argmax(d["logits"][0]))


def _lonely_rank(q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    import time
    sys.path.insert(0, os.path.join(os.path.dirname(TESTS), "project-zero_b200"))
    try:
        import pz_sampling as pz
        torch.cuda.set_device(0)
        s = pz.Sampler(0, max_batch=8, max_vocab=4096, max_top_k=64, max_history=0)
        uid = pz.Sampler.nccl_unique_id()
        t0 = time.time()
        try:
            s.init_nccl(2, 0, uid, timeout_ms=3000)  # rank 1 never joins
            q.put(("joined", time.time() - t0))
        except pz.PZError as e:
            q.put((e.status, time.time() - t0))
        s.close()
    except Exception as e:  # report, never hang the parent
        q.put(("err", repr(e)))


def test_nccl_init_times_out_when_a_rank_never_joins():
    """A communicator of two ranks whose second rank never arrives: the
    non-blocking set-up is polled against its 3 s deadline and comes back
    PZ_ERR_TIMEOUT (the communicator aborted) instead of waiting for ever.
    Nothing is launched on the GPU while the rank waits."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import pz_sampling as pz
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    status, took = q.get(timeout=120)
    p.join(timeout=60)
    assert status == pz.PZ_ERR_TIMEOUT, (status, took)
    assert 2.5 < took < 30.0


# ---- pz_sample_batch_multi: several devices from one host thread ----------
MULTI_SPEC = dict(seed=63, B=96, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=512,
                  cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1))


def _multi_devices(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    return list(range(n))


def _to(d, dev, rows=slice(None)):
    x = np.ascontiguousarray(d["logits"][rows])
    if x.dtype == np.uint16:  # bf16 bits
        x = torch.from_numpy(x.view(np.int16).copy()).to(f"cuda:{dev}").view(torch.bfloat16)
    else:
        x = torch.from_numpy(x).to(f"cuda:{dev}")
    cfg = torch.from_numpy(np.ascontiguousarray(d["cfg"][rows]).view(np.uint8).copy()).to(f"cuda:{dev}")
    rng = torch.from_numpy(np.ascontiguousarray(d["rng"][rows]).view(np.int64).copy()).to(f"cuda:{dev}")
    return x, cfg, rng


def _csr_rows(d, b, c):
    """The history CSR of rows [b, b + c), offsets rebased to 0."""
    off = d["hist_off"]
    h = d["hist"][off[b]:off[b + c]]
    o = (off[b:b + c + 1] - off[b]).astype(np.int32)
    return h, o


@pytest.mark.parametrize("n", [1, 2])
def test_multi_row_sharded(n, oracle_lib):
    """PZ_SHARD_ROWS: each device samples its pz_row_shard rows; together they
    give the oracle's tokens and RNG states for the whole batch."""
    import pz_sampling as pz
    devs = _multi_devices(n)
    d = cases.build(MULTI_SPEC)
    B, V = MULTI_SPEC["B"], MULTI_SPEC["V"]
    parts, samplers, outs = [], [], []
    for i, dev in enumerate(devs):
        b, c = pz.row_shard(B, n, i)
        x, cfg, rng = _to(d, dev, slice(b, b + c))
        h, o = _csr_rows(d, b, c)
        s = pz.Sampler(dev, max_batch=c, max_vocab=V, max_top_k=64, max_history=1024)
        out = torch.full((c,), -7, dtype=torch.int32, device=f"cuda:{dev}")
        samplers.append(s)
        outs.append((b, c, out, rng))
        parts.append(dict(sampler=s, logits=x, cfg=cfg, rng_state=rng, out=out,
                          hist=torch.from_numpy(h).to(f"cuda:{dev}"), hist_off=torch.from_numpy(o).to(f"cuda:{dev}")))
    pz.sample_multi(pz.SHARD_ROWS, parts, V, max_top_k=64, max_history=1024, no_full_vocab=True)
    for dev in devs:
        torch.cuda.synchronize(dev)
    tok = np.zeros(B, dtype=np.int64)
    rng_all = np.zeros(B, dtype=np.uint64)
    for b, c, out, rng in outs:
        tok[b:b + c] = out.cpu().numpy()
        rng_all[b:b + c] = rng.cpu().numpy().view(np.uint64)
    for s in samplers:
        s.close()
    t_o, r_o, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
    assert np.array_equal(tok, t_o)
    assert np.array_equal(rng_all, np.asarray(r_o, dtype=np.uint64))


@pytest.mark.parametrize("n", [1, 2])
def test_multi_vocab_sharded(n, oracle_lib):
    """PZ_SHARD_VOCAB from one thread: pz_multi_init_nccl joins the contexts,
    each device holds a column slice of every row, one grouped allgather
    exchanges the lists, and every device returns the oracle's tokens."""
    import pz_sampling as pz
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    devs = _multi_devices(n)
    d = cases.build(SPEC)
    B, V = SPEC["B"], SPEC["V"]
    samplers, parts = [], []
    for i, dev in enumerate(devs):
        b, c = pz.row_shard(V, n, i)
        x, cfg, rng = _to(d, dev)
        s = pz.Sampler(dev, max_batch=B, max_vocab=c, max_top_k=64, max_history=0)
        samplers.append(s)
        parts.append(dict(sampler=s, logits=x[:, b:b + c], v_offset=b, cfg=cfg, rng_state=rng,
                          out=torch.full((B,), -7, dtype=torch.int32, device=f"cuda:{dev}")))
    pz.multi_init_nccl(samplers, timeout_ms=60000)
    pz.sample_multi(pz.SHARD_VOCAB, parts, V)
    for s, p in zip(samplers, parts):
        s.wait(60000, stream=torch.cuda.current_stream(p["out"].device))
    t_o, r_o, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"])
    for p in parts:
        assert p["out"].cpu().tolist() == t_o.tolist()
        assert [int(v) for v in p["rng_state"].cpu().numpy().view(np.uint64)] == [int(v) for v in r_o]
    for s in samplers:
        s.close()
