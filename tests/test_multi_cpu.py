"""The host side of the multi-GPU modes, as world-size-2 gloo process groups
on the CPU: the row partition of pz_row_shard, row-sharded sampling equal to
the single-process batch, and the vocab-sharded decomposition (local exact
top-k lists, one all-gather, merge) equal to the full-row top-k."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases

TESTS = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import sys
    for p in (TESTS, os.path.join(os.path.dirname(TESTS), "oracle"),
              os.path.join(os.path.dirname(TESTS), "project-zero_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _gather_obj(obj, world):
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def _row_shard_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        import pz_sampling as pz
        res = {}
        for B in (0, 1, 2, 3, 7, 1024, 1025):
            res[B] = _gather_obj(pz.row_shard(B, world, rank), world)
        q.put((rank, "ok", res))
    except Exception as e:  # reported to the parent
        q.put((rank, "err", repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _row_sampling_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        import oracle
        import pz_sampling as pz
        spec = dict(seed=3, B=10, V=4096, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=32,
                    cfg=dict(temperature=0.7, top_k=20, top_p=0.9, rep=1.1, freq=0.2, pres=0.1))
        d = cases.build(spec)
        begin, count = pz.row_shard(spec["B"], world, rank)
        sl = slice(begin, begin + count)
        off = d["hist_off"][begin:begin + count + 1]
        hist = d["hist"][off[0]:off[-1]]
        o = oracle.Oracle()
        tok, rng, *_ = o.sample_batch(d["logits"][sl], d["cfg"][sl], d["rng"][sl], hist, off - off[0])
        parts = _gather_obj((begin, tok.tolist(), [int(v) for v in rng]), world)
        q.put((rank, "ok", parts))
    except Exception as e:
        q.put((rank, "err", repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _vocab_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        import oracle
        import pz_sampling as pz
        spec = dict(seed=5, B=6, V=8192, sd=2.5, boosts=[16, 5.0, 15.0],
                    cfg=dict(temperature=1.0, top_k=64, top_p=0.95))
        d = cases.build(spec)
        V, k = spec["V"], 64
        begin, count = pz.row_shard(V, world, rank)  # a contiguous column slice
        x = np.ascontiguousarray(d["logits"][:, begin:begin + count])
        o = oracle.Oracle()
        cfg = d["cfg"].copy()
        # the local exact top-k of the slice (the list the emit pass publishes)
        _, _, cid, cpr, ncd = o.sample_batch(x, cfg, d["rng"].copy(), cand_stride=k)
        local = []
        for r in range(spec["B"]):
            ids = cid[r, :ncd[r]]
            local.append([(float(x[r, i] / np.float32(1.0)), int(i) + begin) for i in ids])
        gathered = _gather_obj(local, world)  # the one all-gather
        merged = []
        for r in range(spec["B"]):
            cand = [c for g in gathered for c in g[r]]
            cand.sort(key=lambda t: (-t[0], t[1]))
            merged.append([i for _, i in cand[:k]])
        q.put((rank, "ok", merged))
    except Exception as e:
        q.put((rank, "err", repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        assert status == "ok", payload
        out[rank] = payload
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_row_shard_tiles_every_batch():
    out = _run(_row_shard_worker)
    for B, shards in out[0].items():
        assert out[1][B] == shards
        pos = 0
        for begin, count in shards:
            assert begin == pos and count >= 0
            pos += count
        assert pos == B
        counts = [c for _, c in shards]
        assert max(counts) - min(counts) <= 1


def test_row_sharded_sampling_equals_one_process(oracle_lib):
    out = _run(_row_sampling_worker)
    spec = dict(seed=3, B=10, V=4096, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=32,
                cfg=dict(temperature=0.7, top_k=20, top_p=0.9, rep=1.1, freq=0.2, pres=0.1))
    d = cases.build(spec)
    tok, rng, *_ = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"])
    parts = sorted(out[0], key=lambda t: t[0])
    assert sum((p[1] for p in parts), []) == tok.tolist()
    assert sum((p[2] for p in parts), []) == [int(v) for v in rng]


def test_vocab_sharded_merge_is_the_global_top_k(oracle_lib):
    out = _run(_vocab_worker)
    assert out[0] == out[1]  # every rank merges the same lists
    spec = dict(seed=5, B=6, V=8192, sd=2.5, boosts=[16, 5.0, 15.0],
                cfg=dict(temperature=1.0, top_k=64, top_p=0.95))
    d = cases.build(spec)
    _, _, cid, _, ncd = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], cand_stride=64)
    for r in range(spec["B"]):
        assert out[0][r] == cid[r, :ncd[r]].tolist(), r
