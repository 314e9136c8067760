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
