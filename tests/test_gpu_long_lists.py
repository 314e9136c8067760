"""Lists longer than 64 against the C restatement of the reference.

A batch of 1024 rows whose lists are 2 to 1024 long runs in two launches:
slice_kernel samples the rows whose list fits 64 and files the others for
slice_long_kernel (the fine sketch, a block-wide select and sort, the
warp-wide decision).  A batch of 8 such rows runs in one slice_long_kernel
launch with every row split over several CTAs.  Both are checked with the
usual bars: top-k id sets and RNG words bit-exact, list probabilities
within 1e-6 relative, sampled ids identical except proved boundary cases."""
import numpy as np
import pytest

import oracle_pool
from gpu_helpers import compare_with_oracle, run_gpu_tensors

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6


def _case(torch, B, V, dtype, seed):
    import cases
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    xf = torch.randn(B, V, generator=g, device="cuda").mul_(2.5)
    ids = torch.randint(0, V, (B, 16), generator=g, device="cuda")
    xf.scatter_add_(1, ids, torch.rand(B, 16, generator=g, device="cuda").mul_(10.0).add_(5.0))
    r = np.random.default_rng(seed)
    k = r.choice(np.array([2, 50, 64, 65, 100, 300, 1024]), B)
    T = np.where(r.random(B) < 0.05, 0.0, 0.3 + 1.2 * r.random(B)).astype(np.float32)
    p = np.where(r.random(B) < 0.3, 1.0, 0.5 + 0.5 * r.random(B)).astype(np.float32)
    # penalties that only lower values on most rows; ones that can raise them on some
    kind = r.integers(0, 4, B)
    rep = np.where(kind == 0, 1.0, np.where(kind == 3, 0.8, 1.0 + 0.3 * r.random(B))).astype(np.float32)
    freq = np.where(kind == 2, 0.3, 0.0).astype(np.float32)
    pres = np.where(kind == 3, -0.5, np.where(kind == 2, 0.2, 0.0)).astype(np.float32)
    flags = np.where(r.random(B) < 0.2, 1, 0).astype(np.uint32)  # PZ_CFG_TEMP_DIVIDE on some rows
    cfg_np = cases.configs(B, temperature=T, top_k=k, top_p=p, rep=rep, freq=freq, pres=pres, flags=flags)
    H = r.integers(0, 2049, B)
    hoff_np = np.zeros(B + 1, dtype=np.int32)
    hoff_np[1:] = np.cumsum(H)
    # histories drawn over the row's largest values too, so penalised ids reach the lists
    hist_np = r.integers(0, V, int(hoff_np[-1]), dtype=np.int32)
    if dtype == "bf16":
        x = xf.to(torch.bfloat16)
        host = x.view(torch.int16).cpu().numpy().view(np.uint16)
    else:
        x = xf
        host = x.cpu().numpy()
    top = torch.topk(xf, 600, dim=1).indices.to(torch.int32).cpu().numpy()
    for b in range(B):
        n = min(int(H[b]), 300)
        if n:
            hist_np[hoff_np[b]:hoff_np[b] + n] = top[b, :n]
    rng_np = np.arange(500, 500 + B, dtype=np.uint64)
    return x, dict(logits=host, cfg=cfg_np, rng=rng_np, hist=hist_np, hist_off=hoff_np)


@pytest.mark.parametrize("B", [1024, 8])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_long_lists(cuda, pz, oracle_lib, B, dtype):
    torch = cuda
    V = 50000
    x, d = _case(torch, B, V, dtype, seed=1100 + B + (7 if dtype == "bf16" else 0))
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=1024, max_history=2048)
    cfg = pz.configs_to_device(d["cfg"], "cuda")
    rng = torch.from_numpy(d["rng"].view(np.int64).copy()).cuda()
    hist = torch.from_numpy(d["hist"]).cuda()
    hoff = torch.from_numpy(d["hist_off"]).cuda()
    gres = run_gpu_tensors(torch, pz, s, x, cfg, rng, hist, hoff, no_full_vocab=True)
    s.close()
    assert (gres["status"] == 0).all()
    ref = oracle_pool.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"], cand_stride=1024)
    mism, n, maxrel = compare_with_oracle(oracle_lib, d, gres, PROB_RTOL, label=f"long lists B={B} {dtype}",
                                          oracle_out=ref)
    n_long = int((d["cfg"]["top_k"] > 64).sum())
    print(f"long lists B={B} {dtype}: {n_long} rows with k > 64, {mism} boundary cases, "
          f"max prob rel err {maxrel:.2e}")
