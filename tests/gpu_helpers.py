"""Runs case dicts (tests/cases.py) through the CUDA library and compares
with the CPU checker."""
from __future__ import annotations

import numpy as np


def to_device(torch, d, device="cuda"):
    x = d["logits"]
    if x.dtype == np.uint16:
        t = torch.from_numpy(x.view(np.int16).copy()).to(device).view(torch.bfloat16)
    else:
        t = torch.from_numpy(x.copy()).to(device)
    raw = np.ascontiguousarray(d["cfg"]).view(np.uint8)
    cfg = torch.from_numpy(raw.copy()).to(device)
    rng = torch.from_numpy(d["rng"].view(np.int64).copy()).to(device)
    hist = hist_off = None
    if d.get("hist") is not None:
        hist = torch.from_numpy(d["hist"].astype(np.int32)).to(device)
        hist_off = torch.from_numpy(d["hist_off"].astype(np.int32)).to(device)
    return t, cfg, rng, hist, hist_off


def run_gpu_tensors(torch, pz, sampler, x, cfg, rng, hist=None, hist_off=None, cand_stride=1024,
                    max_top_k=0, max_history=0, no_full_vocab=False):
    """One pz_sample_batch call on device tensors (rng advanced in place);
    returns the outputs as host arrays."""
    B = x.shape[0]
    dev = x.device
    out = torch.full((B,), -7, dtype=torch.int32, device=dev)
    cid = torch.full((B, cand_stride), -9, dtype=torch.int32, device=dev)
    cpr = torch.full((B, cand_stride), -9.0, dtype=torch.float32, device=dev)
    ncd = torch.full((B,), -9, dtype=torch.int32, device=dev)
    st = torch.full((B,), -9, dtype=torch.int32, device=dev)
    sampler.sample(x, cfg, rng, out, hist, hist_off, max_top_k=max_top_k, max_history=max_history,
                   no_full_vocab=no_full_vocab, cand_ids=cid, cand_probs=cpr, n_cand=ncd,
                   row_status=st)
    torch.cuda.synchronize()
    return dict(tokens=out.cpu().numpy(), rng=rng.cpu().numpy().view(np.uint64),
                cand_ids=cid.cpu().numpy(), cand_probs=cpr.cpu().numpy(), n_cand=ncd.cpu().numpy(),
                status=st.cpu().numpy())


def run_gpu(torch, pz, d, sampler=None, cand_stride=1024, max_top_k=0, max_history=0,
            no_full_vocab=False):
    x, cfg, rng, hist, hist_off = to_device(torch, d)
    B, V = x.shape
    own = sampler is None
    if own:
        sampler = pz.Sampler(0, max_batch=max(B, 1), max_vocab=V, max_top_k=1024, max_history=4096)
    res = run_gpu_tensors(torch, pz, sampler, x, cfg, rng, hist, hist_off, cand_stride, max_top_k,
                          max_history, no_full_vocab)
    if own:
        sampler.close()
    return res


# boundary cases seen by this test session: (test label, rows, count)
BOUNDARY_LOG = []


def compare_with_oracle(oracle_lib, d, g, prob_rtol=1e-6, label="", oracle_out=None):
    """Returns (n_boundary, n_rows, max_prob_rel_err).  Asserts that the
    top-k id sets and the RNG words are bit-exact, the list probabilities
    within prob_rtol, and that every sampled id that differs from the
    oracle's is a boundary case (tests/parity.py); counts those.
    oracle_out: the oracle's (tokens, rng, cand_ids, cand_probs, n_cand)
    for d when already computed (e.g. by tests/oracle_pool.py)."""
    from parity import boundary_rows
    if oracle_out is None:
        oracle_out = oracle_lib.sample_batch(d["logits"], d["cfg"], d["rng"], d["hist"], d["hist_off"],
                                             cand_stride=1024)
    tok, rng, cid, cpr, ncd = oracle_out
    assert (ncd == g["n_cand"]).all(), "list lengths differ"
    maxrel = 0.0
    for r in np.nonzero(ncd)[0]:
        n = int(ncd[r])
        assert (cid[r, :n] == g["cand_ids"][r, :n]).all(), f"top-k id set differs in row {r}"
        a, b = cpr[r, :n].astype(np.float64), g["cand_probs"][r, :n].astype(np.float64)
        rel = np.abs(a - b) / np.maximum(np.abs(a), 1e-30)
        rel[(a == 0) & (b == 0)] = 0.0
        maxrel = max(maxrel, float(rel.max()))
    assert maxrel <= prob_rtol, maxrel
    assert (rng == g["rng"]).all(), "RNG words differ"
    n_boundary, wrong = boundary_rows(oracle_lib, d, tok, g["tokens"])
    assert not wrong, f"rows {wrong[:10]} sample a different id away from any CDF boundary"
    BOUNDARY_LOG.append((label, len(tok), n_boundary))
    return n_boundary, len(tok), maxrel
