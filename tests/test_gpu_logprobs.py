"""OpenAI-style log-probabilities from the batch call (token_logprob,
cand_logprobs).  A floating-point output with no counterpart in the
reference, so it is checked against a float64 numpy log-softmax of the same
penalised, tempered float32 values (the contract's arithmetic, from the C
restatement), within 1e-4 absolute."""
import numpy as np
import pytest

import cases
from gpu_helpers import to_device

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def _drawn_values(oracle_lib, d, r):
    """float32 values the row is drawn from: penalised, then tempered
    (x * fl(1/T)); greedy rows untempered."""
    x = d["logits"][r]
    if x.dtype == np.uint16:
        x = (x.astype(np.uint32) << np.uint32(16)).view(np.float32)
    x = np.array(x, dtype=np.float32)
    c = d["cfg"][r]
    if d.get("hist") is not None and (c["repetition_penalty"] != 1 or c["frequency_penalty"] != 0
                                      or c["presence_penalty"] != 0):
        h = d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        x = oracle_lib.apply_penalties(x, h, c["repetition_penalty"], c["frequency_penalty"],
                                       c["presence_penalty"])
    T = np.float32(c["temperature"])
    if T <= 0 or T < np.float32(1e-6):
        return x
    return oracle_lib.apply_temperature(x, T)


@pytest.mark.parametrize("spec", [
    dict(seed=301, B=24, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=1024,
         cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1)),
    dict(seed=302, B=32, V=151936, sd=2.0, zipf=[256, 10.0], dtype="bf16", cfg="hetero"),
], ids=["config3_rows", "config4_rows"])
def test_logprobs_match_float64_log_softmax(cuda, pz, oracle_lib, spec):
    torch = cuda
    d = cases.build(spec)
    x, cfg, rng, hist, hist_off = to_device(torch, d)
    rng2 = rng.clone()
    B, V = x.shape
    stride = 1024
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=1024, max_history=2048)
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    cid = torch.full((B, stride), -9, dtype=torch.int32, device="cuda")
    ncd = torch.full((B,), -9, dtype=torch.int32, device="cuda")
    tlp = torch.full((B,), -9.0, dtype=torch.float32, device="cuda")
    clp = torch.full((B, stride), -9.0, dtype=torch.float32, device="cuda")
    s.sample(x, cfg, rng, out, hist, hist_off, cand_ids=cid, n_cand=ncd, token_logprob=tlp,
             cand_logprobs=clp)
    out2 = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    s.sample(x, cfg, rng2, out2, hist, hist_off)  # the tokens do not depend on the extra outputs
    torch.cuda.synchronize()
    tok, ids, n = out.cpu().numpy(), cid.cpu().numpy(), ncd.cpu().numpy()
    got_t, got_c = tlp.cpu().numpy(), clp.cpu().numpy()
    assert (tok == out2.cpu().numpy()).all()
    s.close()
    for r in range(B):
        v = _drawn_values(oracle_lib, d, r).astype(np.float64)
        fin = np.isfinite(v)
        m = v[fin].max()
        lse = m + np.log(np.exp(v[fin] - m).sum())
        assert abs(got_t[r] - (v[tok[r]] - lse)) <= ATOL, (r, got_t[r], v[tok[r]] - lse)
        k = int(n[r])
        if k:
            want = v[ids[r, :k]] - lse
            assert np.all(np.abs(got_c[r, :k] - want) <= ATOL), r
            assert np.all(np.diff(got_c[r, :k]) <= 1e-6)  # the list is in descending order
            assert np.all(np.isneginf(got_c[r, k:]))
