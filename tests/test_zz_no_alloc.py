"""pz_sample_batch_static (no context, scratch in the library's fixed device
array, no allocation) against pz_sample_batch on the same inputs, two calls
in a row.  Collected last so it also runs after every other test has used
the device."""
import numpy as np
import pytest

import cases
from gpu_helpers import to_device

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-6


def _outputs(torch, B, stride):
    return dict(cand_ids=torch.full((B, stride), -9, dtype=torch.int32, device="cuda"),
                cand_probs=torch.full((B, stride), -9.0, dtype=torch.float32, device="cuda"),
                n_cand=torch.full((B,), -9, dtype=torch.int32, device="cuda"),
                row_status=torch.full((B,), -9, dtype=torch.int32, device="cuda"))


def _host(torch, out, rng, o):
    torch.cuda.synchronize()
    return dict(tokens=out.cpu().numpy(), rng=rng.cpu().numpy().view(np.uint64),
                **{k: v.cpu().numpy() for k, v in o.items()})


@pytest.mark.parametrize("spec", [
    dict(seed=91, B=512, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], cfg="hetero"),
    dict(seed=92, B=64, V=151936, sd=2.0, zipf=[256, 10.0], dtype="bf16", cfg="hetero"),
    dict(seed=93, B=1024, V=128256, sd=2.5, boosts=[8, 5.0, 15.0], hist_len=1024,
         cfg=dict(temperature=0.7, top_k=50, top_p=0.9, rep=1.1, freq=0.2, pres=0.1)),
], ids=["f32_hetero", "bf16_hetero", "config3_full_batch"])
def test_static_matches_context_two_calls(cuda, pz, spec):
    torch = cuda
    d = cases.build(spec)
    x, cfg, rng_a, hist, hist_off = to_device(torch, d)
    rng_b = rng_a.clone()
    B, V = x.shape
    stride = pz.STATIC_MAX_TOP_K
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=pz.STATIC_MAX_TOP_K,
                   max_history=pz.STATIC_MAX_HISTORY)
    for call in range(2):
        out_a = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        out_b = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        oa, ob = _outputs(torch, B, stride), _outputs(torch, B, stride)
        s.sample(x, cfg, rng_a, out_a, hist, hist_off, max_top_k=pz.STATIC_MAX_TOP_K,
                 max_history=pz.STATIC_MAX_HISTORY, no_full_vocab=True, **oa)
        pz.sample_static(x, cfg, rng_b, out_b, hist, hist_off, **ob)
        a, b = _host(torch, out_a, rng_a, oa), _host(torch, out_b, rng_b, ob)
        for key in ("tokens", "rng", "row_status", "n_cand"):
            assert (a[key] == b[key]).all(), (call, key)
        assert (a["row_status"] == 0).any(), "no row was sampled"
        for r in range(B):
            n = int(a["n_cand"][r])
            assert (a["cand_ids"][r, :n] == b["cand_ids"][r, :n]).all(), (call, r)
            pa = a["cand_probs"][r, :n].astype(np.float64)
            pb = b["cand_probs"][r, :n].astype(np.float64)
            assert (np.abs(pa - pb) <= PROB_RTOL * np.maximum(np.abs(pa), 1e-30)).all(), (call, r)
    s.close()


def test_static_refuses_rows_and_sizes_beyond_its_limits(cuda, pz):
    torch = cuda
    B, V = 8, 5000
    d = cases.build(dict(seed=94, B=B, V=V, sd=2.0, hist_len=0,
                         cfg=dict(temperature=0.8, top_k=50, top_p=0.9)))
    d["cfg"]["top_k"][:4] = [0, 65, 1024, 64]
    x, cfg, rng, _, _ = to_device(torch, d)
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    st = torch.full((B,), -9, dtype=torch.int32, device="cuda")
    pz.sample_static(x, cfg, rng, out, row_status=st)
    torch.cuda.synchronize()
    status = st.cpu().numpy()
    assert (status[:3] == pz.PZ_ROW_HINT_VIOLATED).all() and (out.cpu().numpy()[:3] == -1).all()
    assert (status[3:] == pz.PZ_ROW_OK).all()
    big = torch.zeros((pz.STATIC_MAX_BATCH + 1, 16), dtype=torch.float32, device="cuda")
    cfg_big = pz.configs_to_device(pz.make_configs(pz.STATIC_MAX_BATCH + 1))
    rng_big = torch.ones(pz.STATIC_MAX_BATCH + 1, dtype=torch.int64, device="cuda")
    out_big = torch.zeros(pz.STATIC_MAX_BATCH + 1, dtype=torch.int32, device="cuda")
    with pytest.raises(pz.PZError, match="static scratch") as e:
        pz.sample_static(big, cfg_big, rng_big, out_big)
    assert e.value.status == pz.PZ_ERR_UNSUPPORTED
