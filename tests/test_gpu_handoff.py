"""The LM-head hand-off: the classifier of the reference's forward pass
(bf16 weight rows, fp32 activations, fp32 logits) writes the sampler's
logits buffer on the device, and the sampler reads it on the same stream.
The logits are checked against float64 numpy (fp32 accumulation: 1e-4
relative to the row scale); the tokens against the C restatement run on
those very logits."""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def test_classifier_logits_and_tokens(cuda, pz, oracle_lib):
    torch = cuda
    B, dim, V = 5, 2560, 32000
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    hidden = torch.randn(B, dim, generator=g, device="cuda")
    w32 = torch.randn(V, dim, generator=g, device="cuda") * 0.05
    w = w32.to(torch.bfloat16)
    logits = torch.empty(B, V, device="cuda")
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=64, max_history=0)
    s.lm_head(hidden, w.view(torch.int16), logits)
    torch.cuda.synchronize()
    want = hidden.double().cpu().numpy() @ w.float().double().cpu().numpy().T
    got = logits.cpu().numpy()
    scale = np.abs(hidden.cpu().numpy()) @ np.abs(w.float().cpu().numpy()).T
    assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-6)
    cfg_np = pz.make_configs(B, 0.8, 40, 0.95, 1.0)
    cfg = pz.configs_to_device(cfg_np, "cuda")
    rng = torch.arange(11, 11 + B, dtype=torch.int64, device="cuda")
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    logits2 = torch.empty(B, V, device="cuda")
    s.sample_from_hidden(hidden, w.view(torch.int16), logits2, cfg, rng, out, max_top_k=64,
                         no_full_vocab=True)
    torch.cuda.synchronize()
    assert torch.equal(logits2, logits)
    tok, rr, *_ = oracle_lib.sample_batch(logits2.cpu().numpy(), cfg_np, np.arange(11, 11 + B, dtype=np.uint64))
    assert (out.cpu().numpy() == tok).all()
    assert (rng.cpu().numpy().view(np.uint64) == rr).all()
    s.close()
