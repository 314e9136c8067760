"""The generate loop's sampling step on the device (pz_decode_step_*):
fresh logits are written to one fixed buffer each step (as the LM head
rewrites RunState.logits in the reference), the recorded step graph samples
them, advances the RNG states on the device and appends each sampled id to
its row's penalty window.  Every step's tokens equal the C restatement run
as the same loop on the host, seeded from the parsed --seed."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _host_loop(oracle_lib, xs, cfg_np, states, window):
    N, B, _ = xs.shape
    W = window.shape[1] if window is not None else 0
    out = np.zeros((N, B), dtype=np.int32)
    st = states.copy()
    for i in range(N):
        for r in range(B):
            h = window[r] if window is not None else None
            ho = np.array([0, W], np.int32) if window is not None else None
            tok, s, *_ = oracle_lib.sample_batch(xs[i, r:r + 1], cfg_np[r:r + 1], st[r:r + 1], h, ho)
            out[i, r] = tok[0]
            st[r] = s[0]
            if window is not None:
                window[r, i % W] = tok[0]
    return out, st


@pytest.mark.parametrize("variant", ["pipeline_window", "engine"])
def test_decode_step_graph_equals_the_host_loop(cuda, pz, oracle_lib, variant):
    torch = cuda
    B, V = 3, 128256
    N = 150 if variant == "pipeline_window" else 40
    if variant == "pipeline_window":
        p = pz.params_from_args(["generate", "--seed", "42", "--temperature", "0.8", "--top-k", "40",
                                 "--top-p", "0.95", "--repeat-penalty", "1.1"])
    else:
        p = pz.params_from_args(["generate", "--seed", "7", "--temperature", "0.8", "--top-p", "0.95"])
    cfg_np = p.as_config(B)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    xs = torch.randn(N, B, V, generator=g, device="cuda").mul_(2.5)
    ids = torch.randint(0, V, (N, B, 8), generator=g, device="cuda")
    xs.scatter_add_(2, ids, torch.rand(N, B, 8, generator=g, device="cuda") * 10 + 5)
    buf = torch.empty(B, V, device="cuda")
    cfg = pz.configs_to_device(cfg_np, "cuda")
    rng = torch.empty(B, dtype=torch.int64, device="cuda")
    pz.seed_states(rng, seed_base=p.seed)                       # seed + r, 0 -> 1
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    window = None
    if variant == "pipeline_window":
        w0 = np.random.default_rng(3).integers(0, V, (B, 64)).astype(np.int32)  # the prompt's last ids
        window = torch.from_numpy(w0.copy()).cuda()
    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=64, max_history=64)
    step = pz.DecodeStep(s, buf, cfg, rng, out, window, max_top_k=64, max_history=64,
                         no_full_vocab=variant == "pipeline_window")
    got = torch.empty(N, B, dtype=torch.int32, device="cuda")
    for i in range(N):
        buf.copy_(xs[i])          # the LM head's output for this step
        step.launch()
        got[i].copy_(out)
    torch.cuda.synchronize()
    assert step.steps() == N
    states_end = rng.cpu().numpy().view(np.uint64)
    step.close()
    s.close()
    want, st = _host_loop(oracle_lib, xs.cpu().numpy(), cfg_np,
                          np.array([(p.seed + r) or 1 for r in range(B)], dtype=np.uint64),
                          w0.copy() if window is not None else None)
    # a boundary case would change the window and every later draw, so the
    # sequences must match exactly
    assert (got.cpu().numpy() == want).all()
    assert (states_end == st).all()


def test_rng_state_checkpoint_resume(cuda, pz):
    """Checkpoint and resume of the sampler's only state, the per-row RNG words
    (the reference keeps one word per stream, generate.c:125): a 200-step
    stream split in two, its RNG array saved to the host after 100 steps and
    restored into a fresh context and buffer, draws the same tokens as the
    unbroken stream."""
    torch = cuda
    B, V, N = 8, 32000, 200
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    xs = torch.randn(N, B, V, generator=g, device="cuda").mul_(2.5)
    cfg = pz.configs_to_device(pz.make_configs(B, temperature=0.8, top_k=40, top_p=0.95), "cuda")

    def run(sampler, rng, steps):
        out = torch.empty(B, dtype=torch.int32, device="cuda")
        toks = []
        for i in steps:
            sampler.sample(xs[i], cfg, rng, out, max_top_k=64, no_full_vocab=True)
            toks.append(out.clone())
        return torch.stack(toks)

    s = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=64, max_history=0)
    rng = torch.empty(B, dtype=torch.int64, device="cuda")
    pz.seed_states(rng, seed_base=42)
    whole = run(s, rng, range(N))
    pz.seed_states(rng, seed_base=42)
    first = run(s, rng, range(N // 2))
    saved = rng.cpu().numpy().copy()              # the checkpoint
    s.close()
    s2 = pz.Sampler(0, max_batch=B, max_vocab=V, max_top_k=64, max_history=0)
    rng2 = torch.from_numpy(saved).cuda()         # resume
    second = run(s2, rng2, range(N // 2, N))
    s2.close()
    assert torch.equal(torch.cat([first, second]), whole)
