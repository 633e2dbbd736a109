"""Distribution preservation at T > 0 (the reference's
tests/test_distribution_preserving.py:73-127) through the device engine: the
first output token after a prefilled prompt, over 4000 independent trials,
must pass a chi-squared goodness-of-fit test (p > 0.01) against the target's
exact softmax -- alone and while sharing every step with two other requests.
Uniforms come from a per-trial torch.Generator, as in the reference.  GPU only."""
from __future__ import annotations

import pytest
import torch
from scipy.stats import chisquare

from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu

VOCAB = 12
TRIALS = 4000
ALPHA = 0.01


def _models(seed):
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=VOCAB, d_model=8, n_layers=1, n_heads=2, d_ff=16, max_seq_len=32)
    return TinyGPT(cfg).eval(), TinyGPT(cfg).eval(), cfg


def _pvalue(samples, probs):
    obs = torch.zeros(VOCAB, dtype=torch.float64)
    for s in samples:
        obs[s] += 1
    exp = probs.double() * len(samples)
    exp = exp / exp.sum() * len(samples)
    assert exp.min().item() > 3
    return chisquare(obs.tolist(), exp.tolist())[1]


def _true(target, prompt):
    with torch.no_grad():
        return torch.softmax(target(torch.tensor([prompt]))[0][0, -1], -1)


def test_single_request_first_token_distribution():
    import pse
    d, t, cfg = _models(10)
    prompt = [1, 2, 3]
    hd = cfg.d_model // cfg.n_heads
    samples = []
    for trial in range(TRIALS):
        gen = torch.Generator().manual_seed(trial)
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 16)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 16)
        dn, tn = pse.prefill_request(d, t, dc, tc, "r", prompt)
        step = pse.batched_speculative_step(d, t, ["r"], dc, tc, {"r": dn}, {"r": tn}, k=3, temperature=1.0,
                                            generator=gen, use_graph=False)
        samples.append(step.accepted_tokens["r"][0])
    assert _pvalue(samples, _true(t, prompt)) > ALPHA


def test_batched_request_first_token_distribution():
    import pse
    d, t, cfg = _models(11)
    prompt = [2, 4, 1]
    hd = cfg.d_model // cfg.n_heads
    samples = []
    for trial in range(TRIALS):
        gen = torch.Generator().manual_seed(trial)
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 3, 32)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 3, 32)
        reqs = [pse.Request("target_req", prompt, 1), pse.Request("filler_a", [5, 6], 3),
                pse.Request("filler_b", [7, 8, 9], 2)]
        res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, 3, k=3, temperature=1.0, generator=gen,
                                                     use_graph=False)
        samples.append({r.request_id: r.output_ids for r in res}["target_req"][len(prompt)])
    assert _pvalue(samples, _true(t, prompt)) > ALPHA


def test_device_philox_stream_first_token_distribution():
    """Same claim with the device Philox uniform source (no generator)."""
    import pse
    import pse.speculative as S
    d, t, cfg = _models(10)
    prompt = [1, 2, 3]
    hd = cfg.d_model // cfg.n_heads
    samples = []
    for trial in range(TRIALS):
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 16)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 16)
        dn, tn = pse.prefill_request(d, t, dc, tc, f"r{trial}", prompt)
        S.runner_for(d, t, dc, tc, 3).seed = 1000 + trial
        step = pse.batched_speculative_step(d, t, [f"r{trial}"], dc, tc, {f"r{trial}": dn}, {f"r{trial}": tn},
                                            k=3, temperature=1.0, use_graph=False)
        samples.append(step.accepted_tokens[f"r{trial}"][0])
    assert _pvalue(samples, _true(t, prompt)) > ALPHA


@pytest.mark.parametrize("k", [2, 8])
def test_sampled_workload_first_tokens_match_target_distributions(k):
    """The T = 1 configuration's 64 requests (TinyGPT pair, vocab 256, prompts
    U[8,64]) share every step; over independent trials (device Philox stream,
    one seed per trial) each request's first output token must follow the
    target's softmax after its own prompt.  Per request, a chi-squared test
    (the reference's method; bins whose expected count is below 5 pooled);
    the 64 p-values must pass a Bonferroni bound (min p > 0.01 / 64) and
    Fisher's combined test (p > 0.01)."""
    import numpy as np
    from scipy.stats import chi2

    import pse
    import pse.speculative as S
    from pse import workload as wl
    w = wl.WORKLOADS["tiny-sampled"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=w.pair.vocab, **w.pair.draft)).eval()
    t = TinyGPT(ModelConfig(vocab_size=w.pair.vocab, **w.pair.target)).eval()
    prompts = wl.prompts(w, seed=0)
    n, trials, V = len(prompts), 1500, w.pair.vocab
    pd, pt = w.pair.draft, w.pair.target
    nb = sum((len(p) + 2 * k + 2 + w.block_size - 1) // w.block_size for p in prompts) + 8
    dc = pse.PagedKVCache(pd["n_layers"], pd["n_heads"], pd["d_model"] // pd["n_heads"], w.block_size, nb,
                          max_requests=n)
    tc = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], w.block_size, nb,
                          max_requests=n)
    counts = np.zeros((n, V), dtype=np.int64)
    for trial in range(trials):
        ids = [f"t{trial}_{i}" for i in range(n)]
        out = pse.prefill_requests(d, t, dc, tc, ids, prompts)
        S.runner_for(d, t, dc, tc, k).seed = 5000 + trial
        res = pse.batched_speculative_step(d, t, ids, dc, tc, {r: out[r][0] for r in ids},
                                           {r: out[r][1] for r in ids}, k, 1.0)
        for i, r in enumerate(ids):
            counts[i, res.accepted_tokens[r][0]] += 1
        dc.free_requests(ids)
        tc.free_requests(ids)
    pvals = []
    for i, p in enumerate(prompts):
        probs = _true(t, p).double().numpy()
        exp = probs * trials
        small = exp < 5
        obs_b = np.append(counts[i][~small], counts[i][small].sum())
        exp_b = np.append(exp[~small], exp[small].sum())
        keep = exp_b > 0
        obs_b, exp_b = obs_b[keep], exp_b[keep] / exp_b[keep].sum() * trials
        pvals.append(chisquare(obs_b, exp_b)[1])
    pvals = np.array(pvals)
    fisher = chi2.sf(-2 * np.log(np.maximum(pvals, 1e-300)).sum(), 2 * n)
    assert pvals.min() > ALPHA / n, sorted(pvals)[:5]
    assert fisher > ALPHA, fisher
