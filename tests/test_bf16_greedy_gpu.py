"""Greedy token parity at the benchmark shapes, in bf16.

The engine decodes stated subsamples of the two bf16 configurations through
``pse.run_continuous_speculative_batches`` (both step structures: the default
one, whose target bonus call is deferred into the next verify, and the
reference's own):

* gpt2-small: the GPT-2-small-shaped pair (target d768/12L/12H/ff3072, draft
  d384/4L/6H, vocab 32000, k=5, block 16), the workload's first 16 prompts
  (U[128,1024] tokens), 48 new tokens each;
* llama-1b: the Llama-style pair (target d2048/16L, GQA 32/8, SwiGLU 8192,
  RoPE; draft d1024/2L, GQA 16/4; vocab 32000, k=4, block 32), 6 prompts of
  U[128,384] tokens (the workload's median-2048 prompts are past what the CPU
  oracle runs in seconds), 32 new tokens each.

The oracle is ``generate_cached`` (engine/generate.py:24-38): greedy argmax of
the fp32 CPU model on the same weights rounded to bf16.  Every committed token
is checked by one teacher-forced oracle forward over the engine's own output:
at each position the engine's token must be the oracle's argmax given the same
prefix, or lie within the bf16 logit tolerance (2e-2) of it.  Up to the first
position where they differ, the oracle's argmax sequence *is* generate_cached's
output, so a request with no such position equals generate_cached exactly.
Divergences (near-ties the bf16 arithmetic resolves the other way) are counted
and reported with their logit gaps.  The prefill logits themselves are checked
against the oracle's within 2e-2.  GPU only."""
from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from oracle.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama

pytestmark = pytest.mark.gpu

BF16_LOGIT_TOL = 2e-2


@functools.lru_cache(maxsize=2)
def _pair(name):
    from pse import workload as wl
    w = wl.WORKLOADS[name]
    pr = w.pair
    torch.manual_seed(0)
    if pr.kind == "gpt":
        d = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.draft)).eval()
        t = TinyGPT(ModelConfig(vocab_size=pr.vocab, **pr.target)).eval()
    else:
        d = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.draft)).eval()
        t = TinyLlama(LlamaConfig(vocab_size=pr.vocab, **pr.target)).eval()
    with torch.no_grad():  # the engine runs these weights in bf16: the oracle sees the same values
        for m in (d, t):
            for p in m.parameters():
                p.copy_(p.to(torch.bfloat16).float())
    return w, d, t


def _subsample(name):
    from pse import workload as wl
    w = wl.WORKLOADS[name]
    if name == "gpt2-small":
        return wl.prompts(w, seed=0, n=16), 48
    rng = np.random.default_rng(4)
    return [rng.integers(0, w.pair.vocab, size=int(rng.integers(128, 385))).tolist() for _ in range(6)], 32


def _caches(w, d, t, prompts, max_new):
    import pse
    bs = w.block_size
    out = []
    for m in (d, t):
        c = m.cfg
        kv = getattr(c, "n_kv_heads", c.n_heads)
        nb = sum((len(p) + max_new + 2 * w.k + 2 + bs - 1) // bs for p in prompts) + 8
        out.append(pse.PagedKVCache(c.n_layers, kv, c.d_model // c.n_heads, bs, nb, dtype=torch.bfloat16,
                                    max_requests=len(prompts)))
    return out


_TF_MEMO: dict = {}


def _teacher_forced(t, prompt, generated):
    """Oracle logits at every generated position given the engine's prefix
    (fp32, CPU); memoised, since both step structures usually commit the same
    tokens."""
    key = (id(t), tuple(prompt), tuple(generated))
    if key not in _TF_MEMO:
        seq = torch.tensor([prompt + generated[:-1]])
        with torch.no_grad():
            _TF_MEMO[key] = t(seq)[0][0][len(prompt) - 1:]
    return _TF_MEMO[key]


@pytest.mark.parametrize("name", ["gpt2-small", "llama-1b"])
def test_bf16_greedy_tokens_match_generate_cached(name):
    import pse
    w, d, t = _pair(name)
    prompts, max_new = _subsample(name)
    report = {}
    for structure in (None, False):  # default (deferred bonus), the reference's structure
        dc, tc = _caches(w, d, t, prompts, max_new)
        reqs = [pse.Request(f"q{i}", p, max_new) for i, p in enumerate(prompts)]
        res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, len(reqs), k=w.k, temperature=0.0,
                                                     defer_bonus=structure)
        by = {r.request_id: r.output_ids for r in res}
        flips, gaps, exact = 0, [], 0
        for i, p in enumerate(prompts):
            out = by[f"q{i}"]
            assert out[: len(p)] == p and len(out) == len(p) + max_new
            gen = out[len(p):]
            ol = _teacher_forced(t, p, gen)
            best = ol.max(dim=-1).values
            chosen = ol.gather(1, torch.tensor(gen).view(-1, 1)).view(-1)
            gap = (best - chosen)
            amax = ol.argmax(dim=-1)
            differ = (amax != torch.tensor(gen)).nonzero().view(-1).tolist()
            if not differ:
                exact += 1
            flips += len(differ)
            gaps += [float(gap[j]) for j in differ]
            assert float(gap.max()) < BF16_LOGIT_TOL, (structure, i, differ, gap[differ].tolist())
        report[structure] = dict(exact_requests=exact, requests=len(prompts), divergent_positions=flips,
                                 positions=len(prompts) * max_new, max_gap=max(gaps, default=0.0))
        assert dc.allocator.num_free == dc.num_blocks and tc.allocator.num_free == tc.num_blocks
    print(f"\n{name} bf16 greedy vs generate_cached:", report)
    for r in report.values():
        # divergences are rare near-ties, not drift
        assert r["divergent_positions"] <= 0.05 * r["positions"], report


@pytest.mark.parametrize("name", ["gpt2-small", "llama-1b"])
def test_bf16_prefill_logits_within_tolerance(name):
    import pse
    w, d, t = _pair(name)
    prompts, _ = _subsample(name)
    prompts = prompts[:4]
    dc, tc = _caches(w, d, t, prompts, 1)
    worst = 0.0
    for i, p in enumerate(prompts):
        _, tl = pse.prefill_request(d, t, dc, tc, f"p{i}", p)
        with torch.no_grad():
            want = t(torch.tensor([p]))[0][0, -1]
        worst = max(worst, (tl.float().cpu() - want).abs().max().item())
    assert worst < BF16_LOGIT_TOL, worst
