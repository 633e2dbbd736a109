"""End-to-end parity beyond the reference's own cases.  GPU only.

* Llama-style pair (GQA + RoPE + SwiGLU + RMSNorm), fp32: every request of a
  batched scheduler run equals the oracle's solo greedy ``generate_cached``.
* The same layout in bf16 on the tensor-core attention path (head_dim 64):
  prompt logits within the bf16 tolerance of the oracle's fp32 forward on the
  same (bf16-rounded) weights.
* T > 0 with explicit uniforms: the device step and the oracle step consume
  the same Philox uniforms, so every step's accepted tokens must agree draw
  for draw.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import scheduler as OS
from oracle.generate import generate_cached
from oracle.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama
from oracle.paged_cache import PagedKVCache as OracleCache
from oracle.philox import request_key, step_uniforms

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _llama_pair(seed, **kw):
    torch.manual_seed(seed)
    cfg = LlamaConfig(**kw)
    return TinyLlama(cfg).eval(), TinyLlama(cfg).eval(), cfg


def _pse_caches(cfg, bs, nb, dtype=torch.float32):
    import pse
    hd = cfg.d_model // cfg.n_heads
    kv = getattr(cfg, "n_kv_heads", cfg.n_heads)
    return (pse.PagedKVCache(cfg.n_layers, kv, hd, bs, nb, dtype=dtype),
            pse.PagedKVCache(cfg.n_layers, kv, hd, bs, nb, dtype=dtype))


@pytest.mark.parametrize("seed,k,bs", [(0, 3, 4), (1, 5, 16), (2, 2, 3)])
def test_llama_gqa_scheduler_matches_solo_greedy(seed, k, bs):
    import pse
    d, t, cfg = _llama_pair(seed, vocab_size=96, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=96,
                            max_seq_len=256)
    rng = np.random.default_rng(seed)
    reqs = [pse.Request(f"r{i}", rng.integers(0, 96, size=int(rng.integers(2, 12))).tolist(), int(rng.integers(3, 12)))
            for i in range(5)]
    dc, tc = _pse_caches(cfg, bs, 256)
    res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, 3, k=k, temperature=0.0, use_graph=False)
    by = {r.request_id: r.output_ids for r in res}
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), q


def _round_bf16(model):
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    return model


@pytest.mark.parametrize("kind", ["llama", "gpt"])
def test_bf16_prompt_logits_within_tolerance(kind):
    import pse
    torch.manual_seed(3)
    if kind == "llama":
        cfg = LlamaConfig(vocab_size=512, d_model=256, n_layers=2, n_heads=4, n_kv_heads=1, d_ff=512,
                          max_seq_len=512)
        model = _round_bf16(TinyLlama(cfg).eval())
    else:
        cfg = ModelConfig(vocab_size=512, d_model=256, n_layers=2, n_heads=4, d_ff=512, max_seq_len=512)
        model = _round_bf16(TinyGPT(cfg).eval())
    kv = getattr(cfg, "n_kv_heads", cfg.n_heads)
    c = pse.PagedKVCache(cfg.n_layers, kv, cfg.d_model // cfg.n_heads, 16, 128, dtype=torch.bfloat16)
    rng = np.random.default_rng(0)
    worst = 0.0
    for i in range(4):
        prompt = rng.integers(0, 512, size=int(rng.integers(20, 200))).tolist()
        c.create_request(f"p{i}")
        got = pse.batched_forward_append(model, c, [f"p{i}"], torch.tensor([prompt]))[0].float().cpu()
        with torch.no_grad():
            want = model(torch.tensor([prompt]))[0][0]
        worst = max(worst, (got - want).abs().max().item())
        # a width-3 continuation over the paged state, as the verify call runs it
        more = rng.integers(0, 512, size=3).tolist()
        got2 = pse.batched_forward_append(model, c, [f"p{i}"], torch.tensor([more]))[0].float().cpu()
        with torch.no_grad():
            want2 = model(torch.tensor([prompt + more]))[0][0, -3:]
        worst = max(worst, (got2 - want2).abs().max().item())
    assert worst < BF16_TOL, worst


@pytest.mark.parametrize("k,defer", [(2, False), (4, False), (4, True)])
def test_sampled_steps_match_oracle_draw_for_draw(k, defer):
    """T = 1 with the same explicit Philox uniforms on both sides: identical
    accepted tokens at every step (fp32 TinyGPT pair)."""
    import pse
    torch.manual_seed(0)
    dcfg = ModelConfig(vocab_size=256, d_model=64, n_layers=2, n_heads=2, d_ff=256, max_seq_len=256)
    tcfg = ModelConfig(vocab_size=256, d_model=128, n_layers=4, n_heads=4, d_ff=512, max_seq_len=256)
    d, t = TinyGPT(dcfg).eval(), TinyGPT(tcfg).eval()
    seed = 1234 + k
    rng = np.random.default_rng(k)
    prompts = [rng.integers(0, 256, size=int(rng.integers(8, 30))).tolist() for _ in range(8)]

    def uniform_fn(ids, steps, n):
        return step_uniforms(seed, [request_key(r) for r in ids], steps, n)

    oracle_steps, device_steps = [], []
    oreqs = [OS.Request(f"r{i}", p, 24) for i, p in enumerate(prompts)]
    odc = OracleCache(2, 2, 32, 16, 256)
    otc = OracleCache(4, 4, 32, 16, 256)
    ores = OS.run_continuous_speculative_batches(
        d, t, oreqs, odc, otc, 4, k=k, temperature=1.0, uniform_fn=uniform_fn,
        on_step=lambda ids, r: oracle_steps.append({x: r.accepted_tokens[x] for x in ids}))
    preqs = [pse.Request(f"r{i}", p, 24) for i, p in enumerate(prompts)]
    pdc = pse.PagedKVCache(2, 2, 32, 16, 256)
    ptc = pse.PagedKVCache(4, 4, 32, 16, 256)
    pres = pse.run_continuous_speculative_batches(
        d, t, preqs, pdc, ptc, 4, k=k, temperature=1.0, uniform_fn=uniform_fn, use_graph=False, defer_bonus=defer,
        on_step=lambda ids, r: device_steps.append({x: r.accepted_tokens[x] for x in ids}))
    assert device_steps == oracle_steps
    assert {r.request_id: r.output_ids for r in pres} == {r.request_id: r.output_ids for r in ores}
    assert any(len(v) > 1 for s in device_steps for v in s.values())  # some drafts were accepted


def test_deferred_bonus_property_matches_solo_greedy():
    """Scheduler property of the reference (every request == solo greedy) in
    deferred-bonus mode, over seeded random workloads."""
    import pse
    rng = np.random.default_rng(7)
    for trial in range(25):
        torch.manual_seed(int(rng.integers(0, 1000)))
        cfg = ModelConfig(vocab_size=32, d_model=12, n_layers=2, n_heads=2, d_ff=24, max_seq_len=256)
        d, t = TinyGPT(cfg).eval(), TinyGPT(cfg).eval()
        k, bs, mb = int(rng.integers(1, 6)), int(rng.integers(1, 6)), int(rng.integers(1, 5))
        reqs = [pse.Request(f"r{i}", rng.integers(1, 32, size=int(rng.integers(1, 6))).tolist(), int(rng.integers(1, 9)))
                for i in range(int(rng.integers(1, 7)))]
        nb = sum(len(r.prompt_ids) + r.max_new_tokens + k + 2 for r in reqs) // bs * len(reqs) + 16
        hd = cfg.d_model // cfg.n_heads
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, bs, nb)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, bs, nb)
        res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, mb, k=k, temperature=0.0,
                                                     use_graph=False, defer_bonus=True)
        by = {r.request_id: r.output_ids for r in res}
        for q in reqs:
            assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), (trial, q)
        assert dc.allocator.num_free == nb and tc.allocator.num_free == nb


@pytest.mark.parametrize("k", [2, 4, 8])
def test_sampled_workload_matches_oracle_draw_for_draw(k):
    """The T = 1 configuration itself (TinyGPT pair fp32, 64 requests, prompts
    U[8,64], 128 new tokens, block 16, all 64 rows in every step) at k = 2, 4,
    8: with the same explicit Philox uniforms, every step's accepted tokens
    (hence accepted_len) equal the oracle's."""
    import pse
    from pse import workload as wl
    w = wl.WORKLOADS["tiny-sampled"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=w.pair.vocab, **w.pair.draft)).eval()
    t = TinyGPT(ModelConfig(vocab_size=w.pair.vocab, **w.pair.target)).eval()
    prompts = wl.prompts(w, seed=0)
    seed = 77 + k

    def uniform_fn(ids, steps, n):
        return step_uniforms(seed, [request_key(r) for r in ids], steps, n)

    nb = sum((len(p) + w.max_new_tokens + 2 * k + 2 + w.block_size - 1) // w.block_size for p in prompts) + 8
    pd, pt = w.pair.draft, w.pair.target
    oracle_steps, device_steps = [], []
    ores = OS.run_continuous_speculative_batches(
        d, t, [OS.Request(f"r{i}", p, w.max_new_tokens) for i, p in enumerate(prompts)],
        OracleCache(pd["n_layers"], pd["n_heads"], pd["d_model"] // pd["n_heads"], w.block_size, nb),
        OracleCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], w.block_size, nb),
        w.max_batch_size, k=k, temperature=1.0, uniform_fn=uniform_fn,
        on_step=lambda ids, r: oracle_steps.append([r.num_draft_accepted[x] for x in ids]))
    dc = pse.PagedKVCache(pd["n_layers"], pd["n_heads"], pd["d_model"] // pd["n_heads"], w.block_size, nb)
    tc = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], w.block_size, nb)
    pres = pse.run_continuous_speculative_batches(
        d, t, [pse.Request(f"r{i}", p, w.max_new_tokens) for i, p in enumerate(prompts)], dc, tc,
        w.max_batch_size, k=k, temperature=1.0, uniform_fn=uniform_fn, device_bookkeeping=False,
        on_step=lambda ids, r: device_steps.append([r.num_draft_accepted[x] for x in ids]))
    assert device_steps == oracle_steps  # accepted_len of every row at every step
    assert {r.request_id: r.output_ids for r in pres} == {r.request_id: r.output_ids for r in ores}
    assert max(max(s) for s in device_steps) >= 2  # multi-draft accepts happened
