"""Host-side logic that needs no GPU: workloads, sharding, request keys,
the oracle's uniform source and sampling helpers.  CPU only."""
from __future__ import annotations

import numpy as np

from oracle.philox import request_key, step_uniforms
from oracle.sampling import inverse_cdf, sample_with_uniform, weights
from pse import workload as wl
from pse.speculative import _fnv1a


def test_workload_prompts_are_seeded_and_in_range():
    for name, w in wl.WORKLOADS.items():
        a = wl.prompts(w, seed=3, n=16)
        b = wl.prompts(w, seed=3, n=16)
        assert a == b
        assert all(w.prompt_lo <= len(p) <= w.prompt_hi for p in a)
        assert all(0 <= x < w.pair.vocab for p in a for x in p)
    assert wl.prompts(wl.WORKLOADS["tiny"], seed=0) != wl.prompts(wl.WORKLOADS["tiny"], seed=1)


def test_llama_prompt_lengths_are_clipped_lognormal():
    w = wl.WORKLOADS["llama-1b"]
    lens = np.array([len(p) for p in wl.prompts(w, seed=0, n=400)])
    assert lens.min() >= 128 and lens.max() <= 8192
    assert 1500 < np.median(lens) < 2700


def test_lpt_shards_balance_and_cover():
    rng = np.random.default_rng(0)
    costs = rng.integers(100, 9000, size=2048).tolist()
    for n in (1, 2, 4, 8):
        shards = wl.lpt_shards(costs, n)
        assert sorted(i for s in shards for i in s) == list(range(len(costs)))
        loads = [sum(costs[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(costs)


def test_request_key_matches_oracle():
    for rid in ("r0", "req-123", "g7r255", "ü-unicode"):
        assert _fnv1a(rid) == request_key(rid)


def test_uniforms_are_in_unit_interval_and_distinct():
    u = step_uniforms(123, [request_key(f"r{i}") for i in range(64)], list(range(64)), 17)
    assert u.shape == (64, 17)
    assert (u >= 0).all() and (u < 1).all()
    assert len(np.unique(u)) == u.size
    assert abs(u.mean() - 0.5) < 0.02


def test_inverse_cdf_edges():
    w = np.array([0.0, 1.0, 0.0, 3.0, 0.0], dtype=np.float32)
    assert inverse_cdf(w, 4.0, 0.0) == 1
    assert inverse_cdf(w, 4.0, 0.2499) == 1
    assert inverse_cdf(w, 4.0, 0.25) == 3
    assert inverse_cdf(w, 4.0, 0.9999999) == 3
    assert inverse_cdf(w, 4.0, 1.0) == 3  # rounding past the total -> last non-zero weight
    assert sample_with_uniform(np.array([1.0, 5.0, 5.0]), 0.0, 0.3) == 1  # greedy, first max
    ww, z = weights(np.array([0.0, 0.0]), 1.0)
    assert z == 2.0 and ww.dtype == np.float32


def test_workloads_have_the_benchmark_configurations_shapes():
    """The synthetic workloads the benchmark runs carry the shapes its metric is
    quoted on: model sizes, request counts, prompt ranges, new tokens, k, block
    size, batch, temperature and dtype."""
    W = wl.WORKLOADS
    t = W["tiny"]
    assert (t.pair.vocab, t.pair.target, t.pair.draft["n_layers"], t.pair.draft["d_model"], t.pair.draft["n_heads"]) == \
        (256, dict(d_model=128, n_layers=4, n_heads=4, d_ff=512, max_seq_len=256), 2, 64, 2)
    assert (t.n_requests, t.prompt_lo, t.prompt_hi, t.max_new_tokens, t.k, t.block_size, t.max_batch_size,
            t.temperature, t.dtype) == (8, 8, 32, 64, 4, 16, 4, 0.0, "float32")
    s = W["tiny-sampled"]
    assert (s.pair, s.n_requests, s.prompt_lo, s.prompt_hi, s.max_new_tokens, s.block_size, s.temperature) == \
        (t.pair, 64, 8, 64, 128, 16, 1.0)
    g = W["gpt2-small"]
    tg, dg = g.pair.target, g.pair.draft
    assert (g.pair.vocab, tg["n_layers"], tg["d_model"], tg["n_heads"], tg["d_model"] // tg["n_heads"], tg["d_ff"]) == \
        (32000, 12, 768, 12, 64, 3072)
    assert (dg["n_layers"], dg["d_model"], dg["n_heads"]) == (4, 384, 6)
    assert (g.n_requests, g.prompt_lo, g.prompt_hi, g.max_new_tokens, g.k, g.block_size, g.max_batch_size,
            g.temperature, g.dtype) == (256, 128, 1024, 256, 5, 16, 256, 0.0, "bfloat16")
    assert tg["max_seq_len"] >= g.prompt_hi + g.max_new_tokens + g.k + 1
    lw = W["llama-1b"]
    tl, dl = lw.pair.target, lw.pair.draft
    assert (lw.pair.kind, lw.pair.vocab, tl["n_layers"], tl["d_model"], tl["n_heads"], tl["n_kv_heads"],
            tl["d_model"] // tl["n_heads"], tl["d_ff"]) == ("llama", 32000, 16, 2048, 32, 8, 64, 8192)
    assert (dl["n_layers"], dl["d_model"], dl["n_heads"], dl["n_kv_heads"]) == (2, 1024, 16, 4)
    assert (lw.n_requests, lw.prompt_lo, lw.prompt_hi, lw.lognormal_median, lw.max_new_tokens, lw.k,
            lw.block_size, lw.dtype) == (2048, 128, 8192, 2048.0, 512, 4, 32, "bfloat16")
