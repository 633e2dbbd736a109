"""Plain continuous batching (engine/benchmark.py:41-84) on the device
kernels: every request equals the target's solo greedy decode
(``generate_cached``), for several batch sizes and block sizes, and the pool is
whole again at the end.  GPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed,bs,batch,use_graph", [(0, 4, 3, True), (1, 16, 5, False), (2, 3, 1, True)])
def test_plain_batches_equal_solo_greedy(seed, bs, batch, use_graph):
    import pse
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=96, d_model=64, n_layers=2, n_heads=4, d_ff=128, max_seq_len=256)
    t = TinyGPT(cfg).eval()
    rng = np.random.default_rng(seed)
    reqs = [pse.Request(f"p{i}", rng.integers(0, 96, size=int(rng.integers(1, 20))).tolist(), int(rng.integers(1, 15)))
            for i in range(7)]
    nb = 200
    cache = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, cfg.d_model // cfg.n_heads, bs, nb)
    res = pse.run_plain_continuous_batches(t, reqs, cache, batch, use_graph=use_graph)
    by = {r.request_id: r.output_ids for r in res}
    for q in reqs:
        n_new = max(q.max_new_tokens, 2)  # the reference's loop always takes one step after admission
        want = generate_cached(t, torch.tensor([q.prompt_ids]), n_new)
        assert by[q.request_id] == want, q
    assert cache.allocator.num_free == nb


@pytest.mark.parametrize("use_graph", [True, False])
def test_plain_device_bookkeeping_equals_host_loop(use_graph):
    """Same results, same order of results and the same free list with the
    per-row bookkeeping on the device (the default) or on the host, including
    max_new_tokens of 0, 1 and 2 (the reference always takes one step)."""
    import pse
    torch.manual_seed(3)
    cfg = ModelConfig(vocab_size=96, d_model=64, n_layers=2, n_heads=4, d_ff=128, max_seq_len=256)
    t = TinyGPT(cfg).eval()
    rng = np.random.default_rng(3)
    max_new = [0, 1, 2, 9, 5, 1, 13, 3, 0, 7, 2]
    prompts = [rng.integers(0, 96, size=int(rng.integers(1, 20))).tolist() for _ in max_new]
    outs = []
    for dev in (True, False):
        reqs = [pse.Request(f"q{i}", p, m) for i, (p, m) in enumerate(zip(prompts, max_new))]
        cache = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, cfg.d_model // cfg.n_heads, 8, 300)
        res = pse.run_plain_continuous_batches(t, reqs, cache, 4, use_graph=use_graph, device_bookkeeping=dev)
        outs.append(([(r.request_id, r.output_ids) for r in res], cache.allocator.free_list()))
    assert outs[0] == outs[1]
    assert len(outs[0][0]) == len(max_new)
