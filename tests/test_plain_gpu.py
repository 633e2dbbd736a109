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
