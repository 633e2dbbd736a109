"""Batched prefill (``pse.prefill_requests``) against one-by-one
``prefill_request`` calls (engine/speculative.py:53-73 as the scheduler makes
them, engine/scheduler.py:78-90).  GPU only.

* Cache state bit for bit: block tables, lengths, free lists and last tokens,
  also when the caches already hold requests and have freed some.
* Next-token logits within the fp32 / bf16 tolerances.
* A pool too small for every prompt: the call raises the reference's
  MemoryError at the same request, leaving the same state.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2


def _pair(kind, seed=0):
    torch.manual_seed(seed)
    if kind == "gpt":
        d = TinyGPT(ModelConfig(vocab_size=300, d_model=64, n_layers=2, n_heads=2, d_ff=128, max_seq_len=512))
        t = TinyGPT(ModelConfig(vocab_size=300, d_model=128, n_layers=3, n_heads=4, d_ff=256, max_seq_len=512))
    else:
        d = TinyLlama(LlamaConfig(vocab_size=300, d_model=128, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=256,
                                  max_seq_len=1024))
        t = TinyLlama(LlamaConfig(vocab_size=300, d_model=256, n_layers=2, n_heads=4, n_kv_heads=1, d_ff=512,
                                  max_seq_len=1024))
    return d.eval(), t.eval()


def _caches(d, t, bs, nb, dtype):
    import pse
    out = []
    for m in (d, t):
        c = m.cfg
        out.append(pse.PagedKVCache(c.n_layers, getattr(c, "n_kv_heads", c.n_heads), c.d_model // c.n_heads, bs, nb,
                                    dtype=dtype))
    return out


def _state(cache, ids):
    return ({r: cache.block_table(r) for r in ids}, {r: cache.length(r) for r in ids}, cache.allocator.free_list(),
            {r: int(cache.last_token[cache.slot(r)].item()) for r in ids}, int(cache.allocator.num_free))


@pytest.mark.parametrize("kind,dtype,bs", [("gpt", torch.float32, 4), ("gpt", torch.bfloat16, 16),
                                           ("llama", torch.bfloat16, 32)])
def test_prefill_requests_equals_one_by_one(kind, dtype, bs):
    import pse
    d, t = _pair(kind)
    rng = np.random.default_rng(bs)
    lens = [1, bs, bs + 1, 3 * bs - 1] + [int(x) for x in rng.integers(2, 300, size=9)]
    prompts = [rng.integers(0, 300, size=n).tolist() for n in lens]
    ids = [f"q{i}" for i in range(len(prompts))]
    warm = [rng.integers(0, 300, size=int(n)).tolist() for n in rng.integers(5, 60, size=3)]
    runs = []
    for batched in (False, True):
        dc, tc = _caches(d, t, bs, 600, dtype)
        # caches already in use: three requests prefilled, one freed
        for i, p in enumerate(warm):
            pse.prefill_request(d, t, dc, tc, f"w{i}", p)
        dc.free_request("w1")
        tc.free_request("w1")
        if batched:
            out = pse.prefill_requests(d, t, dc, tc, ids, prompts)
        else:
            out = {r: pse.prefill_request(d, t, dc, tc, r, p) for r, p in zip(ids, prompts)}
        logits = {r: (a.float().cpu().clone(), b.float().cpu().clone()) for r, (a, b) in out.items()}
        live = ids + ["w0", "w2"]
        runs.append((_state(dc, live), _state(tc, live), logits))
    (sd0, st0, lg0), (sd1, st1, lg1) = runs
    assert sd0 == sd1 and st0 == st1
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    for r in ids:
        for a, b in zip(lg0[r], lg1[r]):
            assert (a - b).abs().max().item() < tol, r


def test_prefill_requests_raises_like_one_by_one_when_the_pool_runs_dry():
    import pse
    d, t = _pair("gpt", seed=3)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 300, size=int(n)).tolist() for n in (40, 70, 30, 90, 50)]
    ids = [f"r{i}" for i in range(len(prompts))]
    states = []
    for batched in (False, True):
        dc, tc = _caches(d, t, 8, 25, torch.float32)  # room for about two and a half prompts
        with pytest.raises(MemoryError):
            if batched:
                pse.prefill_requests(d, t, dc, tc, ids, prompts)
            else:
                for r, p in zip(ids, prompts):
                    pse.prefill_request(d, t, dc, tc, r, p)
        states.append((dc.allocator.free_list(), tc.allocator.free_list(), dc.allocator.num_free,
                       [dc._blocks.nblocks[s].item() for s in range(dc._blocks.num_slots)]))
    assert states[0] == states[1]
