"""Prefix caching (pse.prefix_cache; the reference's README.md:216-219 future
work) on the device engine.  The oracle is the reference's own contract: every
request's output equals its solo ``generate_cached`` decode
(engine/generate.py:24-38) whether or not prompts share blocks, rows never
write into shared blocks (another row's gather is unchanged by anything this
row does), and every block returns to the free list once the index lets go of
it.  GPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu

CFG = ModelConfig(vocab_size=64, d_model=32, n_layers=2, n_heads=4, d_ff=64, max_seq_len=256)


def _pse():
    import pse
    return pse


def _models(seed):
    torch.manual_seed(seed)
    return TinyGPT(CFG).eval(), TinyGPT(CFG).eval()


def _workload(seed, n, sys_len, bs):
    """Prompts sharing a system prompt (some with a second shared layer, some
    identical, some unrelated), each with its own suffix."""
    rng = np.random.default_rng(seed)
    system = rng.integers(0, CFG.vocab_size, size=sys_len).tolist()
    few_shot = rng.integers(0, CFG.vocab_size, size=2 * bs + 3).tolist()
    prompts = []
    for i in range(n):
        kind = i % 5
        tail = rng.integers(0, CFG.vocab_size, size=int(rng.integers(1, 12))).tolist()
        if kind == 0:
            prompts.append(system + tail)
        elif kind == 1:
            prompts.append(system + few_shot + tail)
        elif kind == 2:
            prompts.append(list(system))  # the system prompt alone (its last token is computed)
        elif kind == 3:
            prompts.append(rng.integers(0, CFG.vocab_size, size=int(rng.integers(1, 3 * bs))).tolist())
        else:
            prompts.append(system[: bs * 2] + tail)  # a shorter shared run
    return prompts


def _caches(P, bs, nb, prefix):
    hd = CFG.d_model // CFG.n_heads
    return (P.PagedKVCache(CFG.n_layers, CFG.n_heads, hd, bs, nb, prefix_cache=prefix),
            P.PagedKVCache(CFG.n_layers, CFG.n_heads, hd, bs, nb, prefix_cache=prefix))


def _conserved(cache, nb):
    """Every block is free, or held by the index (idle): each id exactly once."""
    free = cache.allocator.free_list()
    idle = list(cache.prefix.idle) if cache.prefix is not None else []
    assert sorted(free + idle) == list(range(nb))


@pytest.mark.parametrize("seed,bs,batch,k,dev", [(0, 4, 4, 3, True), (1, 16, 6, 4, True), (2, 8, 3, 2, False),
                                                 (3, 1, 5, 5, True)])
def test_prefix_cache_scheduler_equals_solo_greedy(seed, bs, batch, k, dev):
    """Shared prefixes through the unchanged scheduler loop: every output is
    the target's solo greedy decode, the index was hit, and the pool is whole
    again (free list + idle indexed blocks, then the free list alone after
    ``clear``)."""
    P = _pse()
    d, t = _models(seed)
    prompts = _workload(seed, 14, 3 * bs + 5 if bs > 1 else 23, bs)
    rng = np.random.default_rng(seed + 100)
    reqs = [P.Request(f"r{i}", p, int(rng.integers(1, 10))) for i, p in enumerate(prompts)]
    nb = 600
    dc, tc = _caches(P, bs, nb, True)
    res = P.run_continuous_speculative_batches(d, t, reqs, dc, tc, batch, k=k, device_bookkeeping=dev)
    by = {r.request_id: r.output_ids for r in res}
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), q
    for c in (dc, tc):
        assert c.prefix.stats()["hit_tokens"] > 0
        _conserved(c, nb)
        c.prefix.clear()
        assert sorted(c.allocator.free_list()) == list(range(nb))


def test_prefix_cache_same_outputs_as_without():
    """The same workload with and without the index: identical outputs and
    result order; fewer prompt tokens computed with it."""
    P = _pse()
    d, t = _models(7)
    prompts = _workload(7, 20, 29, 4)
    outs = []
    for prefix in (False, True):
        reqs = [P.Request(f"r{i}", p, 6) for i, p in enumerate(prompts)]
        dc, tc = _caches(P, 4, 800, prefix)
        res = P.run_continuous_speculative_batches(d, t, reqs, dc, tc, 5, k=3)
        outs.append([(r.request_id, r.output_ids) for r in res])
        if prefix:
            s = tc.prefix.stats()
            assert s["hit_tokens"] >= 4 * 7  # most system-prompt prompts reuse its 7 full blocks
    assert outs[0] == outs[1]


def test_prefix_cache_truncate_below_shared_and_append():
    """A row truncated inside its shared run gets its own copy of the partly
    kept block; appends after it land in its own blocks; the row it shares
    with reads exactly what it read before."""
    P = _pse()
    d, t = _models(11)
    bs, nb = 4, 64
    dc, tc = _caches(P, bs, nb, True)
    rng = np.random.default_rng(11)
    base = rng.integers(0, CFG.vocab_size, size=3 * bs + 2).tolist()
    P.prefill_requests(d, t, dc, tc, ["a"], [base])
    P.prefill_requests(d, t, dc, tc, ["b"], [base[: 3 * bs] + [5, 6, 7]])
    assert tc.prefix.shared_tokens(tc.slot("b")) == 3 * bs
    ka, va, _, _ = tc.gather(["a"])
    ka = [x.clone() for x in ka]
    va = [x.clone() for x in va]
    kb0, vb0, _, _ = tc.gather(["b"])
    new_len = bs + 1
    tc.truncate("b", new_length=new_len)
    assert tc.length("b") == new_len and tc.num_blocks_in_use("b") == 2
    assert tc.block_table("b")[0] == tc.block_table("a")[0]      # still shared
    assert tc.block_table("b")[1] != tc.block_table("a")[1]      # its own copy
    kb1, vb1, _, _ = tc.gather(["b"])
    for L in range(CFG.n_layers):
        assert torch.equal(kb1[L][0, :, :new_len], kb0[L][0, :, :new_len])
        assert torch.equal(vb1[L][0, :, :new_len], vb0[L][0, :, :new_len])
    hd = CFG.d_model // CFG.n_heads
    nk = [torch.randn(CFG.n_heads, 2 * bs, hd) for _ in range(CFG.n_layers)]
    nv = [torch.randn(CFG.n_heads, 2 * bs, hd) for _ in range(CFG.n_layers)]
    tc.append("b", nk, nv)
    kb2, vb2, _, _ = tc.gather(["b"])
    for L in range(CFG.n_layers):
        assert torch.equal(kb2[L][0, :, :new_len], kb0[L][0, :, :new_len])
        assert torch.equal(kb2[L][0, :, new_len:new_len + 2 * bs].cpu(), nk[L])
        assert torch.equal(vb2[L][0, :, new_len:new_len + 2 * bs].cpu(), nv[L])
    ka2, va2, _, _ = tc.gather(["a"])
    for L in range(CFG.n_layers):
        assert torch.equal(ka2[L], ka[L]) and torch.equal(va2[L], va[L])
    tc.truncate("b", new_length=0)
    assert tc.num_blocks_in_use("b") == 0
    for c in (dc, tc):
        for r in ("a", "b"):
            c.free_request(r)
        _conserved(c, nb)


def test_prefix_cache_evicts_idle_blocks_under_pressure():
    """A pool too small to keep every finished prompt's blocks: idle blocks
    are evicted (least recently used first) for admissions and steps, and the
    outputs are unchanged."""
    P = _pse()
    d, t = _models(5)
    bs = 4
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, CFG.vocab_size, size=int(rng.integers(9, 30))).tolist() for _ in range(16)]
    reqs = [P.Request(f"r{i}", p, 8) for i, p in enumerate(prompts)]
    nb = 2 * ((30 + 8 + 8) // bs + 2) + 4  # room for two active requests only
    dc, tc = _caches(P, bs, nb, True)
    res = P.run_continuous_speculative_batches(d, t, reqs, dc, tc, 2, k=3)
    by = {r.request_id: r.output_ids for r in res}
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), q
    for c in (dc, tc):
        assert c.prefix.stats()["evicted_blocks"] > 0
        _conserved(c, nb)


def test_prefix_cache_llama_bf16_prefill_logits():
    """bf16 Llama-style pair (GQA, RoPE): a prompt prefilled on top of another
    prompt's shared blocks gives the same next-token logits (within the bf16
    tolerance) as prefilling it alone."""
    P = _pse()
    from oracle.model import LlamaConfig, TinyLlama
    torch.manual_seed(3)
    cfg = LlamaConfig(vocab_size=128, d_model=256, n_layers=2, n_heads=4, n_kv_heads=1, d_ff=256, max_seq_len=512)
    d, t = TinyLlama(cfg).eval(), TinyLlama(cfg).eval()
    hd = cfg.d_model // cfg.n_heads
    rng = np.random.default_rng(3)
    system = rng.integers(0, 128, size=70).tolist()
    q = system + rng.integers(0, 128, size=9).tolist()
    outs = []
    for prefix in (False, True):
        dc = P.PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, 16, 64, dtype=torch.bfloat16, prefix_cache=prefix)
        tc = P.PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, 16, 64, dtype=torch.bfloat16, prefix_cache=prefix)
        P.prefill_requests(d, t, dc, tc, ["s"], [system + [1, 2, 3]])
        out = P.prefill_requests(d, t, dc, tc, ["q"], [q])
        outs.append((out["q"][0].float().cpu().clone(), out["q"][1].float().cpu().clone()))
        if prefix:
            assert tc.prefix.shared_tokens(tc.slot("q")) == 64
    for a, b in zip(outs[0], outs[1]):
        assert torch.allclose(a, b, atol=2e-2, rtol=0)
