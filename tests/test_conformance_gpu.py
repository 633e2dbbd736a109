"""The reference's conformance cases (tests/test_paged_cache.py,
test_paged_cache_properties.py, test_speculative_single_request.py,
test_scheduler.py, test_scheduler_properties.py) driven against the device
engine.  Models are built by the oracle's TinyGPT (weights bit-identical to
the reference constructor's); the greedy baseline is the oracle's
``generate_cached`` on the CPU.  GPU only."""
from __future__ import annotations

import pytest
import torch
from hypothesis import HealthCheck, assume, given, settings, strategies as st

from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _eager_steps():
    import pse.speculative as S
    old = S.USE_GRAPHS
    S.USE_GRAPHS = False  # many small one-off caches: capture would dominate
    yield
    S.USE_GRAPHS = old


def _pse():
    import pse
    return pse


# ---------------------------------------------------------------- paged cache unit cases
def _kv(n_layers, n_heads, n, hd, fill):
    return [torch.full((n_heads, n, hd), fill) for _ in range(n_layers)]


def test_allocator_roundtrip_exhaustion_double_free():
    P = _pse()
    a = P.BlockAllocator(num_blocks=4)
    assert a.num_free == 4
    x, y = a.allocate(), a.allocate()
    assert a.num_free == 2 and x != y
    a.free(x)
    assert a.num_free == 3
    a.free(y)
    assert a.num_free == 4
    b = P.BlockAllocator(num_blocks=2)
    b.allocate()
    b.allocate()
    with pytest.raises(MemoryError):
        b.allocate()
    c = P.BlockAllocator(num_blocks=2)
    blk = c.allocate()
    c.free(blk)
    with pytest.raises(ValueError):
        c.free(blk)
    # LIFO order of the reference: first id handed out is n-1
    d = P.BlockAllocator(num_blocks=5)
    assert [d.allocate() for _ in range(3)] == [4, 3, 2]


def test_append_fits_spans_crosses_blocks():
    P = _pse()
    c = P.PagedKVCache(n_layers=2, n_heads=2, head_dim=4, block_size=4, num_blocks=8)
    c.create_request("r1")
    k = _kv(2, 2, 3, 4, 1.0)
    c.append("r1", k, k)
    assert c.length("r1") == 3 and c.num_blocks_in_use("r1") == 1
    ko, vo, mask, lens = c.gather(["r1"])
    assert lens.tolist() == [3] and mask.tolist() == [[True, True, True]]
    assert torch.equal(ko[0][0].cpu(), torch.full((2, 3, 4), 1.0))

    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=8)
    c.create_request("r1")
    c.append("r1", _kv(1, 1, 10, 2, 2.0), _kv(1, 1, 10, 2, 2.0))
    assert c.length("r1") == 10 and c.num_blocks_in_use("r1") == 3

    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=8)
    c.create_request("r1")
    c.append("r1", _kv(1, 1, 3, 2, 5.0), _kv(1, 1, 3, 2, 5.0))
    c.append("r1", _kv(1, 1, 3, 2, 6.0), _kv(1, 1, 3, 2, 6.0))
    ko, _, _, lens = c.gather(["r1"])
    want = torch.tensor([5.0, 5.0, 5.0, 6.0, 6.0, 6.0]).view(1, 6, 1).expand(1, 6, 2)
    assert lens.item() == 6 and torch.equal(ko[0][0, :, :6].cpu(), want)


def test_truncate_and_free_return_blocks():
    P = _pse()
    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=4)
    c.create_request("r1")
    c.append("r1", _kv(1, 1, 8, 2, 1.0), _kv(1, 1, 8, 2, 1.0))
    assert c.num_blocks_in_use("r1") == 2 and c.allocator.num_free == 2
    c.truncate("r1", 3)
    assert c.length("r1") == 3 and c.num_blocks_in_use("r1") == 1 and c.allocator.num_free == 3
    c.truncate("r1", 0)
    assert c.num_blocks_in_use("r1") == 0 and c.allocator.num_free == 4
    with pytest.raises(ValueError):
        c.truncate("r1", 1)

    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=4)
    c.create_request("r1")
    c.append("r1", _kv(1, 1, 8, 2, 1.0), _kv(1, 1, 8, 2, 1.0))
    c.truncate("r1", 4)
    assert c.num_blocks_in_use("r1") == 1 and c.allocator.num_free == 3

    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=4)
    c.create_request("r1")
    c.append("r1", _kv(1, 1, 7, 2, 1.0), _kv(1, 1, 7, 2, 1.0))
    assert c.allocator.num_free == 2
    c.free_request("r1")
    assert c.allocator.num_free == 4
    c.create_request("x")
    with pytest.raises(ValueError):
        c.create_request("x")


def test_no_aliasing_and_padding_mask():
    P = _pse()
    c = P.PagedKVCache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=8)
    c.create_request("a")
    c.create_request("b")
    c.append("a", _kv(1, 1, 2, 2, 10.0), _kv(1, 1, 2, 2, 10.0))
    c.append("b", _kv(1, 1, 2, 2, 20.0), _kv(1, 1, 2, 2, 20.0))
    c.append("a", _kv(1, 1, 5, 2, 10.0), _kv(1, 1, 5, 2, 10.0))
    c.append("b", _kv(1, 1, 5, 2, 20.0), _kv(1, 1, 5, 2, 20.0))
    ko, _, _, lens = c.gather(["a", "b"])
    assert lens.tolist() == [7, 7]
    assert torch.equal(ko[0][0, :, :7].cpu(), torch.full((1, 7, 2), 10.0))
    assert torch.equal(ko[0][1, :, :7].cpu(), torch.full((1, 7, 2), 20.0))
    c.create_request("short")
    c.create_request("long")
    c.append("short", _kv(1, 1, 2, 2, 1.0), _kv(1, 1, 2, 2, 1.0))
    c.append("long", _kv(1, 1, 6, 2, 2.0), _kv(1, 1, 6, 2, 2.0))
    _, _, mask, lens = c.gather(["short", "long"])
    assert lens.tolist() == [2, 6]
    assert mask[0].tolist() == [True, True, False, False, False, False]
    assert mask[1].tolist() == [True] * 6


OPS = st.one_of(
    st.tuples(st.just("append"), st.sampled_from(["r0", "r1", "r2"]), st.integers(1, 5)),
    st.tuples(st.just("truncate"), st.sampled_from(["r0", "r1", "r2"]), st.integers(0, 20)),
    st.tuples(st.just("free"), st.sampled_from(["r0", "r1", "r2"]), st.just(0)),
)


@settings(max_examples=60, deadline=None)
@given(ops=st.lists(OPS, min_size=1, max_size=30))
def test_random_op_sequences_keep_conservation_and_content(ops):
    P = _pse()
    NB = 16
    c = P.PagedKVCache(1, 1, 2, 4, NB)
    truth: dict[str, list[float]] = {}
    fill = 100.0
    for kind, rid, arg in ops:
        if kind == "append":
            if rid not in truth:
                c.create_request(rid)
                truth[rid] = []
            fill += 1.0
            try:
                c.append(rid, [torch.full((1, arg, 2), fill)], [torch.full((1, arg, 2), fill)])
            except MemoryError:
                assume(False)
            truth[rid].extend([fill] * arg)
        elif kind == "truncate" and rid in truth:
            n = min(arg, c.length(rid))
            c.truncate(rid, n)
            truth[rid] = truth[rid][:n]
        elif kind == "free" and rid in truth:
            c.free_request(rid)
            del truth[rid]
        assert c.allocator.num_free + sum(c.num_blocks_in_use(r) for r in truth) == NB
    if truth:
        order = sorted(truth)
        ko, vo, mask, lens = c.gather(order)
        for i, r in enumerate(order):
            n = len(truth[r])
            assert lens[i].item() == n
            if n:
                want = torch.tensor(truth[r]).view(1, n, 1).expand(1, n, 2)
                assert torch.equal(ko[0][i, :, :n].cpu(), want) and torch.equal(vo[0][i, :, :n].cpu(), want)


# ---------------------------------------------------------------- speculative, single request
def _models(seed, vocab_size=64, d_model=16, n_layers=2, n_heads=2, d_ff=32, max_seq_len=128):
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=vocab_size, d_model=d_model, n_layers=n_layers, n_heads=n_heads, d_ff=d_ff,
                      max_seq_len=max_seq_len)
    return TinyGPT(cfg).eval(), TinyGPT(cfg).eval(), cfg


def _spec(draft, target, cfg, prompt, max_new, k, block_size=4, num_blocks=64):
    P = _pse()
    hd = cfg.d_model // cfg.n_heads
    dc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, num_blocks)
    tc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, num_blocks)
    return P.speculative_generate_batched(draft, target, dc, tc, "r1", prompt, max_new, k=k, temperature=0.0)


def test_single_request_exact_match():
    d, t, cfg = _models(0)
    assert _spec(d, t, cfg, [1, 2, 3, 4], 10, 4) == generate_cached(t, torch.tensor([[1, 2, 3, 4]]), 10)


def test_single_request_several_seeds():
    for seed in range(5):
        d, t, cfg = _models(seed, vocab_size=48, d_model=12)
        prompt = [seed % 10 + 1, (seed + 1) % 10 + 1, (seed + 2) % 10 + 1]
        assert _spec(d, t, cfg, prompt, 8, 3) == generate_cached(t, torch.tensor([prompt]), 8), seed


@pytest.mark.parametrize("seed,prompt,max_new,k", [
    (1, list(range(1, 10)), 6, 4),   # prompt longer than a block
    (2, [5, 6, 7], 11, 3),           # k does not divide block_size
    (3, [2, 4, 6], 13, 6),           # k larger than block_size
])
def test_single_request_block_edges(seed, prompt, max_new, k):
    d, t, cfg = _models(seed)
    assert _spec(d, t, cfg, prompt, max_new, k) == generate_cached(t, torch.tensor([prompt]), max_new)


def test_max_new_tokens_one_and_self_speculation():
    d, t, cfg = _models(4)
    out = _spec(d, t, cfg, [1, 1, 1], 1, 4)
    assert len(out) - 3 == 1
    _, t, cfg = _models(5)
    assert _spec(t, t, cfg, [3, 3, 3], 9, 4) == generate_cached(t, torch.tensor([[3, 3, 3]]), 9)


# ---------------------------------------------------------------- scheduler
def _run(draft, target, cfg, requests, max_batch_size, k=4, block_size=4, num_blocks=128):
    P = _pse()
    hd = cfg.d_model // cfg.n_heads
    dc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, num_blocks)
    tc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, num_blocks)
    return P.run_continuous_speculative_batches(draft, target, requests, dc, tc, max_batch_size, k=k,
                                                temperature=0.0), dc, tc


def test_scheduler_matches_solo_baselines():
    P = _pse()
    d, t, cfg = _models(0, vocab_size=48)
    res, _, _ = _run(d, t, cfg, [P.Request("a", [1, 2, 3], 7)], 4)
    assert res[0].output_ids == generate_cached(t, torch.tensor([[1, 2, 3]]), 7)
    d, t, cfg = _models(7, vocab_size=48)
    reqs = [P.Request("a", [1, 2, 3], 8), P.Request("b", [4, 5], 6), P.Request("c", [6, 7, 8, 9], 10),
            P.Request("d", [2, 2], 5)]
    res, _, _ = _run(d, t, cfg, reqs, 2, k=4)
    by = {r.request_id: r.output_ids for r in res}
    assert len(res) == 4
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens)


def test_scheduler_completion_eviction_no_overshoot():
    P = _pse()
    d, t, cfg = _models(3, vocab_size=48)
    reqs = [P.Request(f"r{i}", [i % 10 + 1, (i + 1) % 10 + 1], 4) for i in range(9)]
    res, _, _ = _run(d, t, cfg, reqs, 3, k=3)
    assert {r.request_id for r in res} == {f"r{i}" for i in range(9)}
    d, t, cfg = _models(1, vocab_size=48)
    _, dc, tc = _run(d, t, cfg, [P.Request("a", [1, 2], 5)], 2, k=3, num_blocks=16)
    assert dc.allocator.num_free == 16 and tc.allocator.num_free == 16
    d, t, cfg = _models(2, vocab_size=48)
    res, _, _ = _run(d, t, cfg, [P.Request("a", [1, 1], 1), P.Request("b", [2, 2], 1)], 4, k=4)
    assert all(len(r.output_ids) - 2 == 1 for r in res)


def test_scheduler_batch_pressure_many_seeds():
    P = _pse()
    for seed in range(4):
        d, t, cfg = _models(seed, vocab_size=40, d_model=12)
        reqs = [P.Request(f"r{i}", [(i + j) % 10 + 1 for j in range(2 + i % 3)], 5 + i % 4) for i in range(6)]
        res, _, _ = _run(d, t, cfg, reqs, 2, k=3)
        by = {r.request_id: r.output_ids for r in res}
        for q in reqs:
            want = generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens)
            assert by[q.request_id] == want, (seed, q.request_id)


REQ = st.tuples(st.lists(st.integers(1, 31), min_size=1, max_size=5), st.integers(1, 8))


@settings(max_examples=120, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(seed=st.integers(0, 1000), spec=st.lists(REQ, min_size=1, max_size=6, unique_by=lambda r: tuple(r[0])),
       max_batch_size=st.integers(1, 4), k=st.integers(1, 5), block_size=st.integers(1, 5))
def test_scheduler_property_every_request_matches_solo(seed, spec, max_batch_size, k, block_size):
    P = _pse()
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=32, d_model=12, n_layers=2, n_heads=2, d_ff=24, max_seq_len=256)
    d, t = TinyGPT(cfg).eval(), TinyGPT(cfg).eval()
    reqs = [P.Request(f"r{i}", p, m) for i, (p, m) in enumerate(spec)]
    ceiling = sum(len(r.prompt_ids) + r.max_new_tokens + k + 1 for r in reqs)
    nb = (ceiling // block_size + 1) * len(reqs) + 4
    hd = cfg.d_model // cfg.n_heads
    dc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, nb)
    tc = P.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, nb)
    res = P.run_continuous_speculative_batches(d, t, reqs, dc, tc, max_batch_size, k=k, temperature=0.0)
    by = {r.request_id: r.output_ids for r in res}
    assert set(by) == {r.request_id for r in reqs}
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), (
            seed, k, block_size, max_batch_size, q)
