"""Properties of the CPU oracle itself, beyond the golden vectors: the
reference's own property tests (tests/test_paged_cache_properties.py:34-100,
tests/test_scheduler_properties.py:49-81) run against the oracle, the
device-allocator restatement (``oracle.alloc.BlockState``) against the
sequential cache under random op sequences, the greedy accept rule, the
scheduler's per-row commit, the reference's distribution test on the
explicit-uniform accept rule, the paged-attention oracle against the model's
masked attention, the batched forward over ragged rows against each row's
own forward, the Llama-style restatement (RoPE, cached against
recomputed decoding, the reference scheduler over GQA caches), and
Philox4x32-10 against the published known-answer vectors.  CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import alloc
from oracle.accept import accept_row
from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT
from oracle.paged_cache import PagedKVCache
from oracle.philox import philox4x32_10
from oracle.scheduler import Request, commit_rows, run_continuous_speculative_batches


# Random123's kat_vectors for philox4x32_10: (counter, key) -> output words.
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers():
    for ctr, key, want in PHILOX_KAT:
        got = philox4x32_10(np.array(ctr, dtype=np.uint32), np.array(key, dtype=np.uint32))
        assert [int(x) for x in got] == list(want)
    # vectorised form: the same vectors stacked give the same words
    ctrs = np.array([c for c, _, _ in PHILOX_KAT], dtype=np.uint32)
    keys = np.array([k for _, k, _ in PHILOX_KAT], dtype=np.uint32)
    assert philox4x32_10(ctrs, keys).tolist() == [list(w) for _, _, w in PHILOX_KAT]


NUM_BLOCKS = 16
RIDS = ("a", "b", "c")
OP = st.one_of(
    st.tuples(st.just("append"), st.sampled_from(RIDS), st.integers(1, 9)),
    st.tuples(st.just("truncate"), st.sampled_from(RIDS), st.integers(0, 40)),
    st.tuples(st.just("free"), st.sampled_from(RIDS), st.just(0)),
)


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(ops=st.lists(OP, min_size=1, max_size=40), block_size=st.integers(1, 5), seed=st.integers(0, 2**16))
def test_block_state_tracks_sequential_cache(ops, block_size, seed):
    """The reference's cache property (block conservation after every op,
    content fidelity through gather) on the oracle cache, with the batched
    prefix-scan restatement driven alongside: same tables, lengths and free
    list after every op, exhaustion included (the reference's test discards
    exhausted draws; here both sides must agree on the state they leave)."""
    g = torch.Generator().manual_seed(seed)
    cache = PagedKVCache(1, 2, 3, block_size, NUM_BLOCKS)
    bs = alloc.BlockState(NUM_BLOCKS, block_size, num_slots=len(RIDS), max_blocks=NUM_BLOCKS + 10)
    slot = {r: i for i, r in enumerate(RIDS)}
    shadow: dict[str, list[torch.Tensor]] = {}
    for r in RIDS:
        cache.create_request(r)
        shadow[r] = []
    for kind, r, n in ops:
        if kind == "append":
            k = torch.randn(2, n, 3, generator=g)
            try:
                cache.append(r, [k], [k + 1])
            except MemoryError:
                bs.status = 0
                bs.reserve([slot[r]], n)
                assert bs.status & alloc.OOM
                # the reference keeps the blocks the failed append got; the
                # row's length (and so what gather returns) is unchanged
                bs.status = 0
            else:
                bs.reserve([slot[r]], n)
                assert bs.status == 0
                shadow[r].extend(k.unbind(1))
        elif kind == "truncate":
            m = min(n, cache.length(r))
            cache.truncate(r, m)
            bs.truncate([slot[r]], [m])
            del shadow[r][m:]
        else:
            cache.free_request(r)
            cache.create_request(r)
            bs.release([slot[r]])
            shadow[r] = []
        assert bs.status == 0
        used = sum(cache.num_blocks_in_use(x) for x in RIDS)
        assert cache.allocator.num_free + used == NUM_BLOCKS
        assert bs.free_list() == cache.allocator.free_list()
        for x in RIDS:
            assert bs.row_table(slot[x]) == cache.block_table(x)
            assert int(bs.seq_len[slot[x]]) == cache.length(x)
    lens = [cache.length(x) for x in RIDS]
    if max(lens) == 0:
        return
    (kk,), (vv,), mask, _ = cache.gather(list(RIDS))
    for i, x in enumerate(RIDS):
        assert mask[i].tolist() == [j < lens[i] for j in range(max(lens))]
        if lens[i]:
            want = torch.stack(shadow[x], 1)
            assert torch.equal(kk[i, :, : lens[i]], want)
            assert torch.equal(vv[i, :, : lens[i]], want + 1)
        assert not kk[i, :, lens[i]:].any()


def test_block_state_reports_errors_instead_of_raising():
    """The reference raises ValueError on truncate past the length
    (engine/paged_cache.py:140-154) and on a double free (:50-56); the
    restatement records them in its status word, which the device mirrors."""
    bs = alloc.BlockState(8, 2, num_slots=2, max_blocks=8)
    bs.reserve([0], 3)
    bs.truncate([0], [5])
    assert bs.status & alloc.TRUNCATE_BEYOND_LENGTH
    assert int(bs.seq_len[0]) == 3 and bs.row_table(0) == [7, 6]
    bs.status = 0
    bs._push([[0]])  # block 0 is still free
    assert bs.status & alloc.DOUBLE_FREE
    bs = alloc.BlockState(4, 2, num_slots=1, max_blocks=2)
    bs.reserve([0], 5)
    assert bs.status & alloc.TABLE_OVERFLOW and bs.free_list() == [0, 1, 2, 3]
    cache = PagedKVCache(1, 1, 1, 2, 8)
    cache.create_request("a")
    cache.append("a", [torch.ones(1, 3, 1)], [torch.ones(1, 3, 1)])
    with pytest.raises(ValueError):
        cache.truncate("a", 5)
    with pytest.raises(ValueError):
        cache.allocator.free(0)
    with pytest.raises(MemoryError):
        cache.append("a", [torch.ones(1, 20, 1)], [torch.ones(1, 20, 1)])


REQ = st.tuples(st.lists(st.integers(1, 31), min_size=1, max_size=5), st.integers(1, 8))


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(seed=st.integers(0, 1000), spec=st.lists(REQ, min_size=1, max_size=5, unique_by=lambda r: tuple(r[0])),
       max_batch_size=st.integers(1, 4), k=st.integers(1, 5), block_size=st.integers(1, 5))
def test_oracle_scheduler_matches_solo_generation(seed, spec, max_batch_size, k, block_size):
    """The reference's main conformance property on the oracle: every request
    through the continuous speculative scheduler at T = 0 equals its solo
    ``generate_cached``, and both caches get every block back."""
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=32, d_model=12, n_layers=2, n_heads=2, d_ff=24, max_seq_len=256)
    d, t = TinyGPT(cfg).eval(), TinyGPT(cfg).eval()
    reqs = [Request(f"r{i}", p, m) for i, (p, m) in enumerate(spec)]
    ceiling = sum(len(r.prompt_ids) + r.max_new_tokens + k + 1 for r in reqs)
    nb = (ceiling // block_size + 1) * len(reqs) + 4
    hd = cfg.d_model // cfg.n_heads
    dc = PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, nb)
    tc = PagedKVCache(cfg.n_layers, cfg.n_heads, hd, block_size, nb)
    res = run_continuous_speculative_batches(d, t, reqs, dc, tc, max_batch_size, k=k, temperature=0.0)
    by = {r.request_id: r.output_ids for r in res}
    assert sorted(by) == sorted(r.request_id for r in reqs)
    for r in reqs:
        assert by[r.request_id] == generate_cached(t, torch.tensor([r.prompt_ids]), r.max_new_tokens)
    assert dc.allocator.num_free == nb and tc.allocator.num_free == nb


@settings(max_examples=300, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), k=st.integers(1, 6), vocab=st.integers(2, 9))
def test_greedy_accept_is_longest_agreeing_prefix(seed, k, vocab):
    """engine/speculative.py:146-155: at T = 0 the step keeps the drafts up to
    the first one that differs from the target's argmax, then emits the
    target's argmax there (or the bonus argmax when all k agree)."""
    rng = np.random.default_rng(seed)
    target = rng.standard_normal((k + 1, vocab)).astype(np.float32)
    best = target.argmax(-1)
    drafts = np.where(rng.random(k) < 0.7, best[:k], rng.integers(0, vocab, size=k))
    tokens, n = accept_row(target, None, drafts, None, k, 0.0)
    assert len(tokens) == n + 1
    assert tokens[:n] == drafts[:n].tolist() == best[:n].tolist()
    assert tokens[n] == best[n]
    if n < k:
        assert drafts[n] != best[n]


@settings(max_examples=200, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), n_req=st.integers(1, 12), k=st.integers(1, 5))
def test_commit_rows_counts_and_trims(seed, n_req, k):
    """engine/scheduler.py:107-126 restated on row arrays: a request finishes
    at the first step where its count reaches max_new and leaves exactly
    max_new tokens; an unfinished one holds every token it accepted."""
    rng = np.random.default_rng(seed)
    max_new = rng.integers(0, 15, size=n_req).tolist()
    generated = [0] * n_req
    outputs: list[list[int]] = [[] for _ in range(n_req)]
    stream: list[list[int]] = [[] for _ in range(n_req)]
    live = list(range(n_req))
    while live:
        ords = [int(o) for o in rng.permutation(live)[: int(rng.integers(1, len(live) + 1))]]
        tokens = rng.integers(0, 1000, size=(len(ords), k + 1))
        n_acc = rng.integers(0, k + 1, size=len(ords))
        before = list(generated)
        fin = commit_rows(tokens.tolist(), n_acc.tolist(), ords, generated, max_new, outputs)
        assert fin == sorted(fin)
        for i, o in enumerate(ords):
            stream[o].extend(tokens[i, : n_acc[i] + 1].tolist())
            assert generated[o] == before[o] + n_acc[i] + 1
            done = generated[o] >= max_new[o]
            assert (i in fin) == done
            assert outputs[o] == (stream[o][: max_new[o]] if done else stream[o])
        live = [o for o in live if generated[o] < max_new[o]]


@pytest.mark.parametrize("rows,width,hq,hk,hd,bs,seed", [
    (3, 1, 4, 4, 8, 4, 0),     # width-1 draft/bonus calls, MHA
    (4, 6, 6, 2, 8, 3, 1),     # verify width k + 1, GQA 3, block size not a power of two
    (2, 17, 8, 1, 4, 16, 2),   # prompt-shaped call, one KV head for all query heads
    (5, 4, 2, 2, 16, 1, 3),    # block size 1
])
def test_paged_attention_oracle_equals_model_attention(rows, width, hq, hk, hd, bs, seed):
    """The check of the paged-attention kernels (oracle.attention, float64 on
    the block layout) against the model's own masked attention over the
    reference cache's padded gather (engine/model.py:99-116 with the padding
    mask of engine/batched_forward.py:44), on ragged rows whose blocks come
    from one shared pool in allocation order."""
    from oracle.attention import paged_attention
    from oracle.model import _masked_attention
    g = torch.Generator().manual_seed(seed)
    base = torch.randint(0, 3 * bs + 5, (rows,), generator=g)
    ctx = base + width
    nb = int(sum((int(c) + bs - 1) // bs for c in ctx)) + 2
    cache = PagedKVCache(1, hk, hd, bs, nb, dtype=torch.float64)
    rids = [f"r{i}" for i in range(rows)]
    for r in rids:
        cache.create_request(r)
    # interleaved appends so each row's blocks are scattered through the pool
    done = [0] * rows
    while any(done[i] < int(ctx[i]) for i in range(rows)):
        for i, r in enumerate(rids):
            n = min(int(torch.randint(1, 4, (1,), generator=g)), int(ctx[i]) - done[i])
            if n > 0:
                kv = torch.randn(2, hk, n, hd, generator=g, dtype=torch.float64)
                cache.append(r, [kv[0]], [kv[1]])
                done[i] += n
    q = torch.randn(rows, hq, width, hd, generator=g, dtype=torch.float64)
    (k,), (v,), mask, _ = cache.gather(rids)
    want = _masked_attention(q, k, v, width, base, mask, None)  # [R, Hq, W, hd]
    got = paged_attention(q.permute(0, 2, 1, 3).numpy(), cache._k_pool[0].numpy(), cache._v_pool[0].numpy(),
                          [cache.block_table(r) for r in rids], base.tolist())
    np.testing.assert_allclose(got, want.permute(0, 2, 1, 3).numpy(), rtol=0, atol=1e-12)


def test_rope_keeps_norms_and_depends_on_relative_position():
    """The Llama-style restatement's rotary embedding: each rotation keeps the
    vector's length, and a query-key dot product depends only on the distance
    between their positions (shifting both leaves it unchanged)."""
    from oracle.model import rope_rotate
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, 3, 1, 64, generator=g)
    k = torch.randn(1, 3, 1, 64, generator=g)
    for m, n, shift in ((0, 0, 7), (5, 2, 100), (300, 17, 4000), (1, 1000, 123)):
        qm = rope_rotate(q, torch.tensor([[m]]), 10000.0)
        kn = rope_rotate(k, torch.tensor([[n]]), 10000.0)
        qs = rope_rotate(q, torch.tensor([[m + shift]]), 10000.0)
        ks = rope_rotate(k, torch.tensor([[n + shift]]), 10000.0)
        torch.testing.assert_close(qm.norm(dim=-1), q.norm(dim=-1), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close((qm * kn).sum(-1), (qs * ks).sum(-1), rtol=1e-4, atol=1e-4)
    assert torch.equal(rope_rotate(q, torch.tensor([[0]]), 10000.0), q)


def _llama_pair(seed):
    from oracle.model import LlamaConfig, TinyLlama
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=48, d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, max_seq_len=256)
    return TinyLlama(cfg).eval(), TinyLlama(cfg).eval(), cfg


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_llama_cached_generation_equals_full_recompute(seed):
    """The Llama-style model follows the reference model's forward contract
    (past_kv, position_offset; engine/model.py:158-206): greedy decoding over
    its cache equals decoding that recomputes the whole sequence each token
    (engine/generate.py:12-38), so RoPE positions and the GQA cache agree."""
    from oracle.generate import generate_naive
    _, t, _ = _llama_pair(seed)
    rng = np.random.default_rng(seed)
    for plen in (1, 5, 13):
        prompt = torch.tensor([rng.integers(0, 48, size=plen).tolist()])
        assert generate_cached(t, prompt, 12) == generate_naive(t, prompt, 12)


@pytest.mark.parametrize("seed,k,block_size", [(0, 3, 4), (1, 1, 1), (2, 5, 3)])
def test_llama_pair_through_the_reference_scheduler(seed, k, block_size):
    """The reference scheduler drives the Llama-style pair unchanged over
    caches of n_kv_heads heads: every request equals its solo greedy decode."""
    d, t, cfg = _llama_pair(seed)
    rng = np.random.default_rng(10 + seed)
    reqs = [Request(f"q{i}", rng.integers(0, 48, size=int(rng.integers(1, 9))).tolist(), int(rng.integers(1, 10)))
            for i in range(5)]
    hd = cfg.d_model // cfg.n_heads
    nb = 4 * sum(len(r.prompt_ids) + r.max_new_tokens + k + 1 for r in reqs) // block_size + 8
    dc = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, block_size, nb)
    tc = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, block_size, nb)
    res = run_continuous_speculative_batches(d, t, reqs, dc, tc, 3, k=k, temperature=0.0)
    by = {r.request_id: r.output_ids for r in res}
    for r in reqs:
        assert by[r.request_id] == generate_cached(t, torch.tensor([r.prompt_ids]), r.max_new_tokens)
    assert dc.allocator.num_free == nb and tc.allocator.num_free == nb


@pytest.mark.parametrize("case", [
    dict(seed=0, k=3, T=1.0, same=False),   # independent draft
    dict(seed=1, k=1, T=0.7, same=False),
    dict(seed=2, k=4, T=1.3, same=True),    # draft = target: every draft is accepted
])
def test_sampled_accept_preserves_the_target_distribution(case):
    """The reference's distribution test (tests/test_distribution_preserving.py:
    73-92: 4000 trials, vocab 12, chi-squared p > 0.01 on the first output
    token against softmax(target / T)) on the explicit-uniform accept rule the
    kernels implement: draft token 0 drawn from the draft distribution with
    u[0], then accept / residual / bonus with u[k..2k]."""
    from scipy.stats import chisquare
    from oracle.sampling import sample_with_uniform
    rng = np.random.default_rng(case["seed"])
    k, T, V, trials = case["k"], case["T"], 12, 4000
    target = (rng.standard_normal((k + 1, V)) * 1.5).astype(np.float32)
    draft = target[:k].copy() if case["same"] else (rng.standard_normal((k, V)) * 1.5).astype(np.float32)
    counts = np.zeros(V)
    accepted_first = 0
    for _ in range(trials):
        u = rng.random(2 * k + 1)
        drafts = [sample_with_uniform(draft[j], T, u[j]) for j in range(k)]
        tokens, n = accept_row(target, draft, drafts, u, k, T)
        counts[tokens[0]] += 1
        accepted_first += n > 0
    p = np.exp((target[0].astype(np.float64) - target[0].max()) / T)
    p /= p.sum()
    keep = p * trials >= 5  # the reference renormalises over the cells with enough expected mass
    exp_counts = p[keep] / p[keep].sum() * counts[keep].sum()
    assert chisquare(counts[keep], exp_counts).pvalue > 0.01
    if case["same"]:
        assert accepted_first == trials


@pytest.mark.parametrize("seed,width,block_size", [(0, 1, 4), (1, 3, 2), (2, 5, 16)])
def test_batched_forward_over_ragged_rows_equals_each_rows_own_forward(seed, width, block_size):
    """engine/batched_forward.py:27-72 restated: one padded forward over rows
    of different lengths (gathered from the paged cache, per-row positions)
    gives each row the logits of its own forward over its whole sequence, and
    appends each row's new K/V to its own blocks."""
    from oracle.batched_forward import batched_forward_append
    torch.manual_seed(seed)
    cfg = ModelConfig(vocab_size=40, d_model=16, n_layers=2, n_heads=2, d_ff=32, max_seq_len=128)
    model = TinyGPT(cfg).eval()
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, 40, size=int(n)).tolist() for n in (3, 11, 1, 7)]
    cache = PagedKVCache(cfg.n_layers, cfg.n_heads, cfg.d_model // cfg.n_heads, block_size, 64)
    rids = [f"r{i}" for i in range(len(prompts))]
    for r, p in zip(rids, prompts):  # each prompt prefilled on its own (a batch of one row)
        cache.create_request(r)
        batched_forward_append(model, cache, [r], torch.tensor([p]))
    new = torch.from_numpy(rng.integers(0, 40, size=(len(rids), width)))
    got = batched_forward_append(model, cache, rids, new)
    with torch.no_grad():
        for i, p in enumerate(prompts):
            full = torch.tensor([p + new[i].tolist()])
            want = model(full)[0][0, len(p):]
            torch.testing.assert_close(got[i], want, rtol=1e-5, atol=1e-5)
            assert cache.length(rids[i]) == len(p) + width


@settings(max_examples=300, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), vocab=st.integers(1, 40), temp=st.sampled_from([0.3, 1.0, 2.5]))
def test_inverse_cdf_is_monotone_and_skips_zero_weights(seed, vocab, temp):
    """The explicit-uniform draw the sampling kernels implement: the token is a
    non-decreasing function of u, never a zero-weight entry, and agrees with a
    float64 cumulative-sum search away from bucket edges."""
    from oracle.sampling import inverse_cdf, weights
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal(vocab) * 4).astype(np.float32)
    logits[rng.random(vocab) < 0.2] = -np.inf  # masked-out entries have zero weight
    if np.isinf(logits).all():
        logits[0] = 0.0
    w, z = weights(logits, temp)
    assert w.dtype == np.float32 and z > 0
    us = np.sort(rng.random(64))
    toks = [inverse_cdf(w, float(z), float(u)) for u in us]
    assert toks == sorted(toks)
    assert all(w[t] > 0 for t in toks)
    cdf = np.cumsum(w.astype(np.float64)) / float(z)
    for u, t in zip(us, toks):
        if np.min(np.abs(cdf - u)) > 1e-9:
            assert t == int(np.searchsorted(cdf, u, side="right"))
