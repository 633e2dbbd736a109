"""Pin the CPU oracle against vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import torch

from conftest import GOLDEN
from oracle import alloc
from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT
from oracle.paged_cache import PagedKVCache
from oracle.scheduler import Request, run_continuous_speculative_batches
from pse import workload as wl


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def _state_sha(model) -> str:
    h = hashlib.sha256()
    for name, t in model.state_dict().items():
        h.update(name.encode())
        h.update(t.detach().contiguous().float().numpy().tobytes())
    return h.hexdigest()


def _tiny_pair():
    tiny = wl.WORKLOADS["tiny"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.draft)).eval()
    t = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.target)).eval()
    return tiny, d, t


def test_constructor_draws_reference_weights():
    for case in _load("init_checksums.json"):
        torch.manual_seed(case["seed"])
        if "cfg" in case:
            a = TinyGPT(ModelConfig(**case["cfg"]))
            b = TinyGPT(ModelConfig(**case["cfg"]))
            assert _state_sha(a) == case["sha_first"]
            assert _state_sha(b) == case["sha_second"]
        else:
            _, d, t = _tiny_pair()
            assert _state_sha(d) == case["sha_draft"]
            assert _state_sha(t) == case["sha_target"]


def test_prompt_logits_match_reference():
    g = _load("tiny_logits.json")
    _, _, t = _tiny_pair()
    with torch.no_grad():
        for p, ref in zip(g["prompts"], g["logits"]):
            got = t(torch.tensor([p]))[0][0, -1]
            assert torch.allclose(got, torch.tensor(ref), atol=1e-5, rtol=0)


def test_generate_cached_matches_reference():
    g = _load("tiny_greedy.json")
    tiny, _, t = _tiny_pair()
    for rid, p in zip(g["request_ids"], g["prompts"][:3]):
        assert generate_cached(t, torch.tensor([p]), tiny.max_new_tokens) == g["generate_cached"][rid]


def test_scheduler_trace_matches_reference_step_by_step():
    """Outputs, per-step accepted tokens and both caches' block tables, lengths
    and free lists equal the reference's after every scheduler step."""
    g = _load("tiny_greedy.json")
    tiny, d, t = _tiny_pair()
    n_layers_d, heads_d = tiny.pair.draft["n_layers"], tiny.pair.draft["n_heads"]
    n_layers_t, heads_t = tiny.pair.target["n_layers"], tiny.pair.target["n_heads"]
    dc = PagedKVCache(n_layers_d, heads_d, tiny.pair.draft["d_model"] // heads_d, tiny.block_size, g["num_blocks"])
    tc = PagedKVCache(n_layers_t, heads_t, tiny.pair.target["d_model"] // heads_t, tiny.block_size, g["num_blocks"])
    trace = []

    def on_step(ids, res):
        trace.append((list(ids), dict(res.accepted_tokens),
                      {r: dc.block_table(r) for r in dc._tables}, dict(dc._lengths), dc.allocator.free_list(),
                      {r: tc.block_table(r) for r in tc._tables}, dict(tc._lengths), tc.allocator.free_list()))

    reqs = [Request(r, p, tiny.max_new_tokens) for r, p in zip(g["request_ids"], g["prompts"])]
    res = run_continuous_speculative_batches(d, t, reqs, dc, tc, tiny.max_batch_size, k=tiny.k,
                                             temperature=0.0, on_step=on_step)
    assert {r.request_id: r.output_ids for r in res} == g["outputs"]
    assert len(trace) == len(g["steps"])
    for got, ref in zip(trace, g["steps"]):
        ids, acc, dtab, dlen, dfree, ttab, tlen, tfree = got
        assert ids == ref["ids"]
        assert acc == ref["accepted"]
        assert dtab == ref["draft"]["tables"] and dlen == ref["draft"]["lengths"] and dfree == ref["draft"]["free"]
        assert ttab == ref["target"]["tables"] and tlen == ref["target"]["lengths"] and tfree == ref["target"]["free"]


def _replay(seq, on_state):
    cache = PagedKVCache(1, 1, 2, seq["block_size"], seq["num_blocks"])
    for (kind, rid, n), ref in zip(seq["ops"], seq["states"]):
        if kind == "create":
            cache.create_request(rid)
        elif kind in ("append", "append_oom"):
            try:
                cache.append(rid, [torch.ones(1, n, 2)], [torch.ones(1, n, 2)])
                assert kind == "append"
            except MemoryError:
                assert kind == "append_oom"
        elif kind == "truncate":
            cache.truncate(rid, n)
        else:
            cache.free_request(rid)
        on_state(cache, ref)


def test_cache_op_sequences_match_reference():
    for seq in _load("cache_ops.json"):
        def check(cache, ref):
            assert {r: cache.block_table(r) for r in cache._tables} == ref["tables"]
            assert dict(cache._lengths) == ref["lengths"]
            assert cache.allocator.free_list() == ref["free"]
        _replay(seq, check)


def test_batched_free_list_matches_reference_sequences():
    """The prefix-scan restatement the kernels use, driven op by op, reproduces
    the reference's tables, lengths and free list, exhaustion included."""
    for seq in _load("cache_ops.json"):
        st = alloc.BlockState(seq["num_blocks"], seq["block_size"], num_slots=64, max_blocks=seq["num_blocks"])
        slot_of: dict[str, int] = {}
        free_slots = list(range(63, -1, -1))
        for (kind, rid, n), ref in zip(seq["ops"], seq["states"]):
            if kind == "create":
                slot_of[rid] = free_slots.pop()
            elif kind in ("append", "append_oom"):
                st.status = 0
                st.reserve([slot_of[rid]], n)
                assert bool(st.status & alloc.OOM) == (kind == "append_oom")
            elif kind == "truncate":
                st.truncate([slot_of[rid]], [n])
            else:
                st.release([slot_of[rid]])
                free_slots.append(slot_of.pop(rid))
            assert {r: st.row_table(s) for r, s in slot_of.items()} == ref["tables"]
            assert {r: int(st.seq_len[s]) for r, s in slot_of.items()} == ref["lengths"]
            assert st.free_list() == ref["free"]
            assert st.status & ~alloc.OOM == 0


def test_batched_reserve_equals_sequential_appends():
    """One batched reserve over several rows == the rows' appends in call order."""
    rng = np.random.default_rng(5)
    for trial in range(200):
        nb, bs = int(rng.integers(4, 40)), int(rng.integers(1, 6))
        rows = int(rng.integers(1, 6))
        width = int(rng.integers(1, 9))
        seq = PagedKVCache(1, 1, 1, bs, nb)
        st = alloc.BlockState(nb, bs, num_slots=rows, max_blocks=nb + 8)
        rids = [f"x{i}" for i in range(rows)]
        for i, r in enumerate(rids):
            seq.create_request(r)
            pre = int(rng.integers(0, 6))
            if pre:
                try:
                    seq.append(r, [torch.ones(1, pre, 1)], [torch.ones(1, pre, 1)])
                    st.reserve([i], pre)
                except MemoryError:
                    st.reserve([i], pre)
                    break
        else:
            st.status = 0
            oom = False
            for r in rids:
                try:
                    seq.append(r, [torch.ones(1, width, 1)], [torch.ones(1, width, 1)])
                except MemoryError:
                    oom = True
                    break
            st.reserve(list(range(rows)), width)
            assert bool(st.status & alloc.OOM) == oom
            assert [st.row_table(i) for i in range(rows)] == [seq.block_table(r) for r in rids]
            assert [int(st.seq_len[i]) for i in range(rows)] == [seq.length(r) for r in rids]
            assert st.free_list() == seq.allocator.free_list()


def test_first_token_distributions_match_reference():
    for case in _load("first_token_dists.json"):
        torch.manual_seed(case["seed"])
        cfg = ModelConfig(vocab_size=12, d_model=8, n_layers=1, n_heads=2, d_ff=16, max_seq_len=32)
        TinyGPT(cfg)
        target = TinyGPT(cfg)
        with torch.no_grad():
            probs = torch.softmax(target(torch.tensor([case["prompt"]]))[0][0, -1], -1)
        assert torch.allclose(probs, torch.tensor(case["probs"]), atol=1e-6)


def test_commit_rows_replays_golden_trace_to_golden_outputs():
    """The scheduler's per-row bookkeeping restated on row arrays (the check of
    pse_sched_commit) turns the reference's per-step accepted tokens into the
    reference's outputs, finishing each request at the step the trace drops it."""
    from oracle.scheduler import commit_rows
    g = _load("tiny_greedy.json")
    tiny = wl.WORKLOADS["tiny"]
    ids = g["request_ids"]
    ordinal = {r: i for i, r in enumerate(ids)}
    outputs = [[] for _ in ids]
    generated = [0] * len(ids)
    max_new = [tiny.max_new_tokens] * len(ids)
    steps = g["steps"]
    for n, step in enumerate(steps):
        rows = step["ids"]
        width = max(len(v) for v in step["accepted"].values())
        tokens = [step["accepted"][r] + [-1] * (width - len(step["accepted"][r])) for r in rows]
        n_acc = [len(step["accepted"][r]) - 1 for r in rows]
        fin = commit_rows(tokens, n_acc, [ordinal[r] for r in rows], generated, max_new, outputs)
        still = set(steps[n + 1]["ids"]) if n + 1 < len(steps) else set()
        assert [rows[i] for i in fin] == [r for r in rows if r not in still]
    for r, p in zip(ids, g["prompts"]):
        assert p + outputs[ordinal[r]] == g["outputs"][r]
