"""End-to-end parity of the device engine with golden vectors produced by the
reference itself (tests/golden/): the "tiny" workload (TinyGPT pair, 8
prompts, 64 new tokens, k=4, block 16, batch 4, greedy) must reproduce the
reference's outputs, its per-step accepted tokens and, after every scheduler
step, both caches' block tables, lengths and free lists bit for bit.  GPU only."""
from __future__ import annotations

import json
import os

import pytest
import torch

from conftest import GOLDEN
from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def _tiny():
    from pse import workload as wl
    tiny = wl.WORKLOADS["tiny"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.draft)).eval()
    t = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.target)).eval()
    return tiny, d, t


def _caches(tiny, num_blocks):
    import pse
    pd, pt = tiny.pair.draft, tiny.pair.target
    dc = pse.PagedKVCache(pd["n_layers"], pd["n_heads"], pd["d_model"] // pd["n_heads"], tiny.block_size, num_blocks)
    tc = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], tiny.block_size, num_blocks)
    return dc, tc


def _state(cache):
    return ({r: cache.block_table(r) for r in cache._slot}, dict(cache._lengths), cache.allocator.free_list())


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("defer", [None, False])
def test_tiny_workload_reproduces_reference_trace(graphs, defer):
    """Both step structures: the default (target bonus call deferred into the
    next verify, its position reserved where the reference appends it) and
    the reference's own (bonus call inside the step) leave the same tables,
    lengths and free lists after every step."""
    import pse
    g = _load("tiny_greedy.json")
    tiny, d, t = _tiny()
    dc, tc = _caches(tiny, g["num_blocks"])
    trace = []

    def on_step(ids, res):
        trace.append((list(ids), dict(res.accepted_tokens), _state(dc), _state(tc)))

    reqs = [pse.Request(r, p, tiny.max_new_tokens) for r, p in zip(g["request_ids"], g["prompts"])]
    res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, tiny.max_batch_size, k=tiny.k,
                                                 temperature=0.0, on_step=on_step, use_graph=graphs,
                                                 defer_bonus=defer)
    assert {r.request_id: r.output_ids for r in res} == g["outputs"]
    assert len(trace) == len(g["steps"])
    for n, (got, ref) in enumerate(zip(trace, g["steps"])):
        ids, acc, (dtab, dlen, dfree), (ttab, tlen, tfree) = got
        assert ids == ref["ids"], n
        assert acc == ref["accepted"], n
        assert dtab == ref["draft"]["tables"] and dlen == ref["draft"]["lengths"], n
        assert dfree == ref["draft"]["free"], n
        assert ttab == ref["target"]["tables"] and tlen == ref["target"]["lengths"], n
        assert tfree == ref["target"]["free"], n
    assert dc.allocator.free_list() == g["final_free"]["draft"]
    assert tc.allocator.free_list() == g["final_free"]["target"]
    assert not tc.pending_slots


def test_prompt_logits_match_reference_fp32():
    import pse
    g = _load("tiny_logits.json")
    tiny, _, t = _tiny()
    pt = tiny.pair.target
    c = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], tiny.block_size, 64)
    for i, (p, ref) in enumerate(zip(g["prompts"], g["logits"])):
        rid = f"p{i}"
        c.create_request(rid)
        logits = pse.batched_forward_append(t, c, [rid], torch.tensor([p]))
        assert logits.shape == (1, len(p), tiny.pair.vocab)
        assert (logits[0, -1].cpu() - torch.tensor(ref)).abs().max().item() < 1e-4
        c.free_request(rid)


def test_batched_forward_rows_of_different_lengths_match_solo():
    """Rows of one batched call see only their own blocks and positions
    (engine/batched_forward.py:44-57)."""
    import pse
    tiny, _, t = _tiny()
    pt = tiny.pair.target
    c = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], 5, 200)
    prompts = {"a": [3, 1, 4, 1, 5, 9, 2, 6], "b": [2, 7], "c": list(range(30, 60))}
    for r, p in prompts.items():
        c.create_request(r)
        pse.batched_forward_append(t, c, [r], torch.tensor([p]))
    new = torch.tensor([[11, 12, 13], [21, 22, 23], [31, 32, 33]])
    out = pse.batched_forward_append(t, c, ["a", "b", "c"], new).cpu()
    with torch.no_grad():
        for i, (r, p) in enumerate(prompts.items()):
            full = t(torch.tensor([p + new[i].tolist()]))[0][0, -3:]
            assert (out[i] - full).abs().max().item() < 1e-4
    assert [c.length(r) for r in prompts] == [11, 5, 33]
