"""Deferred target bonus call behind the reference's API (pse/pending.py).

By default the step leaves each row's final token pending in the target cache
(position reserved where the reference's bonus append puts it, K/V written by
the next verify) and returns ``PendingLogits``.  These tests drive the step
with the reference scheduler's call sequence (engine/scheduler.py:98-115: the
returned logits are handed back unchanged) next to the reference structure
(``defer_bonus=False``) on the same fp32 TinyGPT pair, and check: identical
accepted tokens, identical tables / lengths / free lists after every step,
deferred logits that equal the bonus call's when read (1e-4, fp32), and the
cache calls that must complete a pending row first.  GPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.model import ModelConfig, TinyGPT

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4


def _pair():
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=256, d_model=64, n_layers=2, n_heads=2, d_ff=256, max_seq_len=256)).eval()
    t = TinyGPT(ModelConfig(vocab_size=256, d_model=128, n_layers=4, n_heads=4, d_ff=512, max_seq_len=256)).eval()
    return d, t


def _caches(nb=400, bs=8):
    import pse
    return pse.PagedKVCache(2, 2, 32, bs, nb), pse.PagedKVCache(4, 4, 32, bs, nb)


def _state(c):
    return ({r: c.block_table(r) for r in c._slot}, dict(c._lengths), c.allocator.free_list())


def _prompts(n, seed):
    rng = np.random.default_rng(seed)
    return {f"r{i}": rng.integers(0, 256, size=int(rng.integers(3, 40))).tolist() for i in range(n)}


@pytest.mark.parametrize("graphs", [False, True])
def test_reference_call_sequence_defers_and_matches_reference_structure(graphs):
    import pse
    from pse.pending import PendingLogits
    d, t = _pair()
    prompts = _prompts(5, 1)
    runs = {}
    for defer in (False, None):
        dc, tc = _caches()
        ids = list(prompts)
        dn, tn = {}, {}
        for r, p in prompts.items():
            dn[r], tn[r] = pse.prefill_request(d, t, dc, tc, r, p)
        steps = []
        for step in range(7):
            res = pse.batched_speculative_step(d, t, ids, dc, tc, dn, tn, 3, 0.0, use_graph=graphs,
                                               defer_bonus=defer)
            dn = dict(res.draft_next_logits)
            tn = dict(res.target_next_logits)
            read = {}
            if step in (2, 5):  # the caller reads some rows' target logits now and then
                read = {r: tn[r].cpu().clone() for r in ids[1:3]}
            steps.append((dict(res.accepted_tokens), _state(dc), _state(tc), read,
                          {r: type(v) for r, v in tn.items()}))
        full = {r: tn[r].cpu().clone() for r in ids}  # read every row at the end
        runs[defer] = (steps, full, tc)
    eager, deferred = runs[False], runs[None]
    for n, (a, b) in enumerate(zip(eager[0], deferred[0])):
        assert a[0] == b[0], n                   # accepted tokens
        assert a[1] == b[1] and a[2] == b[2], n  # both caches' tables, lengths, free lists
        for r, v in b[3].items():
            assert (v - eager[0][n][3][r]).abs().max().item() < F32_TOL, (n, r)
        assert all(c is not PendingLogits for c in a[4].values())
        assert all(c is PendingLogits for c in b[4].values())
    for r in eager[1]:
        assert (eager[1][r] - deferred[1][r]).abs().max().item() < F32_TOL, r
    assert not deferred[2].pending_slots  # reading completed every pending row


def test_pending_rows_complete_before_cache_calls_that_read_or_extend_them():
    import pse
    d, t = _pair()
    prompts = _prompts(3, 2)
    outs = {}
    for defer in (False, None):
        dc, tc = _caches()
        ids = list(prompts)
        dn, tn = {}, {}
        for r, p in prompts.items():
            dn[r], tn[r] = pse.prefill_request(d, t, dc, tc, r, p)
        for _ in range(3):
            res = pse.batched_speculative_step(d, t, ids, dc, tc, dn, tn, 4, 0.0, defer_bonus=defer)
            dn, tn = dict(res.draft_next_logits), dict(res.target_next_logits)
        if defer is None:
            assert tc.pending_slots == {tc.slot(r) for r in ids}
        k_layers, v_layers, mask, lengths = tc.gather(["r0"])
        assert tc.slot("r0") not in tc.pending_slots
        more = pse.batched_forward_append(t, tc, ["r1"], torch.tensor([[5, 6]]))
        tc.truncate("r2", tc.length("r2") - 1)
        res = pse.batched_speculative_step(d, t, ids, dc, tc, dn, tn, 4, 0.0, defer_bonus=defer)
        outs[defer] = ([x.cpu() for x in k_layers], [x.cpu() for x in v_layers], lengths.cpu(), more.cpu(),
                       dict(res.accepted_tokens), _state(tc))
    a, b = outs[False], outs[None]
    for x, y in zip(a[0] + a[1], b[0] + b[1]):
        assert (x - y).abs().max().item() < F32_TOL
    assert torch.equal(a[2], b[2])
    assert (a[3] - b[3]).abs().max().item() < F32_TOL
    assert a[4] == b[4] and a[5] == b[5]


def test_reading_deferred_logits_of_a_freed_request_raises():
    import pse
    d, t = _pair()
    dc, tc = _caches()
    dn, tn = pse.prefill_request(d, t, dc, tc, "a", [1, 2, 3, 4])
    res = pse.batched_speculative_step(d, t, ["a"], dc, tc, {"a": dn}, {"a": tn}, 2, 0.0)
    x = res.target_next_logits["a"]
    assert x.shape == (256,) and x.dtype == torch.float32  # metadata needs no call
    dc.free_request("a")
    tc.free_request("a")
    assert tc.allocator.num_free == 400
    with pytest.raises(RuntimeError):
        x.argmax()
    # the slot's next occupant is unaffected
    dn, tn = pse.prefill_request(d, t, dc, tc, "b", [7, 8, 9])
    res = pse.batched_speculative_step(d, t, ["b"], dc, tc, {"b": dn}, {"b": tn}, 2, 0.0)
    assert int(res.target_next_logits["b"].argmax()) >= 0
