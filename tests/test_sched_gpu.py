"""Scheduler bookkeeping on the device (engine/scheduler.py:107-126):
``pse_sched_commit`` against the oracle's ``commit_rows`` on random step
sequences (bit-exact: arena contents, generated counts, finished rows in row
order), and the scheduler's device-bookkeeping loop against its per-row host
loop and the reference's golden outputs.  GPU only."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle.model import ModelConfig, TinyGPT
from oracle.scheduler import commit_rows

pytestmark = pytest.mark.gpu


def _commit_case(n_req, max_rows, k, seed, steps=60):
    import pse._native as N
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda")
    max_new = rng.integers(0, 40, size=n_req)
    max_new[rng.random(n_req) < 0.05] = 0
    off = np.zeros(n_req, dtype=np.int64)
    np.cumsum(max_new[:-1], out=off[1:])
    d_off = torch.from_numpy(off).to(dev)
    d_max = torch.from_numpy(max_new.astype(np.int32)).to(dev)
    d_gen = torch.zeros(n_req, dtype=torch.int32, device=dev)
    d_out = torch.full((max(1, int(max_new.sum())),), -7, dtype=torch.int32, device=dev)
    generated = [0] * n_req
    outputs = [[] for _ in range(n_req)]
    done = np.zeros(n_req, dtype=bool)
    st = N.stream_ptr()
    for _ in range(steps):
        live = np.flatnonzero(~done)
        if len(live) == 0:
            break
        rows = int(min(len(live), rng.integers(1, max_rows + 1)))
        ords = rng.permutation(live)[:rows].astype(np.int32)
        tokens = rng.integers(0, 50000, size=(rows, k + 1)).astype(np.int32)
        n_acc = rng.integers(0, k + 1, size=rows).astype(np.int32)
        d_tok = torch.from_numpy(tokens).to(dev)
        d_nacc = torch.from_numpy(n_acc).to(dev)
        d_ords = torch.from_numpy(ords).to(dev)
        d_fin = torch.full((rows + 1,), -1, dtype=torch.int32, device=dev)
        N.call("pse_sched_commit", d_tok.data_ptr(), k + 1, d_nacc.data_ptr(), d_ords.data_ptr(), rows,
               d_off.data_ptr(), d_max.data_ptr(), d_gen.data_ptr(), d_out.data_ptr(), d_fin.data_ptr(), st)
        fin = commit_rows(tokens.tolist(), n_acc.tolist(), ords.tolist(), generated, max_new.tolist(), outputs)
        got = d_fin.cpu().numpy()
        assert got[0] == len(fin)
        assert got[1:1 + len(fin)].tolist() == fin
        done[ords[fin]] = True
    assert d_gen.cpu().tolist() == generated
    out = d_out.cpu().numpy()
    for o in range(n_req):
        m = min(generated[o], int(max_new[o]))
        assert out[off[o]:off[o] + m].tolist() == outputs[o][:m], o


@pytest.mark.parametrize("n_req,max_rows,k,seed", [
    (40, 16, 4, 0),       # small batches, many steps per request
    (3000, 2500, 5, 1),   # more rows than one CTA pass (the finished list carries across passes)
    (1100, 1024, 1, 2),   # exactly one full pass, k = 1
    (200, 200, 8, 3),
])
def test_sched_commit_matches_oracle(n_req, max_rows, k, seed):
    _commit_case(n_req, max_rows, k, seed)


def test_sched_commit_zero_rows_and_bad_args():
    import pse._native as N
    dev = torch.device("cuda")
    fin = torch.full((1,), 5, dtype=torch.int32, device=dev)
    N.call("pse_sched_commit", None, 1, None, None, 0, None, None, None, None, fin.data_ptr(), N.stream_ptr())
    assert fin.item() == 0
    lib = N.load()
    assert lib.pse_sched_commit(None, 0, None, None, 0, None, None, None, None, fin.data_ptr(), None) != 0
    assert lib.pse_sched_commit(None, 2, None, None, 3, None, None, None, None, fin.data_ptr(), None) != 0


def _pair(vocab=64, seed=0):
    torch.manual_seed(seed)
    dcfg = ModelConfig(vocab_size=vocab, d_model=32, n_layers=2, n_heads=2, d_ff=64, max_seq_len=256)
    tcfg = ModelConfig(vocab_size=vocab, d_model=64, n_layers=3, n_heads=4, d_ff=128, max_seq_len=256)
    return TinyGPT(dcfg).eval(), TinyGPT(tcfg).eval()


def _run(d, t, reqs, mb, k, T, *, device_bookkeeping, **kw):
    import pse
    dc = pse.PagedKVCache(2, 2, 16, 8, 600)
    tc = pse.PagedKVCache(3, 4, 16, 8, 600)
    res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, mb, k=k, temperature=T,
                                                 device_bookkeeping=device_bookkeeping, **kw)
    return ([(r.request_id, r.output_ids) for r in res], dc.allocator.free_list(), tc.allocator.free_list())


@pytest.mark.parametrize("T,defer,graphs,source", [
    (0.0, False, True, None), (0.0, True, True, None), (0.0, False, False, None),
    (1.0, False, True, "philox"), (1.0, True, True, "philox"), (1.0, False, True, "uniform_fn"),
    (0.8, True, False, "generator"),
])
def test_device_bookkeeping_equals_host_loop(T, defer, graphs, source):
    """Same requests, same order of results, same tokens and free lists whether
    the per-row bookkeeping runs on the device or on the host."""
    import pse
    from oracle.philox import request_key, step_uniforms
    d, t = _pair()
    rng = np.random.default_rng(5)
    k = 3
    prompts = [rng.integers(0, 64, size=int(rng.integers(3, 20))).tolist() for _ in range(11)]
    max_new = [int(x) for x in rng.integers(0, 30, size=11)]
    outs = []
    for dev_bk in (True, False):
        reqs = [pse.Request(f"q{i}", p, m) for i, (p, m) in enumerate(zip(prompts, max_new))]
        kw = dict(use_graph=graphs, defer_bonus=defer)
        if source == "uniform_fn":
            kw["uniform_fn"] = lambda ids, steps, n: step_uniforms(77, [request_key(r) for r in ids], steps, n)
        if source == "generator":
            kw["generator"] = torch.Generator().manual_seed(3)
        outs.append(_run(d, t, reqs, 4, k, T, device_bookkeeping=dev_bk, **kw))
    assert outs[0] == outs[1]
    assert sorted(r for r, _ in outs[0][0]) == sorted(f"q{i}" for i in range(11))


def test_device_bookkeeping_reproduces_golden_outputs():
    """The reference's tiny workload (golden outputs and final free lists)
    through the default scheduler loop, which keeps the bookkeeping on the device."""
    import pse
    from pse import workload as wl
    with open(os.path.join(GOLDEN, "tiny_greedy.json")) as f:
        g = json.load(f)
    tiny = wl.WORKLOADS["tiny"]
    torch.manual_seed(0)
    d = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.draft)).eval()
    t = TinyGPT(ModelConfig(vocab_size=tiny.pair.vocab, **tiny.pair.target)).eval()
    pd, pt = tiny.pair.draft, tiny.pair.target
    for defer in (False, True):
        dc = pse.PagedKVCache(pd["n_layers"], pd["n_heads"], pd["d_model"] // pd["n_heads"], tiny.block_size,
                              g["num_blocks"])
        tc = pse.PagedKVCache(pt["n_layers"], pt["n_heads"], pt["d_model"] // pt["n_heads"], tiny.block_size,
                              g["num_blocks"])
        reqs = [pse.Request(r, p, tiny.max_new_tokens) for r, p in zip(g["request_ids"], g["prompts"])]
        res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, tiny.max_batch_size, k=tiny.k,
                                                     temperature=0.0, defer_bonus=defer)
        assert {r.request_id: r.output_ids for r in res} == g["outputs"]
        assert dc.allocator.free_list() == g["final_free"]["draft"]
        assert tc.allocator.free_list() == g["final_free"]["target"]
        assert dc.allocator.num_free == g["num_blocks"] and tc.allocator.num_free == g["num_blocks"]


def test_on_step_with_device_bookkeeping_is_refused():
    import pse
    d, t = _pair()
    with pytest.raises(ValueError):
        _run(d, t, [pse.Request("a", [1, 2], 3)], 2, 2, 0.0, device_bookkeeping=True, on_step=lambda i, r: None)


def _state(cache):
    return ({r: cache.block_table(r) for r in cache._slot}, dict(cache._lengths), cache.allocator.free_list())


def test_device_bookkeeping_raises_like_host_loop_when_the_pool_runs_dry():
    """A pool too small for the run: both loops raise MemoryError at the same
    step and leave both caches (tables, lengths, free lists) in the same state."""
    import pse
    d, t = _pair()
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 64, size=12).tolist() for _ in range(4)]
    states = []
    for dev in (True, False):
        reqs = [pse.Request(f"m{i}", p, 40) for i, p in enumerate(prompts)]
        dc = pse.PagedKVCache(2, 2, 16, 8, 14)
        tc = pse.PagedKVCache(3, 4, 16, 8, 14)
        with pytest.raises(MemoryError):
            pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, 4, k=3, temperature=0.0,
                                                   device_bookkeeping=dev)
        states.append((_state(dc), _state(tc)))
    assert states[0] == states[1]


def test_device_bookkeeping_rejects_duplicate_ids_like_host_loop():
    import pse
    d, t = _pair()
    for dev in (True, False):
        reqs = [pse.Request("dup", [1, 2, 3], 4), pse.Request("dup", [4, 5], 4)]
        dc = pse.PagedKVCache(2, 2, 16, 8, 64)
        tc = pse.PagedKVCache(3, 4, 16, 8, 64)
        with pytest.raises(ValueError):
            pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, 4, k=2, temperature=0.0,
                                                   device_bookkeeping=dev)


@pytest.mark.parametrize("rows,k", [(1, 1), (7, 3), (300, 5), (2500, 8)])
def test_step_glue_kernels_match_their_tensor_statements(rows, k):
    """The step's integer hand-offs (pse_step_verify_ids, pse_step_bonus_ids,
    pse_step_finish) equal the tensor operations they replace, bit for bit,
    including rows that accepted every draft and slots outside the table."""
    import pse._native as N
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(rows * 10 + k)
    n_slots = rows + 17
    slots_d = torch.randperm(n_slots, generator=g)[:rows].to(torch.int32)
    slots_t = torch.randperm(n_slots, generator=g)[:rows].to(torch.int32)
    drafts = torch.randint(0, 32000, (rows, k), generator=g, dtype=torch.int32)
    final = torch.randint(0, 32000, (rows,), generator=g, dtype=torch.int32)
    n_acc = torch.randint(0, k + 1, (rows,), generator=g, dtype=torch.int32)
    n_acc[::3] = k  # every draft accepted
    base = torch.randint(1, 5000, (rows,), generator=g, dtype=torch.int32)
    last = torch.randint(0, 32000, (n_slots,), generator=g, dtype=torch.int32)
    tokens = torch.randint(-1, 32000, (rows, k + 1), generator=g, dtype=torch.int32)
    to = lambda t: t.to(dev)
    slots_d, slots_t, drafts, final, n_acc, base, last, tokens = map(
        to, (slots_d, slots_t, drafts, final, n_acc, base, last, tokens))
    st = N.stream_ptr()
    # verify ids from pending rows
    ids = torch.full((rows, k + 1), -9, dtype=torch.int32, device=dev)
    first = torch.full((rows,), -9, dtype=torch.int32, device=dev)
    N.call("pse_step_verify_ids", last.data_ptr(), n_slots, slots_t.data_ptr(), drafts.data_ptr(), base.data_ptr(),
           rows, k, ids.data_ptr(), first.data_ptr(), st)
    want = torch.cat([last.index_select(0, slots_t.long()).view(-1, 1), drafts], dim=1)
    assert torch.equal(ids, want) and torch.equal(first, base - 1)
    # the draft's tail call
    ids2 = torch.full((rows, 2), -9, dtype=torch.int32, device=dev)
    pos = torch.full((rows,), -9, dtype=torch.int32, device=dev)
    sel = torch.full((rows,), -9, dtype=torch.int64, device=dev)
    N.call("pse_step_bonus_ids", n_acc.data_ptr(), drafts.data_ptr(), final.data_ptr(), base.data_ptr(), rows, k,
           ids2.data_ptr(), pos.data_ptr(), sel.data_ptr(), st)
    full = n_acc.eq(k)
    assert torch.equal(ids2[:, 0], torch.where(full, drafts[:, k - 1], final))
    assert torch.equal(ids2[:, 1], final)
    assert torch.equal(pos, base + torch.clamp(n_acc, max=k - 1))
    assert torch.equal(sel, torch.arange(0, 2 * rows, 2, device=dev) + full)
    # end of the step
    last_d, last_t = last.clone(), last.clone().flip(0).contiguous()
    want_d, want_t = last_d.clone(), last_t.clone()
    want_d.index_copy_(0, slots_d.long(), final)
    want_t.index_copy_(0, slots_t.long(), final)
    sd_word = torch.tensor([5], dtype=torch.int32, device=dev)
    st_word = torch.tensor([32], dtype=torch.int32, device=dev)
    pack = torch.full((rows * (k + 2) + 2,), -9, dtype=torch.int32, device=dev)
    N.call("pse_step_finish", final.data_ptr(), slots_d.data_ptr(), slots_t.data_ptr(), rows, last_d.data_ptr(),
           n_slots, last_t.data_ptr(), n_slots, tokens.data_ptr(), k, n_acc.data_ptr(), sd_word.data_ptr(),
           st_word.data_ptr(), pack.data_ptr(), st)
    torch.cuda.synchronize()
    assert torch.equal(last_d, want_d) and torch.equal(last_t, want_t)
    nt = rows * (k + 1)
    assert torch.equal(pack[:nt], tokens.view(-1)) and torch.equal(pack[nt:nt + rows], n_acc)
    assert pack[nt + rows].item() == 5 and pack[nt + rows + 1].item() == 32
    # a slot outside the table is skipped (verify ids read 0 for it)
    bad = slots_t.clone()
    bad[0] = n_slots + 3
    N.call("pse_step_verify_ids", last.data_ptr(), n_slots, bad.data_ptr(), drafts.data_ptr(), base.data_ptr(),
           rows, k, ids.data_ptr(), first.data_ptr(), st)
    torch.cuda.synchronize()
    assert ids[0, 0].item() == 0


def test_graph_capture_holds_off_the_collector():
    """The library's captures run with Python's cyclic collector disabled (a
    collection mid-capture can destroy dead runners' CUDA graphs, which is not
    permitted while a stream captures) and restore it afterwards, also when the
    captured program raises."""
    import gc
    import pse._native as N
    x = torch.zeros(4, device="cuda")
    g = torch.cuda.CUDAGraph()
    assert gc.isenabled()
    with N.graph_capture(g):
        assert not gc.isenabled()
        x.add_(1)
    assert gc.isenabled()
    g.replay()
    torch.cuda.synchronize()
    assert x.tolist() == [1.0] * 4
    g2 = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError):
        with N.graph_capture(g2):
            x.add_(1)
            raise RuntimeError("program failed")
    assert gc.isenabled()
