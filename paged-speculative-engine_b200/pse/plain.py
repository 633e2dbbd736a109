"""Plain continuous batching through the paged cache, no speculation
(engine/benchmark.py:41-84, ``run_plain_continuous_batches``): one model, one
greedy token per active request per step.  The reference's own benchmark
measures speculation against this loop; here it runs on the same device
kernels (batched prefill, a CUDA-graph-replayed width-1 step: embed, paged
attention, projections, argmax), so the comparison isolates speculation.
"""
from __future__ import annotations

import time
from collections import deque
from numbers import Integral

import numpy as np
import torch

from . import _native as N
from .device_model import device_model
from .engine import Scratch, forward
from .scheduler import RequestResult
from .speculative import CommitArena, next_logits_buffer, prefill_many


class _DecodeBuffers:
    def __init__(self, B: int, V: int, device):
        i32 = dict(dtype=torch.int32, device=device)
        self.B = B
        self.dev_in = torch.zeros(2 * B, **i32)  # [slots | ords] (ords: request ordinals in the output arena)
        self.slots, self.ords = self.dev_in.view(2, B)
        self.ids = torch.empty(B, **i32)
        self.base = torch.empty(B, **i32)
        self.logits = torch.empty(B, V, dtype=torch.float32, device=device)
        self.tok = torch.empty(B, **i32)
        self.zeros = torch.zeros(B, **i32)  # one token per row and step (accepted drafts: none)
        # [tokens B | status | finished count | finished rows B]
        self.pack = torch.empty(2 * B + 2, **i32)
        self.host_in = torch.empty(2 * B, dtype=torch.int32, pin_memory=True)
        self.host_pack = torch.empty(2 * B + 2, dtype=torch.int32, pin_memory=True)
        self.host_in_np = self.host_in.numpy()
        self.host_pack_np = self.host_pack.numpy()


class DecodeRunner:
    """The device program of one plain decode step for a (model, cache): the
    token each row holds pending (its last generated one, not yet in the
    cache) is appended and the argmax of the resulting logits becomes the row's
    next pending token.  First call per batch size runs eagerly, the second
    captures a CUDA graph, later calls replay it."""

    def __init__(self, model, cache):
        self.dm = device_model(model, cache.dtype, cache.device)
        self.cache = cache
        self.device = cache.device
        self.sc = Scratch(self.dm)
        self.bufs: dict[int, _DecodeBuffers] = {}
        self.graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.warm: set = set()
        self.pending = torch.zeros(cache.state.num_slots, dtype=torch.int32, device=cache.device)
        self.commit: CommitArena | None = None  # output arena of the device-bookkeeping loop

    def _ctx_bound(self) -> int:
        c = self.cache
        bound = c.max_blocks * c.block_size
        if self.dm.pos_emb is not None:
            bound = min(bound, self.dm.max_seq_len)
        return bound

    def _program(self, b: _DecodeBuffers, max_ctx: int, commit=None) -> None:
        dm, c, B, V = self.dm, self.cache, b.B, self.dm.vocab
        st = N.stream_ptr()
        sl = b.slots.long()
        torch.index_select(self.pending, 0, sl, out=b.ids)
        forward(dm, c, b.slots, b.ids, B, 1, b.base, max_ctx, b.logits, scratch=self.sc)
        N.call("pse_sample_tokens", b.logits.data_ptr(), V, None, B, V, 0.0, None, 0, 0, b.tok.data_ptr(), 1,
               None, 0, st)
        self.pending.index_copy_(0, sl, b.tok)
        c.last_token.index_copy_(0, sl, b.ids)
        b.pack[:B].copy_(b.tok)
        b.pack[B:B + 1].copy_(c.status_tensor())
        if commit is not None:
            # engine/benchmark.py:66-75 on the device: append, count, finish
            N.call("pse_sched_commit", b.tok.data_ptr(), 1, b.zeros.data_ptr(), b.ords.data_ptr(), B,
                   commit.off.data_ptr(), commit.max_new.data_ptr(), commit.generated.data_ptr(),
                   commit.out.data_ptr(), b.pack.data_ptr() + 4 * (B + 1), st)

    def set_pending(self, request_ids, tokens: torch.Tensor) -> None:
        """Device int32 tokens, one per request: each request's next input."""
        if self.pending.shape[0] < self.cache.state.num_slots:
            new = torch.zeros(self.cache.state.num_slots, dtype=torch.int32, device=self.device)
            new[: self.pending.shape[0]] = self.pending
            self.pending = new
            self.graphs.clear()
            self.warm.clear()
        slots = torch.tensor([self.cache.slot(r) for r in request_ids], dtype=torch.long).to(self.device)
        self.pending.index_copy_(0, slots, tokens.to(torch.int32))

    def step(self, request_ids, use_graph: bool = True, slots_np=None, ords_np=None, commit=None):
        """One greedy token per row.  Returns the tokens (a list), or with
        ``commit`` (an output arena; row i extends request ordinal
        ``ords_np[i]``) the finished rows in row order."""
        c, dm = self.cache, self.dm
        B = len(request_ids)
        if slots_np is None:
            slots_np = c.slots_np(request_ids)
        lens = c.lengths_np(slots_np)
        longest = int(lens.max()) + 1
        if dm.pos_emb is not None and longest > dm.max_seq_len:
            raise IndexError(f"position {longest - 1} beyond max_seq_len {dm.max_seq_len}")
        c.ensure_capacity_len(longest)
        b = self.bufs.get(B)
        if b is None:
            b = self.bufs[B] = _DecodeBuffers(B, dm.vocab, self.device)
        b.host_in_np[:B] = slots_np
        if ords_np is not None:
            b.host_in_np[B:] = ords_np
        b.dev_in.copy_(b.host_in, non_blocking=True)
        max_ctx = self._ctx_bound()
        if use_graph:
            self.sc.ensure(B)
            self.sc.ensure_ws(N.size_call("pse_paged_attention_workspace", B, 1, dm.q_heads, dm.kv_heads,
                                          dm.head_dim, max_ctx))
        key = (B, c.generation, self.sc.generation, self.pending.data_ptr(),
               None if commit is None else (id(commit), commit.generation))
        if use_graph and key in self.graphs:
            self.graphs[key].replay()
        elif use_graph and key in self.warm:
            g = torch.cuda.CUDAGraph()
            with N.graph_capture(g):
                self._program(b, max_ctx, commit)
            self.graphs[key] = g
            g.replay()
        else:
            self._program(b, max_ctx, commit)
            if use_graph:
                self.warm.add(key)
        if commit is None:
            b.host_pack[:B + 1].copy_(b.pack[:B + 1], non_blocking=True)
        else:  # the tokens stay on the device
            b.host_pack[B:].copy_(b.pack[B:], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        hp = b.host_pack_np
        if int(hp[B]):
            c.check_status("decode step")
        c.note_lengths_slots(slots_np, lens + 1)
        if commit is None:
            return hp[:B].tolist()
        return hp[B + 2:B + 2 + int(hp[B + 1])].copy()


def decode_runner_for(model, cache) -> DecodeRunner:
    runners = cache.__dict__.setdefault("_decode_runners", {})
    dm = device_model(model, cache.dtype, cache.device)
    r = runners.get(id(dm))
    if r is None or r.dm is not dm:
        r = runners[id(dm)] = DecodeRunner(model, cache)
    return r


def _prefill_admitted(model, cache, dm, ids, prompts) -> None:
    """Prompts of the admitted requests into the cache, each request's next
    logits into its slot's row (together, or one by one where the reference
    would raise part-way)."""
    if prefill_many([(model, cache)], ids, prompts) is None:
        from .batched_forward import batched_forward_append
        for r, p in zip(ids, prompts):
            cache.create_request(r)
            lg = batched_forward_append(model, cache, [r], torch.tensor([p]))
            next_logits_buffer(cache, dm.vocab)[cache.slot(r)].copy_(lg[0, -1])


def _first_tokens(cache, dm, ids) -> torch.Tensor:
    """Argmax of each admitted request's prompt logits (device int32)."""
    buf = next_logits_buffer(cache, dm.vocab)
    slots = torch.tensor([cache.slot(r) for r in ids], dtype=torch.int32).to(cache.device)
    first = torch.empty(len(ids), dtype=torch.int32, device=cache.device)
    N.call("pse_sample_tokens", buf.data_ptr(), dm.vocab, slots.data_ptr(), len(ids), dm.vocab, 0.0, None, 0, 0,
           first.data_ptr(), 1, None, 0, N.stream_ptr())
    return first


def _run_plain_device(model, requests, cache, max_batch_size, use_graph) -> list:
    """The loop below with engine/benchmark.py:66-75 on the device: request
    ordinal o owns max(max_new_tokens, 2) entries of the runner's output arena
    (the reference's first step always runs, so a request gets at least two
    tokens); the first token is written at admission, every step's token by
    pse_sched_commit inside the step's graph, and the host reads back only the
    finished rows."""
    runner = decode_runner_for(model, cache)
    dm = runner.dm
    n = len(requests)
    budget = np.array([max(int(q.max_new_tokens), 2) for q in requests], dtype=np.int64)
    if runner.commit is None:
        runner.commit = CommitArena(cache.device)
    arena = runner.commit
    arena.reset(budget)
    queue = deque(range(n))
    ids: list = []
    ords = np.zeros(0, dtype=np.int32)
    slots = np.zeros(0, dtype=np.int32)
    finished_at: list = []
    t_start = time.perf_counter()

    def admit() -> None:
        nonlocal ords, slots
        take = []
        while queue and len(ids) + len(take) < max_batch_size:
            take.append(queue.popleft())
        if not take:
            return
        new_ids = [requests[o].request_id for o in take]
        _prefill_admitted(model, cache, dm, new_ids, [requests[o].prompt_ids for o in take])
        first = _first_tokens(cache, dm, new_ids)
        runner.set_pending(new_ids, first)
        t_ords = torch.tensor(take, dtype=torch.long).to(cache.device)
        arena.out.index_copy_(0, arena.off.index_select(0, t_ords), first)
        arena.generated.index_fill_(0, t_ords, 1)
        ids.extend(new_ids)
        ords = np.concatenate([ords, np.array(take, dtype=np.int32)])
        slots = np.concatenate([slots, cache.slots_np(new_ids)])

    admit()
    while ids or queue:
        if not ids:
            admit()
            continue
        fin = runner.step(ids, use_graph=use_graph, slots_np=slots, ords_np=ords, commit=arena)
        if len(fin):
            now = time.perf_counter()
            fin_ids = [ids[i] for i in fin.tolist()]
            finished_at.extend((o, now) for o in ords[fin].tolist())
            cache.free_requests(fin_ids)
            keep = np.ones(len(ids), dtype=bool)
            keep[fin] = False
            ids[:] = [r for r, kp in zip(ids, keep.tolist()) if kp]
            ords, slots = ords[keep], slots[keep]
        admit()
    off = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(budget, out=off[1:])
    out = arena.out[: int(off[n])].cpu().numpy() if n else np.zeros(0, dtype=np.int32)
    return [RequestResult(requests[o].request_id, list(requests[o].prompt_ids) + out[off[o]:off[o + 1]].tolist(),
                          t_start, t_done) for o, t_done in finished_at]


@torch.no_grad()
def run_plain_continuous_batches(model, requests, cache, max_batch_size, *, use_graph=True,
                                 device_bookkeeping=None) -> list:
    """engine/benchmark.py:41-84: FIFO admission up to ``max_batch_size`` (the
    admitted prompts prefilled together, the cache left as one-by-one prefills
    would leave it); the first token of a request is the argmax of its prompt's
    last logits; then one batched greedy token per active request per step;
    a request finishes once it has ``max_new_tokens`` generated tokens and its
    blocks are freed; backfill immediately.  The per-row bookkeeping runs on the
    device unless ``device_bookkeeping=False``."""
    requests = list(requests)
    if (device_bookkeeping is None or device_bookkeeping) and \
            all(isinstance(q.max_new_tokens, Integral) for q in requests):
        return _run_plain_device(model, requests, cache, max_batch_size, use_graph)
    runner = decode_runner_for(model, cache)
    dm = runner.dm
    queue = list(requests)
    active: dict[str, dict] = {}
    results: list[RequestResult] = []
    t_start = time.perf_counter()

    def admit() -> None:
        take = []
        while queue and len(active) + len(take) < max_batch_size:
            take.append(queue.pop(0))
        if not take:
            return
        ids = [q.request_id for q in take]
        _prefill_admitted(model, cache, dm, ids, [q.prompt_ids for q in take])
        first = _first_tokens(cache, dm, ids)
        runner.set_pending(ids, first)
        for q, tok in zip(take, first.tolist()):
            active[q.request_id] = {"req": q, "tokens": [*q.prompt_ids, tok], "generated": 1}

    admit()
    while active or queue:
        if not active:
            admit()
            continue
        ids = list(active.keys())
        toks = runner.step(ids, use_graph=use_graph)
        finished = []
        for rid, tok in zip(ids, toks):
            a = active[rid]
            a["tokens"].append(tok)
            a["generated"] += 1
            if a["generated"] >= a["req"].max_new_tokens:
                finished.append(rid)
        t_now = time.perf_counter()
        for rid in finished:
            a = active.pop(rid)
            results.append(RequestResult(rid, a["tokens"], t_start, t_now))
            cache.free_request(rid)
        admit()
    return results
