"""Plain continuous batching through the paged cache, no speculation
(engine/benchmark.py:41-84, ``run_plain_continuous_batches``): one model, one
greedy token per active request per step.  The reference's own benchmark
measures speculation against this loop; here it runs on the same device
kernels (batched prefill, a CUDA-graph-replayed width-1 step: embed, paged
attention, projections, argmax), so the comparison isolates speculation.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _native as N
from .device_model import device_model
from .engine import Scratch, forward
from .scheduler import RequestResult
from .speculative import next_logits_buffer, prefill_many


class _DecodeBuffers:
    def __init__(self, B: int, V: int, device):
        i32 = dict(dtype=torch.int32, device=device)
        self.B = B
        self.dev_in = torch.zeros(B, **i32)  # slots
        self.slots = self.dev_in
        self.ids = torch.empty(B, **i32)
        self.base = torch.empty(B, **i32)
        self.logits = torch.empty(B, V, dtype=torch.float32, device=device)
        self.tok = torch.empty(B, **i32)
        self.pack = torch.empty(B + 1, **i32)
        self.host_in = torch.empty(B, dtype=torch.int32, pin_memory=True)
        self.host_pack = torch.empty(B + 1, dtype=torch.int32, pin_memory=True)
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

    def _ctx_bound(self) -> int:
        c = self.cache
        bound = c.max_blocks * c.block_size
        if self.dm.pos_emb is not None:
            bound = min(bound, self.dm.max_seq_len)
        return bound

    def _program(self, b: _DecodeBuffers, max_ctx: int) -> None:
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

    def step(self, request_ids, use_graph: bool = True) -> list[int]:
        c, dm = self.cache, self.dm
        B = len(request_ids)
        slots_np = c.slots_np(request_ids)
        lens = c.lengths_np(slots_np)
        longest = int(lens.max()) + 1
        if dm.pos_emb is not None and longest > dm.max_seq_len:
            raise IndexError(f"position {longest - 1} beyond max_seq_len {dm.max_seq_len}")
        c.ensure_capacity_len(longest)
        b = self.bufs.get(B)
        if b is None:
            b = self.bufs[B] = _DecodeBuffers(B, dm.vocab, self.device)
        b.host_in_np[:] = slots_np
        b.dev_in.copy_(b.host_in, non_blocking=True)
        max_ctx = self._ctx_bound()
        if use_graph:
            self.sc.ensure(B)
            self.sc.ensure_ws(N.size_call("pse_paged_attention_workspace", B, 1, dm.q_heads, dm.kv_heads,
                                          dm.head_dim, max_ctx))
        key = (B, c.generation, self.sc.generation, self.pending.data_ptr())
        if use_graph and key in self.graphs:
            self.graphs[key].replay()
        elif use_graph and key in self.warm:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._program(b, max_ctx)
            self.graphs[key] = g
            g.replay()
        else:
            self._program(b, max_ctx)
            if use_graph:
                self.warm.add(key)
        b.host_pack.copy_(b.pack, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        if int(b.host_pack_np[B]):
            c.check_status("decode step")
        c.note_lengths_slots(slots_np, lens + 1)
        return b.host_pack_np[:B].tolist()


def decode_runner_for(model, cache) -> DecodeRunner:
    runners = cache.__dict__.setdefault("_decode_runners", {})
    dm = device_model(model, cache.dtype, cache.device)
    r = runners.get(id(dm))
    if r is None or r.dm is not dm:
        r = runners[id(dm)] = DecodeRunner(model, cache)
    return r


@torch.no_grad()
def run_plain_continuous_batches(model, requests, cache, max_batch_size, *, use_graph=True) -> list:
    """engine/benchmark.py:41-84: FIFO admission up to ``max_batch_size`` (the
    admitted prompts prefilled together, the cache left as one-by-one prefills
    would leave it); the first token of a request is the argmax of its prompt's
    last logits; then one batched greedy token per active request per step;
    a request finishes once it has ``max_new_tokens`` generated tokens and its
    blocks are freed; backfill immediately."""
    runner = decode_runner_for(model, cache)
    dm = runner.dm
    queue = list(requests)
    active: dict[str, dict] = {}
    results: list[RequestResult] = []
    t_start = time.perf_counter()
    st = N.stream_ptr()

    def admit() -> None:
        take = []
        while queue and len(active) + len(take) < max_batch_size:
            take.append(queue.pop(0))
        if not take:
            return
        ids = [q.request_id for q in take]
        prompts = [q.prompt_ids for q in take]
        if prefill_many([(model, cache)], ids, prompts) is None:
            # one by one, as the reference admits (raises where it raises)
            from .batched_forward import batched_forward_append
            for q in take:
                cache.create_request(q.request_id)
                lg = batched_forward_append(model, cache, [q.request_id], torch.tensor([q.prompt_ids]))
                next_logits_buffer(cache, dm.vocab)[cache.slot(q.request_id)].copy_(lg[0, -1])
        buf = next_logits_buffer(cache, dm.vocab)
        slots = torch.tensor([cache.slot(r) for r in ids], dtype=torch.int32).to(cache.device)
        first = torch.empty(len(ids), dtype=torch.int32, device=cache.device)
        N.call("pse_sample_tokens", buf.data_ptr(), dm.vocab, slots.data_ptr(), len(ids), dm.vocab, 0.0, None, 0, 0,
               first.data_ptr(), 1, None, 0, st)
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
