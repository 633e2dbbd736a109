"""Continuous-batching speculative scheduler (engine/scheduler.py:32-128),
driving the device engine.

The loop is the reference's: FIFO admission while fewer than
``max_batch_size`` requests are active, one batched speculative step over
every active request, finish once a request has ``generated >=
max_new_tokens`` (overshoot trimmed), free both caches, backfill immediately.
Admitted requests are prefilled together (``prefill_requests``), leaving the
caches as one-by-one prefills would.

Unless a caller observes every step (``on_step``), the per-row bookkeeping
also runs on the device: each step's accepted tokens are appended to a device
output arena, counted and tested against ``max_new_tokens`` by a kernel inside
the step's graph (``pse_sched_commit``), and the host reads back only the
accepted counts and the finished rows.  Host work per step is then
independent of the number of active rows except for a few array operations.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from numbers import Integral

import numpy as np
import torch

from .speculative import _fnv1a, batched_speculative_step, prefill_requests, runner_for, CommitArena
from .tree import batched_tree_speculative_step, tree_uniform_count


@dataclass
class Request:
    request_id: str
    prompt_ids: list
    max_new_tokens: int


@dataclass
class RequestResult:
    request_id: str
    output_ids: list
    submitted_at: float
    completed_at: float

    @property
    def latency_s(self) -> float:
        return self.completed_at - self.submitted_at


@dataclass
class _Active:
    request: Request
    tokens: list
    draft_next_logits: torch.Tensor
    target_next_logits: torch.Tensor
    generated: int = 0
    submitted_at: float = field(default_factory=time.perf_counter)


@torch.no_grad()
def run_continuous_speculative_batches(draft_model, target_model, requests, draft_cache, target_cache,
                                       max_batch_size, k=4, temperature=0.0, generator=None, *,
                                       uniform_fn=None, on_step=None, use_graph=None, defer_bonus=None,
                                       device_bookkeeping=None, tree_branches=None):
    """engine/scheduler.py:61-128.  ``uniform_fn(request_ids, steps, n)`` (optional)
    supplies explicit uniforms per step; ``on_step(ids, result)`` observes steps;
    ``defer_bonus`` (default: on) defers the target's bonus call into the next
    verify (see ``batched_speculative_step``; False runs it in every step); ``device_bookkeeping`` (default: whenever
    ``on_step`` is not given) keeps the per-row token lists and finish tests
    on the device, False runs them on the host as the reference does.
    ``tree_branches`` (optional) runs token-tree steps of that many branches
    (``pse.tree``; the per-row bookkeeping then runs on the host)."""
    requests = list(requests)
    if device_bookkeeping and on_step is not None:
        raise ValueError("on_step needs every step's result on the host: device_bookkeeping must be off")
    if tree_branches is not None:
        if device_bookkeeping:
            raise ValueError("token-tree steps keep the per-row bookkeeping on the host")
        device_bookkeeping = False
    if (device_bookkeeping is None or device_bookkeeping) and on_step is None and \
            all(isinstance(q.max_new_tokens, Integral) and q.max_new_tokens >= 0 for q in requests):
        return _run_device_bookkeeping(draft_model, target_model, requests, draft_cache, target_cache,
                                       max_batch_size, k, temperature, generator, uniform_fn, use_graph, defer_bonus)
    queue = list(requests)
    active: dict[str, _Active] = {}
    steps_taken: dict[str, int] = {}
    results: list[RequestResult] = []
    t_start = time.perf_counter()

    def admit() -> None:
        # FIFO admission up to the batch size (engine/scheduler.py:78-90); the
        # admitted requests are prefilled together, leaving the caches as
        # one-by-one prefills would
        take = []
        while queue and len(active) + len(take) < max_batch_size:
            take.append(queue.pop(0))
        if not take:
            return
        out = prefill_requests(draft_model, target_model, draft_cache, target_cache,
                               [q.request_id for q in take], [q.prompt_ids for q in take])
        for req in take:
            dn, tn = out[req.request_id]
            active[req.request_id] = _Active(req, list(req.prompt_ids), dn, tn, submitted_at=t_start)
            steps_taken[req.request_id] = 0

    admit()
    while active or queue:
        if not active:
            admit()
            continue
        ids = list(active.keys())
        u = None
        if uniform_fn is not None and temperature > 0:
            n_u = 2 * k + 1 if tree_branches is None else tree_uniform_count(k, tree_branches)
            u = uniform_fn(ids, [steps_taken[r] for r in ids], n_u)
        if tree_branches is not None:
            step = batched_tree_speculative_step(
                draft_model, target_model, ids, draft_cache, target_cache,
                {r: active[r].draft_next_logits for r in ids}, {r: active[r].target_next_logits for r in ids},
                k, tree_branches, temperature, generator, uniforms=u)
        else:
            step = batched_speculative_step(
                draft_model, target_model, ids, draft_cache, target_cache,
                {r: active[r].draft_next_logits for r in ids}, {r: active[r].target_next_logits for r in ids},
                k, temperature, generator, uniforms=u, use_graph=use_graph, defer_bonus=defer_bonus,
            )
        if on_step is not None:
            on_step(ids, step)
        finished = []
        for r in ids:
            a = active[r]
            a.tokens.extend(step.accepted_tokens[r])
            a.generated += len(step.accepted_tokens[r])
            steps_taken[r] += 1
            a.draft_next_logits = step.draft_next_logits[r]
            a.target_next_logits = step.target_next_logits[r]
            if a.generated >= a.request.max_new_tokens:
                finished.append(r)
        now = time.perf_counter()
        for r in finished:
            a = active.pop(r)
            over = a.generated - a.request.max_new_tokens
            out = a.tokens[: len(a.tokens) - over] if over > 0 else a.tokens
            results.append(RequestResult(r, out, a.submitted_at, now))
            draft_cache.free_request(r)
            target_cache.free_request(r)
        admit()
    return results


def _run_device_bookkeeping(draft_model, target_model, requests, draft_cache, target_cache, max_batch_size, k,
                            temperature, generator, uniform_fn, use_graph, defer_bonus) -> list:
    """The loop above with engine/scheduler.py:107-126 on the device: request
    ordinal o (its index in ``requests``) owns ``max_new_tokens`` entries of the
    runner's commit arena; the host keeps the active rows as arrays (slots in
    both caches, ordinals) in ``active`` order, which is the reference's dict
    order (finished rows leave, admitted ones join at the end)."""
    runner = runner_for(draft_model, target_model, draft_cache, target_cache, k)
    n = len(requests)
    max_new = np.array([q.max_new_tokens for q in requests], dtype=np.int64)
    if runner.commit is None:
        runner.commit = CommitArena(runner.device)
    arena = runner.commit
    arena.reset(max_new)
    T = float(temperature)
    philox = T > 0 and uniform_fn is None and generator is None
    key_by_ord = np.zeros(n, dtype=np.int32)
    steps_by_ord = np.zeros(n, dtype=np.int32)  # the runner's per-request step count (Philox key)
    taken_by_ord = np.zeros(n, dtype=np.int32)  # steps taken in this run (uniform_fn's argument)
    queue = deque(range(n))
    ids: list = []
    ords = np.zeros(0, dtype=np.int32)
    sd = np.zeros(0, dtype=np.int32)
    st = np.zeros(0, dtype=np.int32)
    finished_at: list = []  # (ordinal, completion time) in completion order
    t_start = time.perf_counter()

    def admit() -> None:
        nonlocal ords, sd, st
        take = []
        while queue and len(ids) + len(take) < max_batch_size:
            take.append(queue.popleft())
        if not take:
            return
        new_ids = [requests[o].request_id for o in take]
        prefill_requests(draft_model, target_model, draft_cache, target_cache, new_ids,
                         [requests[o].prompt_ids for o in take])
        ids.extend(new_ids)
        t_ords = np.array(take, dtype=np.int32)
        ords = np.concatenate([ords, t_ords])
        sd = np.concatenate([sd, draft_cache.slots_np(new_ids)])
        st = np.concatenate([st, target_cache.slots_np(new_ids)])
        steps_by_ord[t_ords] = [runner.request_steps.get(r, 0) for r in new_ids]
        if philox:
            key_by_ord[t_ords] = np.array([_fnv1a(r) for r in new_ids], dtype=np.uint32).view(np.int32)

    try:
        admit()
        while ids or queue:
            if not ids:
                admit()
                continue
            u = None
            if uniform_fn is not None and T > 0:
                u = uniform_fn(list(ids), taken_by_ord[ords].tolist(), 2 * k + 1)
            _, fin = runner.step_rows(ids, sd, st, ords, arena, T, generator, u, use_graph, defer_bonus,
                                      key_by_ord[ords] if philox else None, steps_by_ord[ords] if philox else None)
            steps_by_ord[ords] += 1
            taken_by_ord[ords] += 1
            if len(fin):
                now = time.perf_counter()
                fin_ids = [ids[i] for i in fin.tolist()]
                for o, r in zip(ords[fin].tolist(), fin_ids):
                    finished_at.append((o, now))
                    runner.request_steps[r] = int(steps_by_ord[o])
                draft_cache.free_requests(fin_ids)
                target_cache.free_requests(fin_ids)
                keep = np.ones(len(ids), dtype=bool)
                keep[fin] = False
                ids[:] = [r for r, kp in zip(ids, keep.tolist()) if kp]
                ords, sd, st = ords[keep], sd[keep], st[keep]
            admit()
    finally:
        # requests still active (an exception ended the run) keep their step counts
        for r, o in zip(ids, ords.tolist()):
            runner.request_steps[r] = int(steps_by_ord[o])
    out = arena.out[: int(max_new.sum())].cpu().numpy() if n else np.zeros(0, dtype=np.int32)
    off = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(max_new, out=off[1:])
    results = []
    for o, t_done in finished_at:
        q = requests[o]
        results.append(RequestResult(q.request_id, list(q.prompt_ids) + out[off[o]:off[o + 1]].tolist(),
                                     t_start, t_done))
    return results
