"""Continuous-batching speculative scheduler (engine/scheduler.py:32-128),
driving the device engine.

The loop is the reference's: FIFO admission while fewer than
``max_batch_size`` requests are active (each prefilled on its own), one
batched speculative step over every active request, finish once a request has
``generated >= max_new_tokens`` (overshoot trimmed), free both caches,
backfill immediately.  Only the calls underneath run on the GPU.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .speculative import batched_speculative_step, prefill_requests


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
                                       uniform_fn=None, on_step=None, use_graph=None, defer_bonus=False):
    """engine/scheduler.py:61-128.  ``uniform_fn(request_ids, steps, n)`` (optional)
    supplies explicit uniforms per step; ``on_step(ids, result)`` observes steps;
    ``defer_bonus`` folds the target's bonus call into the next verify (see
    ``batched_speculative_step``)."""
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
            u = uniform_fn(ids, [steps_taken[r] for r in ids], 2 * k + 1)
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
