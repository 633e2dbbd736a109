"""CPU restatement of engine/scheduler.py:32-128 (FIFO admission up to
``max_batch_size``, one batched speculative step over all active rows, finish at
``generated >= max_new_tokens`` with the overshoot trimmed, free both caches,
backfill).

``uniform_fn`` (optional) selects the explicit-uniform mode: it is called each
step as ``uniform_fn(request_ids, steps, n)`` with ``steps[i]`` the number of
steps request i has already taken, and returns ``[B, n]`` uniforms.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from .speculative import batched_speculative_step, prefill_request


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
    draft_next: torch.Tensor
    target_next: torch.Tensor
    generated: int = 0
    steps: int = 0
    submitted_at: float = field(default_factory=time.perf_counter)


@torch.no_grad()
def run_continuous_speculative_batches(draft_model, target_model, requests, draft_cache, target_cache,
                                       max_batch_size, k=4, temperature=0.0, generator=None,
                                       uniform_fn=None, on_step=None):
    queue = list(requests)
    active: dict[str, _Active] = {}
    results = []
    t_start = time.perf_counter()

    def admit():
        while queue and len(active) < max_batch_size:
            req = queue.pop(0)
            d, t = prefill_request(draft_model, target_model, draft_cache, target_cache,
                                   req.request_id, req.prompt_ids)
            active[req.request_id] = _Active(req, list(req.prompt_ids), d, t, submitted_at=t_start)

    admit()
    while active or queue:
        if not active:
            admit()
            continue
        ids = list(active.keys())
        u = None
        if uniform_fn is not None:
            u = uniform_fn(ids, [active[r].steps for r in ids], 2 * k + 1)
        step = batched_speculative_step(
            draft_model, target_model, ids, draft_cache, target_cache,
            {r: active[r].draft_next for r in ids}, {r: active[r].target_next for r in ids},
            k, temperature, generator, uniforms=u,
        )
        if on_step is not None:
            on_step(ids, step)
        finished = []
        for r in ids:
            a = active[r]
            a.tokens.extend(step.accepted_tokens[r])
            a.generated += len(step.accepted_tokens[r])
            a.steps += 1
            a.draft_next = step.draft_next_logits[r]
            a.target_next = step.target_next_logits[r]
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


def commit_rows(tokens, n_acc, ords, generated, max_new, outputs):
    """engine/scheduler.py:107-126 on one step's row arrays: row i, owned by
    request ordinal ``ords[i]``, extends ``outputs[o]`` with
    ``tokens[i][:n_acc[i] + 1]`` and ``generated[o]`` by as many; rows whose
    request reaches ``generated >= max_new`` finish and their overshoot is
    trimmed from the end (:119-121).  Updates ``generated`` and ``outputs`` in
    place and returns the finished rows in row order."""
    fin = []
    for i, o in enumerate(ords):
        acc = list(tokens[i][: n_acc[i] + 1])
        outputs[o].extend(acc)
        generated[o] += len(acc)
        if generated[o] >= max_new[o]:
            fin.append(i)
    for i in fin:
        o = ords[i]
        over = generated[o] - max_new[o]
        if over > 0:
            del outputs[o][len(outputs[o]) - over:]
    return fin
