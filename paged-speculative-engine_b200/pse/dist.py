"""Request sharding across GPUs (one process per GPU) and the end-of-run
statistics exchange.

Rows never interact and a step touches only a row's own blocks
(engine/paged_cache.py:104-160), so the path shards by request: every rank owns
its pools, free list and request subset, and runs the unchanged scheduler loop
on it.  Requests are assigned longest-processing-time first by expected tokens
(prompt + max_new_tokens).  The only collective is one reduction of counters at
the end (sum of committed tokens, max of wall time) plus a gather of per-rank
stats; nothing crosses GPUs on the hot path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .workload import lpt_shards


def shard_requests(requests, world: int, rank: int):
    """This rank's requests, LPT-balanced on prompt + max_new_tokens, in their
    original order."""
    costs = [len(r.prompt_ids) + r.max_new_tokens for r in requests]
    mine = lpt_shards(costs, world)[rank]
    return [requests[i] for i in mine]


def reduce_stats(committed_tokens: int, seconds: float, extra: dict | None = None, device=None):
    """All ranks: (total committed tokens, max seconds, per-rank list of
    (tokens, seconds, extra)).  Works on any initialised process group (NCCL
    with ``device`` a CUDA device, gloo on CPU)."""
    if not dist.is_available() or not dist.is_initialized():
        return committed_tokens, seconds, [(committed_tokens, seconds, extra)]
    dev = torch.device("cpu") if device is None else torch.device(device)
    t = torch.tensor([float(committed_tokens)], dtype=torch.float64, device=dev)
    s = torch.tensor([float(seconds)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    dist.all_reduce(s, op=dist.ReduceOp.MAX)
    per = [None] * dist.get_world_size()
    dist.all_gather_object(per, (committed_tokens, seconds, extra))
    return int(t.item()), float(s.item()), per
