"""CPU restatement of engine/generate.py:12-75: the sequential greedy oracles
(``generate_naive`` full recompute, ``generate_cached`` contiguous KV cache)
and the single-request speculative driver."""
from __future__ import annotations

import torch

from .speculative import batched_speculative_step, prefill_request


@torch.no_grad()
def generate_naive(model, prompt_ids: torch.Tensor, max_new_tokens: int) -> list[int]:
    """engine/generate.py:12-20."""
    model.eval()
    tokens = prompt_ids.clone()
    for _ in range(max_new_tokens):
        logits, _ = model(tokens)
        tokens = torch.cat([tokens, logits[:, -1, :].argmax(dim=-1, keepdim=True)], dim=1)
    return tokens[0].tolist()


@torch.no_grad()
def generate_cached(model, prompt_ids: torch.Tensor, max_new_tokens: int) -> list[int]:
    """engine/generate.py:23-38: prompt in one forward, then width-1 greedy steps
    over a torch.cat-grown cache with position_offset = tokens so far - 1."""
    model.eval()
    tokens = prompt_ids.clone()
    logits, past = model(tokens)
    nxt = logits[:, -1, :].argmax(dim=-1, keepdim=True)
    tokens = torch.cat([tokens, nxt], dim=1)
    for _ in range(max_new_tokens - 1):
        logits, past = model(nxt, past_kv=past, position_offset=tokens.shape[1] - 1)
        nxt = logits[:, -1, :].argmax(dim=-1, keepdim=True)
        tokens = torch.cat([tokens, nxt], dim=1)
    return tokens[0].tolist()


@torch.no_grad()
def speculative_generate_batched(draft_model, target_model, draft_cache, target_cache, request_id,
                                 prompt_ids, max_new_tokens, k=4, temperature=0.0, generator=None):
    """engine/generate.py:41-75."""
    dn, tn = prefill_request(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids)
    tokens = list(prompt_ids)
    while len(tokens) - len(prompt_ids) < max_new_tokens:
        res = batched_speculative_step(draft_model, target_model, [request_id], draft_cache, target_cache,
                                       {request_id: dn}, {request_id: tn}, k, temperature, generator)
        tokens.extend(res.accepted_tokens[request_id])
        dn = res.draft_next_logits[request_id]
        tn = res.target_next_logits[request_id]
    over = (len(tokens) - len(prompt_ids)) - max_new_tokens
    return tokens[: len(tokens) - over] if over > 0 else tokens
