"""Single-request speculative driver (engine/generate.py:41-75) over the
device engine.  The sequential greedy oracles of engine/generate.py:12-38 are
not part of the engine (they are the reference the engine is checked
against)."""
from __future__ import annotations

import torch

from .speculative import batched_speculative_step, prefill_request


@torch.no_grad()
def speculative_generate_batched(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids,
                                 max_new_tokens, k=4, temperature=0.0, generator=None, *, uniforms_fn=None):
    dn, tn = prefill_request(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids)
    tokens = list(prompt_ids)
    step = 0
    while len(tokens) - len(prompt_ids) < max_new_tokens:
        u = uniforms_fn(step) if (uniforms_fn is not None and temperature > 0) else None
        res = batched_speculative_step(draft_model, target_model, [request_id], draft_cache, target_cache,
                                       {request_id: dn}, {request_id: tn}, k, temperature, generator, uniforms=u)
        tokens.extend(res.accepted_tokens[request_id])
        dn = res.draft_next_logits[request_id]
        tn = res.target_next_logits[request_id]
        step += 1
    over = (len(tokens) - len(prompt_ids)) - max_new_tokens
    return tokens[: len(tokens) - over] if over > 0 else tokens
