"""engine/batched_forward.py:27-72 on the device: one uniform-width forward
over the rows' paged state, appending the W new K/V columns of every row.

The reference gathers every row's blocks into a padded tensor and runs a
masked dense attention; here the attention kernel reads the blocks in place
through the device block table, so nothing is gathered or padded."""
from __future__ import annotations

import torch

from .device_model import device_model
from .engine import forward
from .speculative import _check_ids, _check_positions


@torch.no_grad()
def batched_forward_append(model, cache, request_ids, new_input_ids: torch.Tensor) -> torch.Tensor:
    """new_input_ids: [B, W] token ids (any device).  Returns fp32 logits
    [B, W, vocab] on the cache's device and appends the W new positions of
    every row to ``cache`` (rows' blocks allocated in call order)."""
    request_ids = list(request_ids)
    if len(set(request_ids)) != len(request_ids):
        raise ValueError("request_ids must be unique")
    dm = device_model(model, cache.dtype, cache.device)
    cache._flush_ids(request_ids)  # a deferred target call owed to these rows runs first
    B, W = int(new_input_ids.shape[0]), int(new_input_ids.shape[1])
    ids_host = new_input_ids.reshape(-1)
    if ids_host.device.type == "cpu":
        _check_ids(ids_host.tolist(), dm.vocab)
    longest = _check_positions(dm, cache, request_ids, W)
    cache.ensure_capacity(request_ids, W)
    ids = ids_host.to(device=cache.device, dtype=torch.int32)
    slots = cache.slots_tensor(request_ids)
    base = torch.empty(B, dtype=torch.int32, device=cache.device)
    logits = torch.empty(B * W, dm.vocab, dtype=torch.float32, device=cache.device)
    forward(dm, cache, slots, ids, B, W, base, max(longest, 1), logits)
    cache.note_append(request_ids, W)
    cache.note_last_tokens(slots, ids, B, W)
    cache.check_status("batched_forward_append")
    return logits.view(B, W, dm.vocab)
