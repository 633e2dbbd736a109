"""CPU restatement of engine/batched_forward.py:27-72.

Gather the rows' paged state into a right-padded contiguous tensor, run one
ordinary forward of uniform width W with per-row positions
``lengths[b] + w`` for the W new columns, and append the W new K/V columns of
every row back into its own blocks, rows in call order.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def batched_forward_append(model, cache, request_ids, new_input_ids):
    k_layers, v_layers, mask, lengths = cache.gather(request_ids)
    past = list(zip(k_layers, v_layers))
    cached = mask.shape[1]
    batch, width = new_input_ids.shape
    pad_mask = torch.cat([mask, torch.ones(batch, width, dtype=torch.bool)], dim=1)
    # Padded columns keep their raw index as position; the W new columns of row
    # b sit at lengths[b] + w (engine/batched_forward.py:44-57).
    key_pos = torch.arange(cached + width).unsqueeze(0).repeat(batch, 1)
    key_pos[:, cached:] = lengths.view(-1, 1) + torch.arange(width).view(1, -1)
    logits, new_kv = model(
        new_input_ids, past_kv=past, position_offset=lengths,
        padding_mask=pad_mask, key_positions=key_pos,
    )
    for i, rid in enumerate(request_ids):
        cache.append(
            rid,
            [new_kv[l][0][i, :, cached:cached + width, :] for l in range(cache.n_layers)],
            [new_kv[l][1][i, :, cached:cached + width, :] for l in range(cache.n_layers)],
        )
    return logits
