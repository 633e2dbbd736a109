"""CPU restatement of engine/speculative.py:35-177.

Two sampling modes:

* ``uniforms is None``: the reference's generator-driven path, consuming the
  torch generator in the reference's order (draft multinomials row by row per
  round, then per row one ``rand`` per tested position and one multinomial for
  the residual / bonus; engine/speculative.py:97-157);
* ``uniforms`` given (``[B, 2k+1]`` float64, row i for request_ids[i]): the
  explicit-uniform rule of ``oracle.accept`` -- u[i, j] draws draft j,
  u[i, k+j] tests position j, u[i, 2k] is the residual / bonus draw.  This is
  the mode the CUDA path is compared against draw for draw.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .accept import accept_row
from .batched_forward import batched_forward_append
from .sampling import greedy_token, sample_categorical, sample_with_uniform, softmax_with_temperature


@dataclass
class BatchStepResult:
    """engine/speculative.py:35-40."""
    accepted_tokens: dict
    num_draft_accepted: dict
    draft_next_logits: dict
    target_next_logits: dict


def _residual_sample(p, q, generator) -> int:
    """engine/speculative.py:43-50."""
    r = torch.clamp(p - q, min=0.0)
    total = r.sum()
    return sample_categorical(p if total <= 0 else r / total, generator)


@torch.no_grad()
def prefill_request(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids):
    """engine/speculative.py:53-73."""
    draft_cache.create_request(request_id)
    target_cache.create_request(request_id)
    prompt = torch.tensor([prompt_ids])
    d = batched_forward_append(draft_model, draft_cache, [request_id], prompt)
    t = batched_forward_append(target_model, target_cache, [request_id], prompt)
    return d[0, -1, :], t[0, -1, :]


@torch.no_grad()
def batched_speculative_step(draft_model, target_model, request_ids, draft_cache, target_cache,
                             draft_next_logits, target_next_logits, k, temperature,
                             generator=None, uniforms=None):
    """engine/speculative.py:76-177."""
    base_d = {r: draft_cache.length(r) for r in request_ids}
    base_t = {r: target_cache.length(r) for r in request_ids}
    explicit = uniforms is not None
    if explicit:
        uniforms = np.asarray(uniforms, dtype=np.float64)

    # Draft phase: k width-1 rounds (engine/speculative.py:92-113).
    pending = dict(draft_next_logits)
    drafted = {r: [] for r in request_ids}
    draft_dists = {r: [] for r in request_ids}
    for j in range(k):
        chosen = []
        for i, r in enumerate(request_ids):
            if explicit:
                tok = sample_with_uniform(pending[r].float().numpy(), temperature, uniforms[i, j])
                dist = pending[r].float()
            elif temperature > 0:
                dist = softmax_with_temperature(pending[r], temperature)
                tok = sample_categorical(dist, generator)
            else:
                tok = greedy_token(pending[r])
                dist = torch.nn.functional.one_hot(torch.tensor(tok), pending[r].shape[-1]).float()
            chosen.append(tok)
            drafted[r].append(tok)
            draft_dists[r].append(dist)
        logits = batched_forward_append(draft_model, draft_cache, request_ids, torch.tensor(chosen).view(-1, 1))
        for i, r in enumerate(request_ids):
            pending[r] = logits[i, -1, :]

    # Verify: one width-k target call (engine/speculative.py:115-117).
    verify = batched_forward_append(target_model, target_cache, request_ids,
                                    torch.tensor([drafted[r] for r in request_ids]))

    accepted, n_acc = {}, {}
    for i, r in enumerate(request_ids):
        if explicit:
            tgt = torch.cat([target_next_logits[r].float().view(1, -1), verify[i].float()], 0).numpy()
            drf = torch.stack(draft_dists[r]).numpy() if temperature > 0 else None
            toks, n = accept_row(tgt, drf, drafted[r], uniforms[i], k, temperature)
        else:
            toks, n = _reference_accept(r, i, k, temperature, target_next_logits, verify,
                                        drafted, draft_dists, generator)
        accepted[r] = toks
        n_acc[r] = n

    # Commit (engine/speculative.py:159-164).
    for r in request_ids:
        draft_cache.truncate(r, base_d[r] + n_acc[r])
        target_cache.truncate(r, base_t[r] + n_acc[r])

    # Bonus forwards (engine/speculative.py:166-177).
    final = torch.tensor([[accepted[r][-1]] for r in request_ids])
    dl = batched_forward_append(draft_model, draft_cache, request_ids, final)
    tl = batched_forward_append(target_model, target_cache, request_ids, final)
    return BatchStepResult(
        accepted, n_acc,
        {r: dl[i, -1, :] for i, r in enumerate(request_ids)},
        {r: tl[i, -1, :] for i, r in enumerate(request_ids)},
    )


def _reference_accept(r, i, k, temperature, target_next_logits, verify, drafted, draft_dists, generator):
    """engine/speculative.py:125-157, generator-driven."""
    def to_dist(row):
        return softmax_with_temperature(row, temperature) if temperature > 0 else row

    dists = [to_dist(target_next_logits[r])] + [to_dist(verify[i, j, :]) for j in range(k)]
    out = []
    if temperature > 0:
        for j in range(k):
            p, q, x = dists[j], draft_dists[r][j], drafted[r][j]
            prob = min(1.0, (p[x] / q[x]).item()) if q[x] > 0 else 0.0
            if torch.rand((), generator=generator).item() < prob:
                out.append(x)
            else:
                out.append(_residual_sample(p, q, generator))
                return out, j
        out.append(sample_categorical(dists[k], generator))
        return out, k
    for j in range(k):
        best = int(dists[j].argmax(dim=-1).item())
        out.append(best)
        if drafted[r][j] != best:
            return out, j
    out.append(int(dists[k].argmax(dim=-1).item()))
    return out, k
