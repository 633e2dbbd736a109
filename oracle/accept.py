"""Accept / reject / resample with explicit uniforms -- the per-row rule of
engine/speculative.py:119-157 (and ``_residual_sample``, :43-50) in the
arithmetic of the fused CUDA kernel (see ``oracle.sampling`` for the shared
weight / normaliser / inverse-CDF definitions).

Row layout (one speculative step, k drafted tokens):

* ``target[j]`` for j in 0..k: target logits; ``target[0]`` is the previous
  step's ``target_next`` (verifies draft 0), ``target[j]`` the verify call's
  column j-1, ``target[k]`` the bonus distribution;
* ``draft[j]`` for j in 0..k-1: the logits draft token j was sampled from;
* ``drafts[j]``: the drafted token ids;
* ``u[0..k-1]`` draft-sampling uniforms (consumed by the draft rounds),
  ``u[k+j]`` the accept test of position j, ``u[2k]`` the residual or bonus draw.

Returns ``(tokens, n_accepted)`` with ``len(tokens) == n_accepted + 1``.
"""
from __future__ import annotations

import numpy as np

from .sampling import inverse_cdf, weights


def accept_row(target, draft, drafts, u, k: int, temperature: float):
    target = np.asarray(target, dtype=np.float32)
    out: list[int] = []
    if temperature <= 0:
        # engine/speculative.py:146-155
        for j in range(k):
            best = int(np.argmax(target[j]))
            if int(drafts[j]) == best:
                out.append(best)
                continue
            out.append(best)
            return out, j
        out.append(int(np.argmax(target[k])))
        return out, k

    draft = np.asarray(draft, dtype=np.float32)
    for j in range(k):
        # engine/speculative.py:133-142
        x = int(drafts[j])
        wp, zp = weights(target[j], temperature)
        wq, zq = weights(draft[j], temperature)
        zp, zq = float(zp), float(zq)
        if wq[x] > 0:
            ratio = (float(wp[x]) * zq) / (float(wq[x]) * zp)
            prob = min(1.0, ratio)
        else:
            prob = 0.0
        if u[k + j] < prob:
            out.append(x)
            continue
        # engine/speculative.py:43-50: normalize(max(0, p - q)), or p if empty.
        r = np.maximum(wp.astype(np.float64) * (1.0 / zp) - wq.astype(np.float64) * (1.0 / zq), 0.0)
        total = float(r.sum())
        if total <= 0:
            out.append(inverse_cdf(wp, zp, u[2 * k]))
        else:
            out.append(inverse_cdf(r, total, u[2 * k]))
        return out, j
    # engine/speculative.py:143-144: all accepted -> bonus from target[k].
    wp, zp = weights(target[k], temperature)
    out.append(inverse_cdf(wp, float(zp), u[2 * k]))
    return out, k


def accept_rows(target, draft, drafts, u, k: int, temperature: float):
    """Vector form over rows: target [R, k+1, V], draft [R, k, V] (ignored at
    T == 0), drafts [R, k], u [R, 2k+1] -> tokens [R, k+1] (-1 padded), n_acc [R]."""
    rows = target.shape[0]
    tokens = np.full((rows, k + 1), -1, dtype=np.int64)
    n_acc = np.zeros(rows, dtype=np.int64)
    for i in range(rows):
        toks, n = accept_row(target[i], None if draft is None else draft[i], drafts[i],
                             None if u is None else u[i], k, temperature)
        tokens[i, : len(toks)] = toks
        n_acc[i] = n
    return tokens, n_acc


def decision_margins(target, draft, drafts, u, k: int, temperature: float):
    """Distance of each accept test ``u < min(1, p/q)`` from its threshold, for
    positions 0..n_acc of one row (how close a float rounding would have to be
    to flip the decision).  Used by the parity tests to tell a real mismatch
    from a near-tie."""
    target = np.asarray(target, dtype=np.float32)
    draft = np.asarray(draft, dtype=np.float32)
    margins = []
    for j in range(k):
        x = int(drafts[j])
        wp, zp = weights(target[j], temperature)
        wq, zq = weights(draft[j], temperature)
        prob = min(1.0, (float(wp[x]) * float(zq)) / (float(wq[x]) * float(zp))) if wq[x] > 0 else 0.0
        margins.append(abs(u[k + j] - prob))
        if not u[k + j] < prob:
            break
    return margins
