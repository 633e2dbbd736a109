"""Tree speculation: the CPU statement of the rule the CUDA path implements.
TEST INFRASTRUCTURE ONLY (see the package docstring).

The reference lists tree-based speculative decoding ("multiple draft
continuations per step, not a single linear chain of k tokens") as future work
(README.md:210-214) and has no code for it; its linear step
(engine/speculative.py:76-177) is the b = 1 case of what is stated here.

Token tree of one step: b first-level candidates (branches), each followed by
a draft chain, k tokens per branch.  Node (j, d) is branch j's token at depth
d; node (j, 0) is candidate j.

Uniforms per row (``U = b*k + b + k`` float64): u[d*b + j] draws node (j, d)
at T > 0; u[b*k + i] tests candidate i at depth 0; u[b*k + b + d - 1] tests
depth d >= 1 of the accepted branch; u[b*k + b + k - 1] is the final draw.
With b = 1 this is the linear step's layout (draws u[0..k-1], tests
u[k..2k-1], final draw u[2k]).

Acceptance at T > 0, in the arithmetic of ``oracle.sampling`` (fp32 weights,
fp64 normalisers and residuals):

* depth 0, recursive rejection over the candidates x_1..x_b (drawn iid from
  the draft's root distribution q): P_0 = p; round i accepts x_i with
  probability min(1, P_{i-1}(x_i) / Q(x_i)) (round 1: the linear step's
  (w_p[x] Z_q) / (w_q[x] Z_p)); on rejection r_i = max(0, P_{i-1} - Q),
  R_i = sum r_i and P_i = r_i * (1 / R_i) (P_i = P_{i-1} when R_i <= 0).  Each
  round outputs a token distributed as P_{i-1} (the speculative-sampling
  lemma), so the first committed token is distributed as p.  Every candidate
  rejected: a draw from the last non-empty residual (threshold u * R_i), else
  from p.
* depth d >= 1 along the accepted branch j: the linear rule
  (engine/speculative.py:119-157) with p the target and q the draft
  distribution after node (j, d-1).
* all k accepted: the bonus token from the target after node (j, k-1).

At T = 0 the candidates are the draft's top-b (larger logit first, ties to the
lower index), the accepted branch is the first whose candidate is the
target's argmax, and the greedy linear rule runs along it.  Returns
``(tokens, n_accepted, branch)`` with ``len(tokens) == n_accepted + 1``;
branch 0 when no candidate was accepted.
"""
from __future__ import annotations

import numpy as np
import torch

from .sampling import inverse_cdf, sample_with_uniform, weights


def tree_uniform_count(k: int, b: int) -> int:
    return b * k + b + k


def top_candidates(q_root, b: int) -> list:
    """The draft's top-b tokens, larger logit first, ties to the lower index."""
    q = np.asarray(q_root, dtype=np.float32)
    return [int(x) for x in np.argsort(-q, kind="stable")[:b]]


def _linear_depth(p, q, x, u_test, T):
    """One position of the linear rule: (accepted, prob inputs) -> (accepted?, wp, zp, wq, zq)."""
    wp, zp = weights(p, T)
    wq, zq = weights(q, T)
    zp, zq = float(zp), float(zq)
    prob = min(1.0, (float(wp[x]) * zq) / (float(wq[x]) * zp)) if wq[x] > 0 else 0.0
    return u_test < prob, wp, zp, wq, zq


def tree_accept_row(p_root, q_root, chain, p_chain, q_chain, u, k: int, b: int, temperature: float):
    """One row's acceptance.  ``chain`` [b, k] node tokens; ``p_chain`` [b, k, V]
    target logits after node (j, d); ``q_chain`` [b, k-1, V] draft logits after
    node (j, d) for d < k-1 (the distribution node (j, d+1) was drawn from);
    ``u`` [U] (ignored at T = 0)."""
    chain = np.asarray(chain, dtype=np.int64)
    p_root = np.asarray(p_root, dtype=np.float32)
    if temperature <= 0:
        y = int(np.argmax(p_root))
        hit = [j for j in range(b) if int(chain[j, 0]) == y]
        if not hit:
            return [y], 0, 0
        j = hit[0]
        out = [y]
        for d in range(1, k):
            y = int(np.argmax(np.asarray(p_chain[j][d - 1], dtype=np.float32)))
            out.append(y)
            if int(chain[j, d]) != y:
                return out, d, j
        out.append(int(np.argmax(np.asarray(p_chain[j][k - 1], dtype=np.float32))))
        return out, k, j

    T = temperature
    base = b * k
    u_fin = float(u[base + b + k - 1])
    wp, zp = weights(p_root, T)
    wq, zq = weights(q_root, T)
    zp, zq = float(zp), float(zq)
    Q = wq.astype(np.float64) * (1.0 / zq)
    P = wp.astype(np.float64) * (1.0 / zp)
    last_r, last_R = None, 0.0
    chosen = -1
    for i in range(b):
        x = int(chain[i, 0])
        if i == 0:
            prob = min(1.0, (float(wp[x]) * zq) / (float(wq[x]) * zp)) if wq[x] > 0 else 0.0
        else:
            prob = min(1.0, float(P[x]) / float(Q[x])) if Q[x] > 0 else 0.0
        if u[base + i] < prob:
            chosen = i
            break
        r = np.maximum(P - Q, 0.0)
        R = float(r.sum())
        if R > 0:
            last_r, last_R = r, R
            P = r * (1.0 / R)
    if chosen < 0:
        tok = inverse_cdf(last_r, last_R, u_fin) if last_r is not None else inverse_cdf(wp, zp, u_fin)
        return [tok], 0, 0
    j = chosen
    out = [int(chain[j, 0])]
    for d in range(1, k):
        x = int(chain[j, d])
        ok, wp, zp, wq, zq = _linear_depth(p_chain[j][d - 1], q_chain[j][d - 1], x, u[base + b + d - 1], T)
        if ok:
            out.append(x)
            continue
        r = np.maximum(wp.astype(np.float64) * (1.0 / zp) - wq.astype(np.float64) * (1.0 / zq), 0.0)
        total = float(r.sum())
        out.append(inverse_cdf(wp, zp, u_fin) if total <= 0 else inverse_cdf(r, total, u_fin))
        return out, d, j
    wp, zp = weights(p_chain[j][k - 1], T)
    out.append(inverse_cdf(wp, float(zp), u_fin))
    return out, k, j


@torch.no_grad()
def _last_logits(model, ids) -> np.ndarray:
    return model(torch.tensor([ids]))[0][0, -1].float().numpy()


@torch.no_grad()
def tree_step_row(draft_model, target_model, context, k: int, b: int, temperature: float, u=None):
    """One row's whole tree step by full recomputation (no cache): candidates,
    chains, verification, acceptance.  Returns (tokens, n_accepted, branch,
    chain)."""
    T = temperature
    ctx = list(context)
    q_root = _last_logits(draft_model, ctx)
    p_root = _last_logits(target_model, ctx)
    if T <= 0:
        cands = top_candidates(q_root, b)
    else:
        cands = [sample_with_uniform(q_root, T, float(u[j])) for j in range(b)]
    chain = np.zeros((b, k), dtype=np.int64)
    p_chain = [[None] * k for _ in range(b)]
    q_chain = [[None] * max(k - 1, 0) for _ in range(b)]
    for j in range(b):
        seq = ctx + [cands[j]]
        chain[j, 0] = cands[j]
        for d in range(1, k):
            q = _last_logits(draft_model, seq)
            q_chain[j][d - 1] = q
            tok = int(np.argmax(q)) if T <= 0 else sample_with_uniform(q, T, float(u[d * b + j]))
            chain[j, d] = tok
            seq.append(tok)
        full = target_model(torch.tensor([seq]))[0][0].float().numpy()
        for d in range(k):
            p_chain[j][d] = full[len(ctx) + d]
    toks, n, br = tree_accept_row(p_root, q_root, chain, p_chain, q_chain, u, k, b, T)
    return toks, n, br, chain


@torch.no_grad()
def tree_generate(draft_model, target_model, prompt, max_new_tokens: int, k: int, b: int, temperature: float = 0.0,
                  uniforms=None):
    """Steps of ``tree_step_row`` until ``max_new_tokens`` are committed (the
    overshoot trimmed, as engine/scheduler.py:120-126 trims it); ``uniforms``
    (callable step -> [U] array) at T > 0."""
    seq = list(prompt)
    new = 0
    step = 0
    while new < max_new_tokens:
        u = None if uniforms is None else uniforms(step)
        toks, _, _, _ = tree_step_row(draft_model, target_model, seq, k, b, temperature, u)
        seq.extend(toks)
        new += len(toks)
        step += 1
    return seq[: len(prompt) + max_new_tokens]
