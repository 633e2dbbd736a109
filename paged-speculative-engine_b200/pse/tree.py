"""Tree speculation on the device engine: ``branches`` first-level candidates
per step, each followed by a draft chain of k tokens, verified in one target
call and accepted by ``pse_tree_accept``.

The reference lists tree-based speculative decoding ("multiple draft
continuations per step, not a single linear chain of k tokens") as future work
(README.md:210-214) and has no code for it; its linear step
(engine/speculative.py:76-177, ``pse.batched_speculative_step``) is the
one-branch case.  The rule (candidates, recursive rejection at depth 0, the
linear rule along the accepted branch, uniform layout) is stated in
include/pse.h at ``pse_tree_accept``.

Layout: a request's tree lives in its own row.  The nodes are appended after
the row's root length L in depth-major order (node (j, d) at position
L + d*b + j): the draft extends all b branches with one call of width b per
depth, the target verifies all b*k nodes in one call of width b*k, and every
node attends to the root context and its own branch only
(``pse_paged_attention_tree``; its position for the embeddings / RoPE is
L + d), so the context's K/V is read once per request, not once per branch.
After acceptance ``pse_kv_compact`` moves the kept branch's accepted nodes to
positions L, L+1, ... and the row is truncated to them; then the reference's
bonus call (width 1 on both models, the final token) writes the final token's
K/V and the next-token logits, as in the linear step's reference structure.

Steps run eagerly (no CUDA graph).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N
from .device_model import device_model
from .engine import Scratch, forward
from .speculative import (DEFAULT_SEED, BatchStepResult, _check_positions, _fnv1a, next_logits_buffer,
                          next_logits_views)


def tree_uniform_count(k: int, branches: int) -> int:
    """Uniforms one row of a tree step consumes (see ``pse_tree_accept``)."""
    return branches * k + branches + k


class _TreeScratch:
    """Per (draft, target) device models: forward scratch of each side."""

    def __init__(self, dm_d, dm_t):
        self.sc_d = Scratch(dm_d)
        self.sc_t = Scratch(dm_t)


def _scratch(cache, dm_d, dm_t) -> _TreeScratch:
    s = getattr(cache, "_tree_scratch", None)
    if s is None or s.sc_d.dm is not dm_d or s.sc_t.dm is not dm_t:
        s = cache._tree_scratch = _TreeScratch(dm_d, dm_t)
    return s


@torch.no_grad()
def batched_tree_speculative_step(draft_model, target_model, request_ids, draft_cache, target_cache,
                                  draft_next_logits, target_next_logits, k: int, branches: int,
                                  temperature: float, generator=None, uniforms=None) -> BatchStepResult:
    """One token-tree speculative step over ``request_ids`` (same arguments and
    result as ``batched_speculative_step``, plus ``branches``).  T > 0 draws
    from ``uniforms`` ([B, branches*k + branches + k] float64) when given,
    else from ``generator``, else from the device Philox stream keyed by
    (request id, request step)."""
    ids = list(request_ids)
    B, b = len(ids), int(branches)
    if B == 0:
        return BatchStepResult({}, {}, {}, {})
    if len(set(ids)) != B:
        raise ValueError("request_ids must be unique")
    if k < 1 or b < 1 or b > 8:
        raise ValueError("need k >= 1 and 1 <= branches <= 8")
    dc, tc = draft_cache, target_cache
    dm_d = device_model(draft_model, dc.dtype, dc.device)
    dm_t = device_model(target_model, tc.dtype, tc.device)
    V = dm_t.vocab
    if dm_d.vocab != V:
        raise ValueError("draft and target vocabularies differ")
    if b > V:
        raise ValueError("more branches than vocabulary entries")
    dev = tc.device
    st = N.stream_ptr()
    T = float(temperature)
    U = tree_uniform_count(k, b)
    # a target row whose bonus call was deferred by the linear step completes it first
    tc.flush_pending([tc.slot(r) for r in ids])
    p_root = torch.stack([target_next_logits[r].reshape(-1) for r in ids]).float().contiguous()
    q_root = torch.stack([draft_next_logits[r].reshape(-1) for r in ids]).float().contiguous()
    for dm, c in ((dm_d, dc), (dm_t, tc)):
        _check_positions(dm, c, ids, k + 1)  # node positions stop at L + k - 1, the bonus at L + k
    u = None
    if T > 0:
        if uniforms is not None:
            u = torch.as_tensor(np.asarray(uniforms, dtype=np.float64)).reshape(B, U).to(dev)
        elif generator is not None:
            u = torch.rand(B, U, generator=generator, dtype=torch.float64).to(dev)
        else:
            steps = tc.__dict__.setdefault("_tree_steps", {})
            key = torch.from_numpy(np.array([_fnv1a(r) for r in ids], dtype=np.uint32).view(np.int32)).to(dev)
            stp = torch.from_numpy(np.array([steps.get(r, 0) for r in ids], dtype=np.int32)).to(dev)
            u = torch.empty(B, U, dtype=torch.float64, device=dev)
            N.call("pse_philox_uniforms", DEFAULT_SEED, key.data_ptr(), stp.data_ptr(), B, U, u.data_ptr(), st)
            for r in ids:
                steps[r] = steps.get(r, 0) + 1
    L_d = dc.lengths_np(dc.slots_np(ids)).copy()
    L_t = tc.lengths_np(tc.slots_np(ids)).copy()
    for c in (dc, tc):
        c.ensure_capacity(ids, b * k + 1)
    R = B * b
    sd = dc.slots_tensor(ids)
    stt = tc.slots_tensor(ids)
    sc = _scratch(tc, dm_d, dm_t)

    # ---- candidates (node (j, 0)) and draft chains: chain[i, j, d] is node (j, d) of request i
    chain = torch.empty(B, b, k, dtype=torch.int32, device=dev)
    if T <= 0:
        chain[:, :, 0] = torch.topk(q_root, b, dim=-1, sorted=True).indices.to(torch.int32)
    else:
        for j in range(b):
            N.call("pse_sample_tokens", q_root.data_ptr(), V, None, B, V, T, u.data_ptr(), U, j,
                   chain.data_ptr() + 4 * j * k, b * k, None, 0, st)
    dchain = torch.empty(max(k - 1, 1), R, V, dtype=torch.float32, device=dev)
    ids_d = torch.empty(R, dtype=torch.int32, device=dev)
    base = torch.empty(B, dtype=torch.int32, device=dev)
    for d in range(k):
        # depth d of every branch: one call of width b (logits row i*b + j)
        ids_d.copy_(chain[:, :, d].reshape(-1))
        forward(dm_d, dc, sd, ids_d, B, b, base, int(L_d.max()) + (d + 1) * b,
                dchain[d] if d < k - 1 else None, scratch=sc.sc_d, tree=(b, d))
        if d < k - 1:
            ud = None if u is None else u[:, (d + 1) * b:(d + 2) * b].reshape(-1).contiguous()
            N.call("pse_sample_tokens", dchain[d].data_ptr(), V, None, R, V, T, N.ptr(ud), 1, 0,
                   chain.data_ptr() + 4 * (d + 1), k, None, 0, st)
    # ---- verify all b*k nodes (depth-major) in one call
    nodes = chain.permute(0, 2, 1).reshape(-1).contiguous()
    vlog = torch.empty(B * b * k, V, dtype=torch.float32, device=dev)
    forward(dm_t, tc, stt, nodes, B, b * k, base, int(L_t.max()) + b * k, vlog, scratch=sc.sc_t, tree=(b, 0))
    # ---- accept
    toks = torch.empty(B, k + 1, dtype=torch.int32, device=dev)
    res = torch.empty(3, B, dtype=torch.int32, device=dev)  # n_accepted, branch, final token
    N.call("pse_tree_accept", p_root.data_ptr(), V, None, q_root.data_ptr(), V, None, vlog.data_ptr(), b * k * V, V,
           b * V, dchain.data_ptr(), b * V, V, R * V, chain.data_ptr(), N.ptr(u), U, B, b, k, V, T,
           toks.data_ptr(), res[0].data_ptr(), res[1].data_ptr(), res[2].data_ptr(), st)
    # ---- keep the accepted nodes of the kept branch: node (j, m) at L + m*b + j moves to L + m
    dj = torch.arange(k, device=dev, dtype=torch.int32).view(1, -1) * b + res[1].view(-1, 1)
    src = dj.contiguous()
    nacc_d = res[0].contiguous()
    for c, L in ((dc, L_d), (tc, L_t)):
        slots = c.slots_tensor(ids)
        root = torch.from_numpy(L.astype(np.int32)).to(dev)
        for layer in range(c.n_layers):
            N.call("pse_kv_compact", c.state, c.layer(layer), slots.data_ptr(), root.data_ptr(), src.data_ptr(),
                   nacc_d.data_ptr(), B, k, st)
        new_len = (root + nacc_d).contiguous()
        N.call("pse_kv_truncate", c.state, slots.data_ptr(), B, new_len.data_ptr(), None, None, st)
    res_h = res.cpu().numpy()
    toks_h = toks.cpu().numpy()
    nacc, fin = res_h[0].astype(np.int64), res_h[2]
    dc.note_lengths(ids, L_d + nacc)
    tc.note_lengths(ids, L_t + nacc)
    # ---- the bonus call (engine/speculative.py:166-177): the final token on both models
    fin_d = torch.from_numpy(fin.astype(np.int32)).to(dev)
    out = []
    for dm, c, s_ in ((dm_d, dc, sc.sc_d), (dm_t, tc, sc.sc_t)):
        slots = c.slots_tensor(ids)
        bb = torch.empty(B, dtype=torch.int32, device=dev)
        logits = torch.empty(B, V, dtype=torch.float32, device=dev)
        forward(dm, c, slots, fin_d, B, 1, bb, int(c.lengths_np(c.slots_np(ids)).max()) + 1, logits, scratch=s_)
        buf = next_logits_buffer(c, V)
        N.call("pse_scatter_rows", logits.data_ptr(), V, slots.data_ptr(), B, V, buf.data_ptr(), V, buf.shape[0], st)
        c.note_append(ids, 1)
        c.note_last_tokens(slots, fin_d, B, 1)
        c.check_status("tree step")
        views = next_logits_views(c, V)
        out.append({r: views[c.slot(r)] for r in ids})
    accepted = {r: toks_h[i, : nacc[i] + 1].tolist() for i, r in enumerate(ids)}
    return BatchStepResult(accepted, {r: int(nacc[i]) for i, r in enumerate(ids)}, out[0], out[1])


@torch.no_grad()
def speculative_generate_tree(draft_model, target_model, prompt_ids, max_new_tokens: int, draft_cache, target_cache,
                              k: int = 4, branches: int = 2, temperature: float = 0.0, generator=None,
                              request_id: str = "tree0") -> list:
    """One request decoded with token-tree steps until ``max_new_tokens`` are
    committed (the overshoot trimmed as engine/scheduler.py:120-126 trims it);
    the request is freed from both caches at the end.  Returns prompt + new
    tokens."""
    from .speculative import prefill_request
    dn, tn = prefill_request(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids)
    out = list(prompt_ids)
    new = 0
    try:
        while new < max_new_tokens:
            r = batched_tree_speculative_step(draft_model, target_model, [request_id], draft_cache, target_cache,
                                              {request_id: dn}, {request_id: tn}, k, branches, temperature,
                                              generator=generator)
            toks = r.accepted_tokens[request_id]
            out.extend(toks)
            new += len(toks)
            dn, tn = r.draft_next_logits[request_id], r.target_next_logits[request_id]
    finally:
        draft_cache.free_request(request_id)
        target_cache.free_request(request_id)
    return out[: len(prompt_ids) + max_new_tokens]
