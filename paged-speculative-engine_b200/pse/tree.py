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

A step's device program (roots, draws, draft calls, verify, accept, compaction,
truncate, bonus call) is captured as a CUDA graph per batch size and replayed
from the second step of that size on; the host copies the step's inputs in
and reads one packed result back.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N
from .device_model import device_model
from .engine import Scratch, forward
from . import speculative as S
from .speculative import DEFAULT_SEED, BatchStepResult, _fnv1a, next_logits_buffer, next_logits_views


def tree_uniform_count(k: int, branches: int) -> int:
    """Uniforms one row of a tree step consumes (see ``pse_tree_accept``)."""
    return branches * k + branches + k


class _TreeBuffers:
    """Static device buffers of one batch size (the captured program's operands)."""

    def __init__(self, B: int, b: int, k: int, V: int, device):
        i32 = dict(dtype=torch.int32, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.B = B
        U = tree_uniform_count(k, b)
        self.dev_in = torch.empty(6, B, **i32)  # slots_d, slots_t, root_d, root_t, philox key, request step
        self.host_in = torch.empty(6, B, dtype=torch.int32, pin_memory=True)
        self.host_in_np = self.host_in.numpy()
        self.u = torch.empty(B, U, dtype=torch.float64, device=device)
        self.p_root = torch.empty(B, V, **f32)
        self.q_root = torch.empty(B, V, **f32)
        self.chain = torch.empty(B, b, k, **i32)
        self.dchain = torch.empty(max(k - 1, 1), B * b, V, **f32)
        self.ids_d = torch.empty(B * b, **i32)
        self.ud = torch.empty(max(k - 1, 1), B * b, dtype=torch.float64, device=device)
        self.base = torch.empty(B, **i32)
        self.nodes = torch.empty(B * b * k, **i32)
        self.vlog = torch.empty(B * b * k, V, **f32)
        self.toks = torch.empty(B, k + 1, **i32)
        self.res = torch.empty(3, B, **i32)  # n_accepted, branch, final token
        self.src = torch.empty(B, k, **i32)
        self.new_len = torch.empty(2, B, **i32)
        self.logits = torch.empty(2, B, V, **f32)
        self.pack = torch.empty(B * (k + 1) + 3 * B + 2, **i32)  # tokens, res, the two caches' status
        self.host_pack = torch.empty(B * (k + 1) + 3 * B + 2, dtype=torch.int32, pin_memory=True)
        self.host_pack_np = self.host_pack.numpy()


class TreeStepRunner:
    """The device program of one token-tree step for (draft, target, caches, k,
    branches), CUDA-graph replayed per batch size."""

    def __init__(self, dm_d, dm_t, dcache, tcache, k: int, branches: int):
        if dm_d.vocab != dm_t.vocab:
            raise ValueError("draft and target vocabularies differ")
        if k < 1 or branches < 1 or branches > 8 or branches > dm_t.vocab:
            raise ValueError("need k >= 1 and 1 <= branches <= min(8, vocab)")
        self.dm_d, self.dm_t, self.dcache, self.tcache = dm_d, dm_t, dcache, tcache
        self.k, self.b, self.V = k, branches, dm_t.vocab
        self.device = tcache.device
        self.sc_d, self.sc_t = Scratch(dm_d), Scratch(dm_t)
        self.bufs: dict = {}
        self.graphs: dict = {}
        self.warm: set = set()
        self.request_steps: dict = {}
        self.seed = DEFAULT_SEED
        self.use_graphs = S.USE_GRAPHS

    def _ctx_bound(self, cache, dm) -> int:
        bound = cache.max_blocks * cache.block_size
        return min(bound, dm.max_seq_len) if dm.pos_emb is not None else bound

    def _program(self, f: _TreeBuffers, T: float, philox: bool, mcd: int, mct: int) -> None:
        """One step on the device: every operand is a static buffer of ``f``."""
        k, b, V, B = self.k, self.b, self.V, f.B
        R = B * b
        U = tree_uniform_count(k, b)
        st = N.stream_ptr()
        dc, tc = self.dcache, self.tcache
        slots_d, slots_t, root_d, root_t = f.dev_in[0], f.dev_in[1], f.dev_in[2], f.dev_in[3]
        dbuf, tbuf = next_logits_buffer(dc, V), next_logits_buffer(tc, V)
        torch.index_select(tbuf, 0, slots_t.long(), out=f.p_root)
        torch.index_select(dbuf, 0, slots_d.long(), out=f.q_root)
        if T > 0 and philox:
            N.call("pse_philox_uniforms", self.seed, f.dev_in[4].data_ptr(), f.dev_in[5].data_ptr(), B, U,
                   f.u.data_ptr(), st)
        # candidates (node (j, 0)) and draft chains: chain[i, j, d] is node (j, d) of request i
        if T <= 0:
            f.chain[:, :, 0] = torch.topk(f.q_root, b, dim=-1, sorted=True).indices.to(torch.int32)
        else:
            for j in range(b):
                N.call("pse_sample_tokens", f.q_root.data_ptr(), V, None, B, V, T, f.u.data_ptr(), U, j,
                       f.chain.data_ptr() + 4 * j * k, b * k, None, 0, st)
            for d in range(1, k):
                f.ud[d - 1].copy_(f.u[:, d * b:(d + 1) * b].reshape(-1))
        for d in range(k):
            # depth d of every branch: one call of width b (logits row i*b + j)
            f.ids_d.copy_(f.chain[:, :, d].reshape(-1))
            forward(self.dm_d, dc, slots_d, f.ids_d, B, b, f.base, mcd, f.dchain[d] if d < k - 1 else None,
                    scratch=self.sc_d, tree=(b, d))
            if d < k - 1:
                N.call("pse_sample_tokens", f.dchain[d].data_ptr(), V, None, R, V, T,
                       f.ud[d].data_ptr() if T > 0 else None, 1, 0, f.chain.data_ptr() + 4 * (d + 1), k, None, 0,
                       st)
        # verify all b*k nodes (depth-major) in one call
        f.nodes.copy_(f.chain.permute(0, 2, 1).reshape(-1))
        forward(self.dm_t, tc, slots_t, f.nodes, B, b * k, f.base, mct, f.vlog, scratch=self.sc_t, tree=(b, 0))
        N.call("pse_tree_accept", f.p_root.data_ptr(), V, None, f.q_root.data_ptr(), V, None, f.vlog.data_ptr(),
               b * k * V, V, b * V, f.dchain.data_ptr(), b * V, V, R * V, f.chain.data_ptr(),
               f.u.data_ptr() if T > 0 else None, U, B, b, k, V, T, f.toks.data_ptr(), f.res[0].data_ptr(),
               f.res[1].data_ptr(), f.res[2].data_ptr(), st)
        # the kept branch's accepted nodes: node (j, m) at L + m*b + j moves to L + m; truncate to them
        torch.add(torch.arange(k, device=self.device, dtype=torch.int32).view(1, -1) * b, f.res[1].view(-1, 1),
                  out=f.src)
        for n, (c, slots, root) in enumerate(((dc, slots_d, root_d), (tc, slots_t, root_t))):
            for layer in range(c.n_layers):
                N.call("pse_kv_compact", c.state, c.layer(layer), slots.data_ptr(), root.data_ptr(),
                       f.src.data_ptr(), f.res[0].data_ptr(), B, k, st)
            torch.add(root, f.res[0], out=f.new_len[n])
            N.call("pse_kv_truncate", c.state, slots.data_ptr(), B, f.new_len[n].data_ptr(), None, None, st)
        # the bonus call (engine/speculative.py:166-177): the final token on both models
        fin = f.res[2]
        for n, (dm, c, slots, sc, buf) in enumerate(((self.dm_d, dc, slots_d, self.sc_d, dbuf),
                                                     (self.dm_t, tc, slots_t, self.sc_t, tbuf))):
            forward(dm, c, slots, fin, B, 1, f.base, mcd if n == 0 else mct, f.logits[n], scratch=sc)
            N.call("pse_scatter_rows", f.logits[n].data_ptr(), V, slots.data_ptr(), B, V, buf.data_ptr(), V,
                   buf.shape[0], st)
            c.last_token.index_copy_(0, slots.long(), fin)
        nt = B * (k + 1)
        f.pack[:nt].copy_(f.toks.view(-1))
        f.pack[nt:nt + 3 * B].copy_(f.res.view(-1))
        f.pack[nt + 3 * B:nt + 3 * B + 1].copy_(dc.status_tensor())
        f.pack[nt + 3 * B + 1:].copy_(tc.status_tensor())

    def step(self, request_ids, draft_next_logits, target_next_logits, temperature, generator=None,
             uniforms=None, use_graph=None) -> BatchStepResult:
        k, b, V = self.k, self.b, self.V
        ids = list(request_ids)
        B = len(ids)
        if B == 0:
            return BatchStepResult({}, {}, {}, {})
        if len(set(ids)) != B:
            raise ValueError("request_ids must be unique")
        dc, tc = self.dcache, self.tcache
        T = float(temperature)
        U = tree_uniform_count(k, b)
        # a target row whose bonus call the linear step deferred completes it first
        st_np = tc.slots_np(ids)
        if tc.pending_slots:
            tc.flush_pending(st_np.tolist())
        sd_np = dc.slots_np(ids)
        # the roots are read from the per-slot next-logits rows: logits handed
        # in from elsewhere are copied there first
        for c, given, sl in ((dc, draft_next_logits, sd_np), (tc, target_next_logits, st_np)):
            views = next_logits_views(c, V)
            for r, s in zip(ids, sl.tolist()):
                t = given[r]
                if t is not views[s] and t.data_ptr() != views[s].data_ptr():
                    views[s].copy_(t.reshape(-1), non_blocking=True)
        len_d, len_t = dc.lengths_np(sd_np).copy(), tc.lengths_np(st_np).copy()
        for dm, c, lens in ((self.dm_d, dc, len_d), (self.dm_t, tc, len_t)):
            longest = int(lens.max()) + k + 1  # node positions stop at L + k - 1, the bonus at L + k
            if dm.pos_emb is not None and longest > dm.max_seq_len:
                raise IndexError(f"position {longest - 1} beyond max_seq_len {dm.max_seq_len}")
            c.ensure_capacity_len(int(lens.max()) + b * k + 1)  # every node holds a position until compaction
        f = self.bufs.get(B)
        if f is None:
            f = self.bufs[B] = _TreeBuffers(B, b, k, V, self.device)
        hnp = f.host_in_np
        hnp[0], hnp[1], hnp[2], hnp[3] = sd_np, st_np, len_d, len_t
        philox = False
        if T > 0:
            if uniforms is not None:
                uu = torch.as_tensor(np.asarray(uniforms, dtype=np.float64) if not torch.is_tensor(uniforms)
                                     else uniforms, dtype=torch.float64)
                f.u.copy_(uu.reshape(B, U), non_blocking=True)
            elif generator is not None:
                f.u.copy_(torch.rand(B, U, generator=generator, dtype=torch.float64), non_blocking=True)
            else:
                philox = True
                hnp[4] = np.array([_fnv1a(r) for r in ids], dtype=np.uint32).view(np.int32)
                hnp[5] = [self.request_steps.get(r, 0) for r in ids]
        f.dev_in.copy_(f.host_in, non_blocking=True)
        mcd, mct = self._ctx_bound(dc, self.dm_d), self._ctx_bound(tc, self.dm_t)
        self.sc_d.ensure(B * b)
        self.sc_t.ensure(B * b * k)
        for sc, dm, mc, widths in ((self.sc_d, self.dm_d, mcd, (b, 1)), (self.sc_t, self.dm_t, mct, (b * k, 1))):
            sc.ensure_ws(max(N.size_call("pse_paged_attention_workspace", B, w, dm.q_heads, dm.kv_heads, dm.head_dim,
                                         mc) for w in widths))
        graphs = self.use_graphs if use_graph is None else use_graph
        key = (B, T, philox, dc.generation, tc.generation, self.sc_d.generation, self.sc_t.generation)
        if graphs and key in self.graphs:
            self.graphs[key].replay()
        elif graphs and key in self.warm:
            g = torch.cuda.CUDAGraph()
            with N.graph_capture(g):
                self._program(f, T, philox, mcd, mct)
            self.graphs[key] = g
            g.replay()
        else:
            self._program(f, T, philox, mcd, mct)
            if graphs:
                self.warm.add(key)
        f.host_pack.copy_(f.pack, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        hp = f.host_pack_np
        nt = B * (k + 1)
        if hp[nt + 3 * B] or hp[nt + 3 * B + 1]:
            for c in (dc, tc):
                c.check_status("tree step")
        toks = hp[:nt].reshape(B, k + 1)
        nacc = hp[nt:nt + B].astype(np.int64)
        dc.note_lengths_slots(sd_np, len_d + nacc + 1)
        tc.note_lengths_slots(st_np, len_t + nacc + 1)
        if philox:
            for r in ids:
                self.request_steps[r] = self.request_steps.get(r, 0) + 1
        dviews, tviews = next_logits_views(dc, V), next_logits_views(tc, V)
        accepted = {r: toks[i, : nacc[i] + 1].tolist() for i, r in enumerate(ids)}
        return BatchStepResult(accepted, {r: int(nacc[i]) for i, r in enumerate(ids)},
                               {r: dviews[s] for r, s in zip(ids, sd_np.tolist())},
                               {r: tviews[s] for r, s in zip(ids, st_np.tolist())})


def tree_runner_for(draft_model, target_model, draft_cache, target_cache, k: int, branches: int) -> TreeStepRunner:
    dm_d = device_model(draft_model, draft_cache.dtype, draft_cache.device)
    dm_t = device_model(target_model, target_cache.dtype, target_cache.device)
    runners = target_cache.__dict__.setdefault("_tree_runners", {})
    key = (id(draft_cache), id(dm_d), id(dm_t), k, branches)
    r = runners.get(key)
    if r is None or r.dm_d is not dm_d or r.dm_t is not dm_t or r.dcache is not draft_cache:
        r = runners[key] = TreeStepRunner(dm_d, dm_t, draft_cache, target_cache, k, branches)
    return r


@torch.no_grad()
def batched_tree_speculative_step(draft_model, target_model, request_ids, draft_cache, target_cache,
                                  draft_next_logits, target_next_logits, k: int, branches: int,
                                  temperature: float, generator=None, uniforms=None,
                                  use_graph=None) -> BatchStepResult:
    """One token-tree speculative step over ``request_ids`` (same arguments and
    result as ``batched_speculative_step``, plus ``branches``).  T > 0 draws
    from ``uniforms`` ([B, branches*k + branches + k] float64) when given,
    else from ``generator``, else from the device Philox stream keyed by
    (request id, request step).  The returned next-token logits are views of
    the caches' per-slot rows (the next step of the request overwrites them)."""
    r = tree_runner_for(draft_model, target_model, draft_cache, target_cache, int(k), int(branches))
    return r.step(request_ids, draft_next_logits, target_next_logits, temperature, generator, uniforms, use_graph)


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
