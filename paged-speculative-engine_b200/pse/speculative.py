"""Batched speculative step on the device, behind the reference's API
(engine/speculative.py:35-177).

Everything between the call and its single device->host copy runs on the
GPU: k width-1 draft forwards with a sampling kernel between rounds
(speculative.py:92-113), one width-k verify forward (:115-117), the fused
accept / reject / residual / bonus kernel (:119-157), the batched truncate of
both caches (:159-164) and the two width-1 bonus forwards (:166-177).  From the
second step with a given batch size on, the whole program is replayed from a
CUDA graph.

Sampling at T > 0 uses explicit uniforms ([B, 2k+1] per step: u[j] draws draft
j, u[k+j] tests position j, u[2k] is the residual / bonus draw), taken from
``uniforms`` if given, else from ``generator`` (torch.rand on the host), else
from the device Philox stream keyed by (seed, request id, request step).

``draft_next_logits`` / ``target_next_logits`` in the result are views of
per-request device buffers that the next step of the same request overwrites;
passing them back unchanged (as the scheduler does) costs no copy.

By default the target's width-1 bonus call is deferred: the final token's
position is reserved where the reference's bonus append puts it (block
tables, lengths and free lists stay the reference's), and the next step's
verify runs at width k+1 from that position, its column 0 giving the logits
the bonus call would have returned.  The step then costs one target pass
instead of two.  The returned ``target_next_logits`` are ``PendingLogits``
(pse/pending.py): handing them back is free, reading them runs the deferred
call first.  ``defer_bonus=False`` runs the bonus call inside the step.
"""
from __future__ import annotations

import operator
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .device_model import device_model
from .engine import Scratch, forward, lm_head, scratch_for
from .pending import pending_view

DEFAULT_SEED = 0x5EED5EED
USE_GRAPHS = True  # replay steps from CUDA graphs (from the second step of a batch size on)


@dataclass
class BatchStepResult:
    """engine/speculative.py:35-40."""
    accepted_tokens: dict
    num_draft_accepted: dict
    draft_next_logits: dict
    target_next_logits: dict


def _fnv1a(s: str) -> int:
    h = 0x811C9DC5
    for b in s.encode("utf-8"):
        h = ((h ^ b) * 0x01000193) & 0xFFFFFFFF
    return h


def next_logits_buffer(cache, vocab: int) -> torch.Tensor:
    """Per-slot fp32 [num_slots, vocab] buffer holding each request's next-token
    logits (prefill and bonus outputs land here)."""
    buf = getattr(cache, "_next_logits", None)
    slots = cache.state.num_slots
    if buf is None or buf.shape[0] < slots or buf.shape[1] != vocab:
        new = torch.zeros(slots, vocab, dtype=torch.float32, device=cache.device)
        if buf is not None and buf.shape[1] == vocab:
            new[: buf.shape[0]] = buf
        cache._next_logits = new
    return cache._next_logits


def next_logits_views(cache, vocab: int) -> list:
    """One view per slot of ``next_logits_buffer`` (row s is request slot s's
    next-token logits), built once per buffer allocation: handing a request's
    row back to the caller costs a list lookup instead of a tensor index."""
    buf = next_logits_buffer(cache, vocab)
    cached = getattr(cache, "_next_views", None)
    if cached is None or cached[0] is not buf:
        cached = (buf, list(buf.unbind(0)))
        cache._next_views = cached
    return cached[1]


def pending_views(cache, vocab: int, slots: np.ndarray) -> list:
    """One ``PendingLogits`` per slot over ``next_logits_buffer`` (see
    ``next_logits_views``), bound to the slot's current occupant: entries of
    ``slots`` whose occupant changed since they were made are remade."""
    buf = next_logits_buffer(cache, vocab)
    cached = getattr(cache, "_pending_views", None)
    if cached is None or cached[0] is not buf or len(cached[2]) != buf.shape[0]:
        rows = next_logits_views(cache, vocab)
        ser = cache._serial[: buf.shape[0]].copy()
        cached = (buf, ser, [pending_view(rows[s], cache, s) for s in range(buf.shape[0])])
        cache._pending_views = cached
        return cached[2]
    _, ser, views = cached
    stale = slots[cache._serial[slots] != ser[slots]]
    if len(stale):
        rows = next_logits_views(cache, vocab)
        for s in stale.tolist():
            views[s] = pending_view(rows[s], cache, s)
            ser[s] = cache._serial[s]
    return views


@torch.no_grad()
def _flush_pending(cache, slots) -> None:
    """The target call a deferred step left owing for ``slots`` (pending slots
    of ``cache``): one width-1 forward over each row's final token at its
    reserved position (nothing allocated), writing its K/V and the slot's
    next-token logits -- the reference's bonus call (engine/speculative.py:
    170-175), run late."""
    dm = cache._pending_dm
    st_np = np.asarray(slots, dtype=np.int32)
    B = len(st_np)
    lens = cache.lengths_np(st_np)
    dev = cache.device
    slots_t = torch.from_numpy(st_np).to(dev)
    base = torch.from_numpy((lens - 1).astype(np.int32)).to(dev)
    ids = cache.last_token.index_select(0, slots_t.long())
    buf = next_logits_buffer(cache, dm.vocab)
    logits = torch.empty(B, dm.vocab, dtype=torch.float32, device=dev)
    forward(dm, cache, slots_t, ids, B, 1, base, int(lens.max()), logits, scratch=scratch_for(dm), reserve=False)
    N.call("pse_scatter_rows", logits.data_ptr(), dm.vocab, slots_t.data_ptr(), B, dm.vocab, buf.data_ptr(), dm.vocab,
           buf.shape[0], N.stream_ptr())
    cache.pending_slots.difference_update(st_np.tolist())
    cache.check_status("deferred target call")


def _check_ids(ids, vocab: int) -> None:
    if len(ids) and (min(ids) < 0 or max(ids) >= vocab):
        raise IndexError(f"token id out of range for vocabulary of {vocab}")


def _check_positions(dm, cache, request_ids, extra: int) -> int:
    longest = max((cache.length(r) for r in request_ids), default=0) + extra
    if dm.pos_emb is not None and longest > dm.max_seq_len:
        raise IndexError(f"position {longest - 1} beyond max_seq_len {dm.max_seq_len}")
    return longest


@torch.no_grad()
def prefill_request(draft_model, target_model, draft_cache, target_cache, request_id, prompt_ids):
    """engine/speculative.py:53-73: seed both caches with the prompt and
    return the two next-token logits rows (device views)."""
    if draft_cache.prefix is not None or target_cache.prefix is not None:
        out = _prefill_prefix([(draft_model, draft_cache), (target_model, target_cache)], [request_id],
                              [list(prompt_ids)])
        if out is not None:
            return out[0][0], out[1][0]
    draft_cache.create_request(request_id)
    target_cache.create_request(request_id)
    prompt_ids = list(prompt_ids)
    P = len(prompt_ids)
    outs = []
    for model, cache in ((draft_model, draft_cache), (target_model, target_cache)):
        dm = device_model(model, cache.dtype, cache.device)
        _check_ids(prompt_ids, dm.vocab)
        _check_positions(dm, cache, [request_id], P)
        cache.ensure_capacity([request_id], P)
        buf = next_logits_buffer(cache, dm.vocab)
        slot = cache.slot(request_id)
        ids = torch.tensor(prompt_ids, dtype=torch.int32).to(cache.device, non_blocking=True)
        slots = torch.tensor([slot], dtype=torch.int32).to(cache.device, non_blocking=True)
        base = torch.empty(1, dtype=torch.int32, device=cache.device)
        forward(dm, cache, slots, ids, 1, P, base, P, buf[slot:slot + 1], last_only=True)
        cache.note_append([request_id], P)
        cache.note_last_tokens(slots, ids, 1, P)
        outs.append(buf[slot])
    draft_cache.check_status("prefill")
    target_cache.check_status("prefill")
    return outs[0], outs[1]


def _batch_prefill_safe(pairs, request_ids, prompts) -> bool:
    """True when prefilling these requests one by one could not raise part-way
    (so one batched pass leaves exactly the same state).  Idle blocks of a
    prefix index count as free (they are evicted on demand)."""
    if len(set(request_ids)) != len(request_ids):
        return False
    for dm, cache in pairs:
        bs = cache.block_size
        need = 0
        for r, p in zip(request_ids, prompts):
            if r in cache._slot or not p:
                return False
            if min(p) < 0 or max(p) >= dm.vocab:
                return False
            if dm.pos_emb is not None and len(p) > dm.max_seq_len:
                return False
            need += (len(p) + bs - 1) // bs
        idle = len(cache.prefix.idle) if cache.prefix is not None else 0
        if need > cache.allocator.num_free + idle:
            return False
    return True


def _prefill_prefix(models_caches, request_ids, prompts, max_tokens_per_call: int = 32768):
    """``prefill_many`` for caches with a prefix index (``pse.prefix_cache``):
    each prompt's longest indexed prefix of full blocks (leaving at least its
    last token) is mapped into the head of its block table and only the rest
    is computed, at positions from the end of the shared prefix; the prompt's
    full blocks are then indexed.  Inside one call the first prompt of every
    distinct first block is prefilled before the others, so they find its
    blocks.  Caches without an index take every prompt whole.  Returns what
    ``prefill_many`` returns (None, having changed nothing, when one-by-one
    prefills could raise part-way)."""
    ids = list(request_ids)
    prompts = [list(p) for p in prompts]
    pairs = [(device_model(m, c.dtype, c.device), c) for m, c in models_caches]
    if not ids or not _batch_prefill_safe(pairs, ids, prompts):
        return None
    for r in ids:
        for _, cache in pairs:
            cache.create_request(r)
    n = len(ids)
    P_all = np.array([len(p) for p in prompts], dtype=np.int64)
    st = N.stream_ptr()
    for dm, cache in pairs:
        dev, bs, idx = cache.device, cache.block_size, cache.prefix
        cache.ensure_capacity_len(int(P_all.max()))
        buf = next_logits_buffer(cache, dm.vocab)
        sc = scratch_for(dm)
        for wave in (idx.waves(prompts) if idx is not None else [list(range(n))]):
            wids = [ids[i] for i in wave]
            wprom = [prompts[i] for i in wave]
            m = len(wave)
            slots_np = np.fromiter((cache.slot(r) for r in wids), np.int32, m)
            hits = [idx.lookup(p) for p in wprom] if idx is not None else [[] for _ in wave]
            shared = np.array([len(h) * bs for h in hits], dtype=np.int64)
            P = P_all[wave]
            widths = P - shared
            if idx is not None:
                need = int(sum((int(q) + bs - 1) // bs - len(h) for q, h in zip(P, hits)))
                idx.make_room(need, keep=[b for h in hits for b in h])
                idx.attach(slots_np.tolist(), hits)
            slots = torch.from_numpy(slots_np).to(dev)
            wd = torch.from_numpy(widths.astype(np.int32)).to(dev)
            base = torch.empty(m, dtype=torch.int32, device=dev)
            N.call("pse_kv_reserve_rows", cache.state, slots.data_ptr(), m, wd.data_ptr(), base.data_ptr(), st)
            order = np.argsort(-widths, kind="stable")  # groups of similar suffix length, longest first
            i0 = 0
            while i0 < m:
                W = int(widths[order[i0]])
                grp = order[i0:i0 + max(1, max_tokens_per_call // W)]
                i0 += len(grp)
                g = len(grp)
                ids_pad = np.zeros((g, W), dtype=np.int32)
                for j, q in enumerate(grp):
                    ids_pad[j, : widths[q]] = wprom[q][shared[q]:]
                gids = torch.from_numpy(ids_pad).to(dev)
                gslots = torch.from_numpy(slots_np[grp]).to(dev)
                gbase = torch.from_numpy(shared[grp].astype(np.int32)).to(dev)
                forward(dm, cache, gslots, gids.view(-1), g, W, gbase, int(shared[grp].max()) + W, None, scratch=sc,
                        reserve=False)
                last = torch.from_numpy(np.arange(g, dtype=np.int64) * W + widths[grp] - 1).to(dev)
                hsel = torch.index_select(sc.h[: g * W], 0, last)
                logits = torch.empty(g, dm.vocab, dtype=torch.float32, device=dev)
                lm_head(dm, hsel, logits)
                N.call("pse_scatter_rows", logits.data_ptr(), dm.vocab, gslots.data_ptr(), g, dm.vocab,
                       buf.data_ptr(), dm.vocab, buf.shape[0], st)
                last_tok = torch.from_numpy(np.array([wprom[q][-1] for q in grp], dtype=np.int32)).to(dev)
                cache.last_token.index_copy_(0, gslots.long(), last_tok)
            cache.note_lengths(wids, P.tolist())
            if idx is not None:
                cache.check_status("prefill")  # the blocks are indexed only once they hold their K/V
                idx.register(slots_np.tolist(), wprom)
    for _, cache in pairs:
        cache.check_status("prefill")
    out = []
    for dm, cache in pairs:
        views = next_logits_views(cache, dm.vocab)
        out.append([views[cache.slot(r)] for r in ids])
    return out


@torch.no_grad()
def prefill_many(models_caches, request_ids, prompts, max_tokens_per_call: int = 32768):
    """Batched prompt prefill of ``request_ids`` into every (model, cache) pair,
    leaving each cache as one-by-one appends of the prompts in request order
    would: requests are created in order, each cache reserves every prompt's
    blocks in one launch with rows in request order (``pse_kv_reserve_rows``),
    and the forwards run over groups of similar-length prompts padded to the
    group's longest (padding is never allocated: its K/V lands past the row's
    length in a block the row holds, or is dropped).  Returns, per pair, the
    list of the requests' next-token logits rows (device views), or None --
    having changed nothing -- when one-by-one prefills could raise part-way
    (bad ids, positions past ``max_seq_len``, a pool too small, duplicate or
    existing ids, empty prompts): the caller then takes the one-by-one path,
    which raises at the same request."""
    ids = list(request_ids)
    prompts = [list(p) for p in prompts]
    if len(ids) != len(prompts):
        raise ValueError("one prompt per request id")
    if any(c.prefix is not None for _, c in models_caches):
        return _prefill_prefix(models_caches, ids, prompts, max_tokens_per_call)
    pairs = [(device_model(m, c.dtype, c.device), c) for m, c in models_caches]
    if len(ids) <= 1 or not _batch_prefill_safe(pairs, ids, prompts):
        return None
    for r in ids:
        for _, cache in pairs:
            cache.create_request(r)
    n = len(ids)
    P = np.array([len(p) for p in prompts], dtype=np.int64)
    order = np.argsort(-P, kind="stable")  # groups of similar length, longest first
    st = N.stream_ptr()
    out = []
    for dm, cache in pairs:
        dev = cache.device
        cache.ensure_capacity_len(int(P.max()))
        slots_np = np.fromiter((cache.slot(r) for r in ids), np.int32, n)
        slots = torch.from_numpy(slots_np).to(dev)
        widths = torch.from_numpy(P.astype(np.int32)).to(dev)
        base = torch.empty(n, dtype=torch.int32, device=dev)
        N.call("pse_kv_reserve_rows", cache.state, slots.data_ptr(), n, widths.data_ptr(), base.data_ptr(), st)
        buf = next_logits_buffer(cache, dm.vocab)
        sc = scratch_for(dm)
        i0 = 0
        while i0 < n:
            W = int(P[order[i0]])
            grp = order[i0:i0 + max(1, max_tokens_per_call // W)]
            i0 += len(grp)
            g = len(grp)
            ids_pad = np.zeros((g, W), dtype=np.int32)
            for j, idx in enumerate(grp):
                ids_pad[j, : P[idx]] = prompts[idx]
            gids = torch.from_numpy(ids_pad).to(dev)
            gslots = torch.from_numpy(slots_np[grp]).to(dev)
            gbase = torch.zeros(g, dtype=torch.int32, device=dev)
            forward(dm, cache, gslots, gids.view(-1), g, W, gbase, W, None, scratch=sc, reserve=False)
            last = torch.from_numpy(np.arange(g, dtype=np.int64) * W + P[grp] - 1).to(dev)
            hsel = torch.index_select(sc.h[: g * W], 0, last)
            logits = torch.empty(g, dm.vocab, dtype=torch.float32, device=dev)
            lm_head(dm, hsel, logits)
            N.call("pse_scatter_rows", logits.data_ptr(), dm.vocab, gslots.data_ptr(), g, dm.vocab,
                   buf.data_ptr(), dm.vocab, buf.shape[0], st)
            last_tok = torch.from_numpy(np.array([prompts[idx][-1] for idx in grp], dtype=np.int32)).to(dev)
            cache.last_token.index_copy_(0, gslots.long(), last_tok)
        cache.note_lengths(ids, P.tolist())
    for _, cache in pairs:
        cache.check_status("prefill")
    for dm, cache in pairs:
        views = next_logits_views(cache, dm.vocab)
        out.append([views[cache.slot(r)] for r in ids])
    return out


@torch.no_grad()
def prefill_requests(draft_model, target_model, draft_cache, target_cache, request_ids, prompts,
                     max_tokens_per_call: int = 32768) -> dict:
    """Batched ``prefill_request`` (engine/speculative.py:53-73) for many
    requests, as the scheduler admits them (engine/scheduler.py:78-90): the
    result and both caches' state are those of calling ``prefill_request`` for
    each request in order (see ``prefill_many``).  Returns
    ``{request_id: (draft_logits, target_logits)}`` (device views of the
    per-slot next-logits rows)."""
    ids = list(request_ids)
    prompts = [list(p) for p in prompts]
    out = prefill_many([(draft_model, draft_cache), (target_model, target_cache)], ids, prompts,
                       max_tokens_per_call)
    if out is None:
        return {r: prefill_request(draft_model, target_model, draft_cache, target_cache, r, p)
                for r, p in zip(ids, prompts)}
    return {r: (dv, tv) for r, dv, tv in zip(ids, out[0], out[1])}


class _StepBuffers:
    def __init__(self, B: int, k: int, V: int, device, d_draft: int, draft_dtype):
        i32 = dict(dtype=torch.int32, device=device)
        self.B = B
        # the draft's tail call (its last round + its bonus, width 2): ids, the
        # row each request's next logits come from, those hidden rows
        self.ids2 = torch.empty(B, 2, **i32)
        self.sel = torch.empty(B, dtype=torch.int64, device=device)
        self.hsel = torch.empty(B, d_draft, dtype=draft_dtype, device=device)
        # the step's per-row host inputs, copied to the device in one transfer:
        # [slots_d | slots_t | req_key | steps | order_d | order_t | ords]
        # (ords: each row's request ordinal in the scheduler's output arena)
        self.dev_in = torch.zeros(7 * B, **i32)
        (self.slots_d, self.slots_t, self.req_key, self.steps, self.order_d, self.order_t,
         self.ords) = self.dev_in.view(7, B)
        self.base = torch.empty(k + 4, B, **i32)  # per-call base lengths (rounds, verify, bonus calls)
        self.round_ids = torch.empty(B, **i32)
        self.drafts = torch.empty(B, k, **i32)
        self.dlog = torch.empty(k, B, V, dtype=torch.float32, device=device)
        self.vlog = torch.empty(B * k, V, dtype=torch.float32, device=device)
        self.blog = torch.empty(B, V, dtype=torch.float32, device=device)
        self.tokens = torch.empty(B, k + 1, **i32)
        self.n_acc = torch.empty(B, **i32)
        self.final = torch.empty(B, **i32)
        self.u = torch.zeros(B, 2 * k + 1, dtype=torch.float64, device=device)
        self.vids = None    # verify from pending rows: ids [B, k+1], logits [B*(k+1), V], first positions [B]
        self.vlog2 = None
        self.basem1 = torch.empty(B, **i32)
        self.nacc1 = torch.empty(B, **i32)
        # the step's result, copied to pinned host memory in one transfer:
        # [tokens B*(k+1) | n_acc B | status_d | status_t | finished count | finished rows B]
        # (the last two only when the scheduler's commit runs in the step)
        n_pack = B * (k + 1) + B + 3 + B
        self.pack = torch.empty(n_pack, **i32)
        self.host_pack = torch.empty(n_pack, dtype=torch.int32, pin_memory=True)
        self.host_in = torch.empty(7 * B, dtype=torch.int32, pin_memory=True)
        self.host_pack_np = self.host_pack.numpy()  # same pinned memory
        self.host_in_np = self.host_in.numpy()


class CommitArena:
    """Device output arena of a scheduler run (engine/scheduler.py:107-126
    kept on the device): request ordinal o owns ``max_new[o]`` int32 entries at
    ``off[o]``; ``generated[o]`` counts its accepted tokens, overshoot
    included.  Buffers are reused across runs while they are large enough
    (``generation`` changes when they move, so captured steps are rebuilt)."""

    def __init__(self, device):
        self.device = device
        self.generation = 0
        self.cap_req = 0
        self.cap_out = 0
        self.off = self.max_new = self.generated = self.out = None

    def reset(self, max_new: np.ndarray) -> None:
        n = int(max_new.shape[0])
        off = np.zeros(n, dtype=np.int64)
        if n > 1:
            np.cumsum(max_new[:-1], out=off[1:])
        total = int(max_new.sum()) if n else 0
        if n > self.cap_req or total > self.cap_out or self.off is None:
            self.cap_req = max(n, 2 * self.cap_req, 64)
            self.cap_out = max(total, 2 * self.cap_out, 1024)
            i32 = dict(dtype=torch.int32, device=self.device)
            self.off = torch.zeros(self.cap_req, dtype=torch.int64, device=self.device)
            self.max_new = torch.zeros(self.cap_req, **i32)
            self.generated = torch.zeros(self.cap_req, **i32)
            self.out = torch.zeros(self.cap_out, **i32)
            self.generation += 1
        if n:
            self.off[:n].copy_(torch.from_numpy(off))
            self.max_new[:n].copy_(torch.from_numpy(max_new.astype(np.int32)))
        self.generated.zero_()


class StepRunner:
    """The device program of one speculative step for a (draft, target, caches, k)."""

    def __init__(self, dm_d, dm_t, dcache, tcache, k: int):
        if dm_d.vocab != dm_t.vocab:
            raise ValueError("draft and target vocabularies differ")
        self.dm_d, self.dm_t, self.dcache, self.tcache, self.k = dm_d, dm_t, dcache, tcache, k
        self.V = dm_t.vocab
        self.device = tcache.device
        self.bufs: dict[int, _StepBuffers] = {}
        self.graphs: dict = {}
        self.warm: set = set()
        self.request_steps: dict[str, int] = {}
        self.seed = DEFAULT_SEED
        self.use_graphs = USE_GRAPHS
        self.sc_d = Scratch(dm_d)
        self.sc_t = Scratch(dm_t)
        self.commit: CommitArena | None = None  # the scheduler's device output arena
        self._slots_key, self._slots_ids, self._slots_np = None, None, None
        self._ws_sizes: dict = {}  # (rows, draft / target context bound) -> split-KV workspace bytes

    # ---------------------------------------------------------------- device program
    def _ctx_bound(self, cache, dm) -> int:
        bound = cache.max_blocks * cache.block_size
        if dm.pos_emb is not None:
            bound = min(bound, dm.max_seq_len)
        return bound

    def _program(self, b: _StepBuffers, T: float, philox: bool, max_ctx_d: int, max_ctx_t: int,
                 in_pending: bool = False, out_defer: bool = False, commit: CommitArena | None = None) -> None:
        """One step on the device.  ``in_pending``: every row's last target
        position is pending (reserved, K/V unwritten); ``out_defer``: leave the
        rows pending instead of running the target's bonus call."""
        k, V, B = self.k, self.V, b.B
        st = N.stream_ptr()
        dnext = next_logits_buffer(self.dcache, V)
        tnext = next_logits_buffer(self.tcache, V)
        nu = 2 * k + 1
        if T > 0 and philox:
            N.call("pse_philox_uniforms", self.seed, b.req_key.data_ptr(), b.steps.data_ptr(), B, nu,
                   b.u.data_ptr(), st)
        # draft rounds (engine/speculative.py:92-113).  The last round's draft
        # call is not made here: its logits are never tested, and its KV write
        # merges with the bonus call below into one width-2 call.
        for j in range(k):
            if j == 0:
                src, idx = dnext, b.slots_d.data_ptr()
            else:
                src, idx = b.dlog[j - 1], None
            N.call("pse_sample_tokens", src.data_ptr(), V, idx, B, V, float(T), b.u.data_ptr(), nu, j,
                   b.drafts.data_ptr() + 4 * j, k, b.round_ids.data_ptr(), 1, st)
            if j + 1 < k:
                forward(self.dm_d, self.dcache, b.slots_d, b.round_ids, B, 1, b.base[j], max_ctx_d, b.dlog[j],
                        scratch=self.sc_d, row_order=b.order_d)
            else:
                # the last round's position is still allocated here, so the draft's
                # block tables and free list follow the reference's sequence exactly
                N.call("pse_kv_reserve", self.dcache.state, b.slots_d.data_ptr(), B, 1, b.base[j].data_ptr(), st)
        if not in_pending:
            # verify: one width-k target call (engine/speculative.py:115-117)
            forward(self.dm_t, self.tcache, b.slots_t, b.drafts.view(-1), B, k, b.base[k], max_ctx_t, b.vlog,
                    scratch=self.sc_t, row_order=b.order_t)
            t0, t0_stride, t0_index = tnext.data_ptr(), V, b.slots_t.data_ptr()
            ver, v_row = b.vlog.data_ptr(), k * V
        else:
            # every row's last position holds the previous step's final token,
            # reserved and counted but not yet computed.  The k draft positions
            # are reserved as the reference's width-k verify appends them, then
            # one width-(k+1) call runs from the pending position over
            # [final, d_1..d_k] without allocating; its column 0 gives what the
            # reference's bonus call returned as target_next.
            N.call("pse_kv_reserve", self.tcache.state, b.slots_t.data_ptr(), B, k, b.base[k].data_ptr(), st)
            lt = self.tcache.last_token
            N.call("pse_step_verify_ids", lt.data_ptr(), lt.numel(), b.slots_t.data_ptr(), b.drafts.data_ptr(),
                   b.base[k].data_ptr(), B, k, b.vids.data_ptr(), b.basem1.data_ptr(), st)
            forward(self.dm_t, self.tcache, b.slots_t, b.vids.view(-1), B, k + 1, b.basem1, max_ctx_t, b.vlog2,
                    scratch=self.sc_t, row_order=b.order_t, reserve=False)
            t0, t0_stride, t0_index = b.vlog2.data_ptr(), (k + 1) * V, None
            ver, v_row = b.vlog2.data_ptr() + 4 * V, (k + 1) * V
        # accept / reject / resample (engine/speculative.py:119-157)
        N.call("pse_spec_accept", t0, t0_stride, t0_index, ver, v_row, V,
               dnext.data_ptr(), V, b.slots_d.data_ptr(), b.dlog.data_ptr(), V, B * V,
               b.drafts.data_ptr(), b.u.data_ptr(), nu, B, k, V, float(T), b.tokens.data_ptr(),
               b.n_acc.data_ptr(), b.final.data_ptr(), st)
        if commit is not None:
            # the scheduler's per-row bookkeeping (engine/scheduler.py:107-126)
            nt = B * (k + 1)
            N.call("pse_sched_commit", b.tokens.data_ptr(), k + 1, b.n_acc.data_ptr(), b.ords.data_ptr(), B,
                   commit.off.data_ptr(), commit.max_new.data_ptr(), commit.generated.data_ptr(),
                   commit.out.data_ptr(), b.pack.data_ptr() + 4 * (nt + B + 2), st)
        # commit (engine/speculative.py:159-164)
        N.call("pse_kv_truncate", self.dcache.state, b.slots_d.data_ptr(), B, None, b.base[0].data_ptr(),
               b.n_acc.data_ptr(), st)
        N.call("pse_kv_truncate", self.tcache.state, b.slots_t.data_ptr(), B, None, b.base[k].data_ptr(),
               b.n_acc.data_ptr(), st)
        # bonus forwards (engine/speculative.py:166-177); the target's is
        # deferred to the next verify when out_defer.  The draft's is one width-2
        # call: [x_{k-1}, final] when every draft was accepted (the last round's
        # token was never computed), else [final, final] whose second position
        # lies past the row's length (its K/V lands in a block the row holds
        # and is overwritten by the next append, or is dropped); the next
        # logits are those after `final`.  The bonus position is allocated first
        # (as the reference's bonus append does), then the call runs at
        # base + min(n, k-1) without allocating.
        N.call("pse_kv_reserve", self.dcache.state, b.slots_d.data_ptr(), B, 1, b.base[k + 1].data_ptr(), st)
        N.call("pse_step_bonus_ids", b.n_acc.data_ptr(), b.drafts.data_ptr(), b.final.data_ptr(),
               b.base[0].data_ptr(), B, k, b.ids2.data_ptr(), b.base[k + 3].data_ptr(), b.sel.data_ptr(), st)
        forward(self.dm_d, self.dcache, b.slots_d, b.ids2.view(-1), B, 2, b.base[k + 3], max_ctx_d, None,
                scratch=self.sc_d, row_order=b.order_d, reserve=False)
        torch.index_select(self.sc_d.h[:2 * B], 0, b.sel, out=b.hsel)
        lm_head(self.dm_d, b.hsel, b.blog)
        N.call("pse_scatter_rows", b.blog.data_ptr(), V, b.slots_d.data_ptr(), B, V, dnext.data_ptr(), V,
               dnext.shape[0], st)
        if not out_defer:
            forward(self.dm_t, self.tcache, b.slots_t, b.final, B, 1, b.base[k + 2], max_ctx_t, b.blog,
                    scratch=self.sc_t, row_order=b.order_t)
            N.call("pse_scatter_rows", b.blog.data_ptr(), V, b.slots_t.data_ptr(), B, V, tnext.data_ptr(), V,
                   tnext.shape[0], st)
        else:
            # the reference's bonus append without its forward: the final
            # token's position is reserved in the same order (same blocks)
            N.call("pse_kv_reserve", self.tcache.state, b.slots_t.data_ptr(), B, 1, b.base[k + 2].data_ptr(), st)
        ld, lt = self.dcache.last_token, self.tcache.last_token
        N.call("pse_step_finish", b.final.data_ptr(), b.slots_d.data_ptr(), b.slots_t.data_ptr(), B, ld.data_ptr(),
               ld.numel(), lt.data_ptr(), lt.numel(), b.tokens.data_ptr(), k, b.n_acc.data_ptr(),
               self.dcache.status_tensor().data_ptr(), self.tcache.status_tensor().data_ptr(), b.pack.data_ptr(), st)

    # ---------------------------------------------------------------- host side
    def step(self, request_ids, draft_next_logits, target_next_logits, temperature, generator=None,
             uniforms=None, use_graph=None, defer_bonus=None) -> BatchStepResult:
        k, V = self.k, self.V
        B = len(request_ids)
        if B == 0:
            return BatchStepResult({}, {}, {}, {})
        # (the previous step's list, unchanged, is known to be unique)
        if self._slots_ids != request_ids and len(set(request_ids)) != B:
            raise ValueError("request_ids must be unique")
        dc, tc = self.dcache, self.tcache
        # slot arrays: reused while the request list and the slot assignment are unchanged
        skey = (dc.slot_version, tc.slot_version)
        if self._slots_key == skey and self._slots_ids == request_ids:
            sd_np, st_np = self._slots_np
        else:
            sd_np, st_np = dc.slots_np(request_ids), tc.slots_np(request_ids)
            self._slots_key, self._slots_ids, self._slots_np = skey, list(request_ids), (sd_np, st_np)
        dviews = next_logits_views(dc, V)
        tviews = next_logits_views(tc, V)
        pviews = pending_views(tc, V, st_np)
        sd = sd_np.tolist()
        stt = st_np.tolist()
        # logits handed back unchanged (the previous step's views) need no copy
        vals = [draft_next_logits[r] for r in request_ids]
        own = [dviews[x] for x in sd]
        if not all(map(operator.is_, vals, own)):
            for t, v in zip(vals, own):
                if t is not v and t.data_ptr() != v.data_ptr():
                    v.copy_(t.reshape(-1), non_blocking=True)
        vals = [target_next_logits[r] for r in request_ids]
        if not all(map(operator.is_, vals, map(pviews.__getitem__, stt))):
            foreign = [(t, x) for t, x in zip(vals, stt) if t is not pviews[x] and t is not tviews[x]]
            if foreign:
                # rows given other logits: a pending row's deferred call runs first
                # (it writes the row's K/V), then the given values replace its logits
                tc.flush_pending([x for _, x in foreign])
                for t, x in foreign:
                    v = tviews[x]
                    if t.data_ptr() != v.data_ptr():
                        v.copy_(t.reshape(-1), non_blocking=True)
        steps = self.request_steps
        key_np = steps_np = None
        if float(temperature) > 0 and uniforms is None and generator is None:
            key_np = np.array([_fnv1a(r) for r in request_ids], dtype=np.uint32).view(np.int32)
            steps_np = np.fromiter((steps.get(r, 0) for r in request_ids), np.int32, B)
        views = []
        prev_steps = []

        def while_device_runs():
            # the next-logits dicts depend only on the slots, and the per-request
            # step counts on nothing the step computes: both are done during the step
            views.append(dict(zip(request_ids, map(dviews.__getitem__, sd))))
            views.append(dict(zip(request_ids, map((tviews if defer_bonus is False else pviews).__getitem__, stt))))
            prev_steps.extend(map(steps.get, request_ids))
            for r, n in zip(request_ids, prev_steps):
                steps[r] = (n or 0) + 1

        try:
            b, nacc_np = self._run(request_ids, sd_np, st_np, temperature, generator, uniforms, use_graph,
                                   defer_bonus, key_np, steps_np, while_device_runs=while_device_runs)
        except BaseException:
            # a failed step does not count
            for r, n in zip(request_ids, prev_steps):
                if n is None:
                    steps.pop(r, None)
                else:
                    steps[r] = n
            raise
        toks = b.host_pack_np[:B * (k + 1)].reshape(B, k + 1).tolist()
        nacc = nacc_np.tolist()
        accepted = {r: toks[i][: nacc[i] + 1] for i, r in enumerate(request_ids)}
        n_acc = dict(zip(request_ids, nacc))
        dn, tn = views
        return BatchStepResult(accepted, n_acc, dn, tn)

    def step_rows(self, request_ids, sd_np, st_np, ords_np, commit: CommitArena, temperature, generator=None,
                  uniforms=None, use_graph=None, defer_bonus=None, req_key_np=None, steps_np=None):
        """The scheduler's form of ``step``: rows come as slot arrays, each
        request's next logits are already in its slot's row (as prefill and
        every step leave them), the accepted tokens stay on the device in
        ``commit`` (row i extends request ordinal ``ords_np[i]``) and nothing
        per row is built on the host.  ``req_key_np`` / ``steps_np`` key the
        device Philox stream when T > 0 and neither ``uniforms`` nor
        ``generator`` is given.  Returns (n_acc [B] int64, finished row
        indices in row order)."""
        B = len(request_ids)
        b, nacc_np = self._run(request_ids, sd_np, st_np, temperature, generator, uniforms, use_graph, defer_bonus,
                               req_key_np, steps_np, ords_np, commit)
        at = B * (self.k + 1) + B + 2
        nfin = int(b.host_pack_np[at])
        return nacc_np, b.host_pack_np[at + 1:at + 1 + nfin].copy()

    def _run(self, request_ids, sd_np, st_np, temperature, generator, uniforms, use_graph, defer_bonus,
             req_key_np=None, steps_np=None, ords_np=None, commit: CommitArena | None = None,
             while_device_runs=None):
        """Launch one step (replaying its graph when captured), copy its result
        to the host, raise a latched device error, update the host length
        mirrors.  ``while_device_runs`` (optional) is called after the launch,
        before waiting for the device.  Returns the step's buffers and n_acc as
        int64."""
        k, V = self.k, self.V
        B = len(request_ids)
        dc, tc = self.dcache, self.tcache
        out_defer = defer_bonus is not False
        for c in (dc, tc):
            if c.prefix is not None and c.prefix.idle:
                # idle prefix blocks give way to the step's worst-case growth (k + 2 tokens per row)
                c.prefix.make_room(B * ((k + 2 + c.block_size - 1) // c.block_size + 1))
        # rows whose target call is still owed: the fast program needs all of
        # them pending; a mixed batch (rows just admitted, or given other
        # logits) or an eager step first completes the pending ones
        in_pending = False
        if tc.pending_slots:
            stl = st_np.tolist()
            n_p = sum(map(tc.pending_slots.__contains__, stl))
            if n_p == B and out_defer:
                in_pending = True
            elif n_p:
                tc.flush_pending(stl)
        len_d = dc.lengths_np(sd_np)
        len_t = tc.lengths_np(st_np)
        for dm, c, lens in ((self.dm_d, dc, len_d), (self.dm_t, tc, len_t)):
            longest = int(lens.max()) + k + 1
            if dm.pos_emb is not None and longest > dm.max_seq_len:
                raise IndexError(f"position {longest - 1} beyond max_seq_len {dm.max_seq_len}")
            c.ensure_capacity_len(longest)
        b = self.bufs.get(B)
        if b is None:
            b = self.bufs[B] = _StepBuffers(B, k, V, self.device, self.dm_d.d_model, self.dm_d.dtype)
        if in_pending and b.vids is None:
            b.vids = torch.empty(B, k + 1, dtype=torch.int32, device=self.device)
            b.vlog2 = torch.empty(B * (k + 1), V, dtype=torch.float32, device=self.device)
        T = float(temperature)
        philox = False
        hin = b.host_in
        hnp = b.host_in_np
        hnp[:B] = sd_np
        hnp[B:2 * B] = st_np
        if T > 0:
            if uniforms is not None:
                u = torch.as_tensor(np.asarray(uniforms, dtype=np.float64) if not torch.is_tensor(uniforms)
                                    else uniforms, dtype=torch.float64)
                b.u.copy_(u.reshape(B, 2 * k + 1), non_blocking=True)
            elif generator is not None:
                b.u.copy_(torch.rand(B, 2 * k + 1, generator=generator, dtype=torch.float64), non_blocking=True)
            else:
                philox = True
                hnp[2 * B:3 * B] = req_key_np
                hnp[3 * B:4 * B] = steps_np
        # longest rows first: the attention kernels hand out work in this order
        hnp[4 * B:5 * B] = np.argsort(-len_d, kind="stable")
        hnp[5 * B:6 * B] = np.argsort(-len_t, kind="stable")
        if ords_np is not None:
            hnp[6 * B:7 * B] = ords_np
        b.dev_in.copy_(hin, non_blocking=True)

        graphs = self.use_graphs if use_graph is None else use_graph
        mcd, mct = self._ctx_bound(dc, self.dm_d), self._ctx_bound(tc, self.dm_t)
        if graphs:
            # size every buffer the program touches before the graph key is taken
            self.sc_d.ensure(2 * B)
            self.sc_t.ensure(B * (k + 1))
            ws = self._ws_sizes.get((B, mcd, mct))
            if ws is None:
                dmd, dmt = self.dm_d, self.dm_t
                ws = self._ws_sizes[(B, mcd, mct)] = (
                    max(N.size_call("pse_paged_attention_workspace", B, w, dmd.q_heads, dmd.kv_heads, dmd.head_dim,
                                    mcd) for w in (1, 2)),
                    max(N.size_call("pse_paged_attention_workspace", B, w, dmt.q_heads, dmt.kv_heads, dmt.head_dim,
                                    mct) for w in (k + 1, k, 1)))
            self.sc_d.ensure_ws(ws[0])
            self.sc_t.ensure_ws(ws[1])
        key = (B, T, philox, in_pending, out_defer, dc.generation, tc.generation, self.sc_d.generation,
               self.sc_t.generation, None if commit is None else (id(commit), commit.generation))
        if graphs and key in self.graphs:
            self.graphs[key].replay()
        elif graphs and key in self.warm:
            g = torch.cuda.CUDAGraph()
            with N.graph_capture(g):
                self._program(b, T, philox, mcd, mct, in_pending, out_defer, commit)
            self.graphs[key] = g
            g.replay()
        else:
            if graphs:
                # eager steps use the same context bound so the captured
                # program's buffers (split-KV workspace) are already sized
                self._program(b, T, philox, mcd, mct, in_pending, out_defer, commit)
                self.warm.add(key)
            else:
                ld = int(len_d.max()) + k + 1
                lt = int(len_t.max()) + k + 1
                self._program(b, T, philox, ld, lt + 1, in_pending, out_defer, commit)
        nt = B * (k + 1)
        if commit is None:
            b.host_pack.copy_(b.pack, non_blocking=True)
        else:  # the tokens stay on the device
            b.host_pack[nt:].copy_(b.pack[nt:], non_blocking=True)
        if while_device_runs is not None:
            while_device_runs()
        torch.cuda.current_stream().synchronize()
        hpn = b.host_pack_np
        status_d, status_t = int(hpn[nt + B]), int(hpn[nt + B + 1])
        if status_d or status_t:
            for c, s in ((dc, status_d), (tc, status_t)):
                if s:
                    c.check_status("speculative step")
        nacc_np = hpn[nt:nt + B].astype(np.int64)
        dc.note_lengths_slots(sd_np, len_d + nacc_np + 1)
        tc.note_lengths_slots(st_np, len_t + nacc_np + 1)
        if out_defer:
            tc.pending_slots.update(st_np.tolist())
            tc._pending_dm = self.dm_t
            tc._flusher = _flush_pending
        return b, nacc_np


def runner_for(draft_model, target_model, draft_cache, target_cache, k: int) -> StepRunner:
    dm_d = device_model(draft_model, draft_cache.dtype, draft_cache.device)
    dm_t = device_model(target_model, target_cache.dtype, target_cache.device)
    runners = target_cache.__dict__.setdefault("_runners", {})
    key = (id(draft_cache), id(dm_d), id(dm_t), k)
    r = runners.get(key)
    if r is None or r.dm_d is not dm_d or r.dm_t is not dm_t or r.dcache is not draft_cache:
        r = runners[key] = StepRunner(dm_d, dm_t, draft_cache, target_cache, k)
    return r


@torch.no_grad()
def batched_speculative_step(draft_model, target_model, request_ids, draft_cache, target_cache,
                             draft_next_logits, target_next_logits, k, temperature, generator=None, *,
                             uniforms=None, use_graph=None, defer_bonus=None) -> BatchStepResult:
    """engine/speculative.py:76-177 on the device.

    By default (``defer_bonus`` None or True) the target's width-1 bonus call
    is deferred into the next step's verify, which runs at width k+1 (the
    final token, then the k drafts): one target pass per step instead of two,
    same accepted tokens, same block tables, lengths and free lists.  The
    result's ``target_next_logits`` are then ``PendingLogits``: passing them
    back unchanged is free, reading them runs the deferred call first.
    ``defer_bonus=False`` runs the bonus call inside the step (the reference's
    structure; the logits are plain views)."""
    runner = runner_for(draft_model, target_model, draft_cache, target_cache, k)
    return runner.step(list(request_ids), draft_next_logits, target_next_logits, temperature, generator,
                       uniforms, use_graph, defer_bonus)
