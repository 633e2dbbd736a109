"""Prefix caching for a PagedKVCache: requests whose prompts start with the
same tokens share the physical blocks of that prefix (the reference lists it
as future work, README.md:216-219, and has no code for it: the block-table
structure of engine/paged_cache.py:59-198 is what makes shared blocks
possible).

With ``PagedKVCache(..., prefix_cache=True)`` the full blocks of every
prefilled prompt are indexed by content: block j of a prompt is keyed by the
chain (key of block j-1, its ``block_size`` token ids), so a key names the
whole prefix up to the end of that block.  A later prompt that starts with an
indexed prefix maps those physical blocks into the head of its own block table
and computes only the rest: the K/V of a position depends only on the tokens
up to it, so the shared positions' K/V are already in the pool.

Ownership.  An indexed block is held by the index and by every live row whose
table starts with it (``refs``); it never returns to the free list while a row
uses it.  Rows never write into a shared block: sharing stops before a prompt's
last token (at least one token is computed, for the next-token logits), every
later position lies in a block the row owns, and a truncate that keeps part of
a shared block first copies it into a block of the row's own.  When the last
row using a block is freed, the block stays indexed but idle; idle blocks go
back to the free list, least recently used first, when an admission or a step
needs room (``make_room``) or on ``clear``.

Block tables and free lists then differ from the reference's allocation order
(blocks are reused instead of reallocated); with the default
``prefix_cache=False`` none of this runs and the order is the reference's.
"""
from __future__ import annotations

from collections import OrderedDict

import torch


class PrefixIndex:
    """Content index of one cache's full prompt blocks (see the module docstring)."""

    def __init__(self, cache):
        self.c = cache
        self.by_key: dict = {}                  # chain key -> (block id, parent block id, token ids)
        self.key_of: dict = {}                  # block id -> chain key
        self.refs: dict = {}                    # block id -> holders (the index + live rows)
        self.idle: OrderedDict = OrderedDict()  # blocks only the index holds, least recently used first
        self.row_blocks: dict = {}              # slot -> block ids shared at the head of its table
        self.hit_tokens = 0
        self.lookup_tokens = 0
        self.evicted = 0

    # ------------------------------------------------------------------ lookup
    def _keys(self, prompt, n_blocks):
        bs = self.c.block_size
        keys, parent = [], None
        for j in range(n_blocks):
            toks = tuple(prompt[j * bs:(j + 1) * bs])
            parent = hash((parent, toks))
            keys.append((parent, toks))
        return keys

    def lookup(self, prompt) -> list:
        """Block ids of the longest indexed prefix of ``prompt`` that leaves at
        least its last token to compute."""
        bs = self.c.block_size
        n = (len(prompt) - 1) // bs if prompt else 0
        found, parent_blk, parent_key = [], None, None
        for j in range(n):
            toks = tuple(prompt[j * bs:(j + 1) * bs])
            key = hash((parent_key, toks))
            e = self.by_key.get(key)
            if e is None or e[1] != parent_blk or e[2] != toks:
                break
            found.append(e[0])
            parent_blk, parent_key = e[0], key
        self.lookup_tokens += len(prompt)
        self.hit_tokens += len(found) * bs
        return found

    def waves(self, prompts) -> list:
        """Order of prefill inside one admission: the first prompt of every
        distinct first block goes in the first wave, the others in the second,
        so they find the first wave's blocks indexed.  Lists of indices."""
        bs = self.c.block_size
        first, second, seen = [], [], set()
        for i, p in enumerate(prompts):
            key = tuple(p[:bs]) if len(p) > bs else None
            if key is None or key not in seen:
                first.append(i)
                if key is not None:
                    seen.add(key)
            else:
                second.append(i)
        return [w for w in (first, second) if w]

    # ------------------------------------------------------------------ rows
    def attach(self, slots, hits) -> None:
        """Start each row ``slots[i]`` (empty, just created) with the shared
        blocks ``hits[i]``: table head, block count and length on the device,
        the host length mirror, references."""
        c = self.c
        bs = c.block_size
        rows = [(s, h) for s, h in zip(slots, hits) if h]
        if not rows:
            return
        for s, h in rows:
            for b in h:
                self.refs[b] += 1
                self.idle.pop(b, None)
            self.row_blocks[s] = list(h)
            c._len_np[s] = len(h) * bs
        dev = c.device
        width = max(len(h) for _, h in rows)
        tbl = torch.full((len(rows), width), -1, dtype=torch.int32)
        for i, (_, h) in enumerate(rows):
            tbl[i, :len(h)] = torch.tensor(h, dtype=torch.int32)
        idx = torch.tensor([s for s, _ in rows], dtype=torch.long).to(dev)
        nb = torch.tensor([len(h) for _, h in rows], dtype=torch.int32).to(dev)
        blocks = c._blocks
        # a created row's table is all -1: write its head
        blocks.block_table[idx.view(-1, 1), torch.arange(width, device=dev).view(1, -1)] = tbl.to(dev)
        blocks.nblocks.index_copy_(0, idx, nb)
        blocks.seq_len.index_copy_(0, idx, nb * bs)

    def register(self, slots, prompts) -> None:
        """Index the full prompt blocks of freshly prefilled rows.  A row's
        shared run grows over the blocks it indexes (stopping at the first block
        whose content another physical block already holds)."""
        c = self.c
        bs = c.block_size
        todo = [(s, p) for s, p in zip(slots, prompts) if len(p) // bs > len(self.row_blocks.get(s, ()))]
        if not todo:
            return
        idx = torch.tensor([s for s, _ in todo], dtype=torch.long).to(c.device)
        tables = c._blocks.block_table.index_select(0, idx).cpu().tolist()
        for (s, p), row in zip(todo, tables):
            shared = self.row_blocks.setdefault(s, [])
            full = len(p) // bs
            keys = self._keys(p, full)
            parent = shared[-1] if shared else None
            for j in range(len(shared), full):
                key, toks = keys[j]
                if key in self.by_key:
                    break
                b = row[j]
                self.by_key[key] = (b, parent, toks)
                self.key_of[b] = key
                self.refs[b] = 2  # the index and this row
                shared.append(b)
                parent = b
            if not shared:
                del self.row_blocks[s]

    def detach(self, slot) -> int:
        """Drop a row's references to its shared blocks (before it is released
        or its blocks are taken over); returns how many it had."""
        shared = self.row_blocks.pop(slot, None)
        if not shared:
            return 0
        for b in shared:
            self.refs[b] -= 1
            if self.refs[b] == 1:
                self.idle[b] = None
                self.idle.move_to_end(b)
        return len(shared)

    def release_rows(self, slots) -> None:
        """Before the release kernel frees ``slots``: shared blocks leave the
        head of each row's table (so only the row's own blocks are freed, in
        table order) and the row's references are dropped."""
        blocks = self.c._blocks
        for s in slots:
            n = self.detach(s)
            if n:
                mb = blocks.block_table.shape[1]
                blocks.block_table[s, :mb - n] = blocks.block_table[s, n:].clone()
                blocks.block_table[s, mb - n:] = -1
                blocks.nblocks[s] -= n

    def shared_tokens(self, slot) -> int:
        return len(self.row_blocks.get(slot, ())) * self.c.block_size

    def truncate_shared(self, slot, new_length) -> None:
        """Truncate ``slot`` below the end of its shared run; the row holds its
        shared run and nothing else (its own blocks were released first).  A
        shared block that stays partly in use is copied into a block of the
        row's own; shared blocks past the new length leave the row's table (the
        index keeps them)."""
        c = self.c
        bs = c.block_size
        shared = self.row_blocks.get(slot, [])
        keep_full = new_length // bs
        partial = new_length % bs != 0
        blocks = c._blocks
        n_keep = keep_full
        if partial:
            old = shared[keep_full]
            self.make_room(1)
            new = c.allocator.allocate()  # raises MemoryError like any allocation
            for pool in (c.k_pool, c.v_pool):
                pool[:, new].copy_(pool[:, old])
            blocks.block_table[slot, keep_full] = new
            n_keep += 1
        blocks.block_table[slot, n_keep:len(shared)] = -1
        blocks.nblocks[slot] = n_keep
        blocks.seq_len[slot] = new_length
        for b in shared[keep_full:]:
            self.refs[b] -= 1
            if self.refs[b] == 1:
                self.idle[b] = None
                self.idle.move_to_end(b)
        if keep_full:
            self.row_blocks[slot] = shared[:keep_full]
        else:
            self.row_blocks.pop(slot, None)
        c._len_np[slot] = new_length

    # ------------------------------------------------------------------ room
    def make_room(self, blocks_needed: int, keep=()) -> None:
        """Return idle blocks (least recently used first, none of ``keep``) to
        the free list until ``blocks_needed`` are free or none is idle.  Reads
        the free count from the device only when idle blocks exist."""
        if not self.idle:
            return
        free = self.c.allocator.num_free
        if free >= blocks_needed:
            return
        keep = set(keep)
        out = []
        for b in self.idle:
            if free + len(out) >= blocks_needed:
                break
            if b not in keep:
                out.append(b)
        self._evict(out)

    def clear(self) -> None:
        """Return every idle block to the free list and forget them."""
        self._evict(list(self.idle))

    def _evict(self, ids) -> None:
        if not ids:
            return
        c = self.c
        blocks = c._blocks
        for b in ids:
            del self.idle[b]
            del self.refs[b]
            key = self.key_of.pop(b)
            del self.by_key[key]
        # the free stack's top is read here (stream-ordered after the device's own pushes and pops)
        top = int(blocks.free_top.item())
        t = torch.tensor(ids, dtype=torch.int32).to(c.device)
        blocks.free_stack[top:top + len(ids)] = t
        blocks.block_free[t.long()] = 1
        blocks.free_top.fill_(top + len(ids))
        self.evicted += len(ids)

    def stats(self) -> dict:
        return {"indexed_blocks": len(self.refs), "idle_blocks": len(self.idle), "hit_tokens": self.hit_tokens,
                "lookup_tokens": self.lookup_tokens, "evicted_blocks": self.evicted}
