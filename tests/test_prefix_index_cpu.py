"""Host logic of the prefix index (pse.prefix_cache.PrefixIndex) on a CPU
stand-in of a cache's bookkeeping arrays: chained content keys, the
longest-prefix lookup that leaves the last token, admission waves, reference
counts, least-recently-used eviction onto the free stack, and the copy a
truncate inside a shared block makes.  No GPU."""
from __future__ import annotations

import numpy as np
import torch

from pse.prefix_cache import PrefixIndex

BS, NB, SLOTS, WIDTH = 4, 32, 8, 16


class _Blocks:
    def __init__(self):
        self.block_table = torch.full((SLOTS, WIDTH), -1, dtype=torch.int32)
        self.nblocks = torch.zeros(SLOTS, dtype=torch.int32)
        self.seq_len = torch.zeros(SLOTS, dtype=torch.int32)
        self.free_stack = torch.arange(NB - 1, -1, -1, dtype=torch.int32)  # pops 0, 1, 2, ...
        self.scalars = torch.tensor([NB, 0, 0, 0], dtype=torch.int32)
        self.block_free = torch.ones(NB, dtype=torch.uint8)

    @property
    def free_top(self):
        return self.scalars[0:1]


class _Alloc:
    def __init__(self, b):
        self.b = b

    @property
    def num_free(self):
        return int(self.b.free_top.item())

    def allocate(self):
        top = self.num_free - 1
        if top < 0:
            raise MemoryError
        blk = int(self.b.free_stack[top])
        self.b.free_top.fill_(top)
        self.b.block_free[blk] = 0
        return blk


class _Cache:
    def __init__(self):
        self.block_size, self.device = BS, torch.device("cpu")
        self._blocks = _Blocks()
        self.allocator = _Alloc(self._blocks)
        self._len_np = np.zeros(SLOTS, dtype=np.int64)
        self.k_pool = torch.randn(2, NB, 1, BS, 3)
        self.v_pool = torch.randn(2, NB, 1, BS, 3)

    def grow_row(self, slot, n_tokens):
        """What the reserve kernel does: blocks for the row's new tokens, after its head."""
        b = self._blocks
        have = int(b.nblocks[slot])
        need = (int(b.seq_len[slot]) + n_tokens + BS - 1) // BS
        for j in range(have, need):
            b.block_table[slot, j] = self.allocator.allocate()
        b.nblocks[slot] = need
        b.seq_len[slot] += n_tokens
        self._len_np[slot] = int(b.seq_len[slot])

    def release(self, slot):
        """What the release kernel does: free the row's table entries in order."""
        b = self._blocks
        for j in range(int(b.nblocks[slot])):
            blk = int(b.block_table[slot, j])
            top = self.allocator.num_free
            b.free_stack[top] = blk
            b.free_top.fill_(top + 1)
            b.block_free[blk] = 1
            b.block_table[slot, j] = -1
        b.nblocks[slot] = 0
        b.seq_len[slot] = 0


def _prefill(c, idx, slot, prompt):
    hits = idx.lookup(prompt)
    idx.attach([slot], [hits])
    c.grow_row(slot, len(prompt) - len(hits) * BS)
    idx.register([slot], [prompt])
    return hits


def _conserved(c, idx, live_slots):
    b = c._blocks
    free = b.free_stack[: c.allocator.num_free].tolist()
    owned = [int(x) for s in live_slots for x in b.block_table[s, : int(b.nblocks[s])].tolist()]
    held = set(owned) | set(idx.idle)
    assert sorted(set(free)) == sorted(free)  # no id twice on the free list
    assert sorted(set(free) | held) == list(range(NB)) and not set(free) & held
    assert all(b.block_free[x] == 1 for x in free) and all(b.block_free[x] == 0 for x in held)


def test_lookup_leaves_last_token_and_follows_chains():
    c = _Cache()
    idx = PrefixIndex(c)
    p = list(range(10))  # 2 full blocks + 2 tokens
    assert _prefill(c, idx, 0, p) == []
    assert idx.row_blocks[0] == c._blocks.block_table[0, :2].tolist()
    assert idx.lookup(p) == idx.row_blocks[0]                  # 9 tokens shared at most: both full blocks
    assert idx.lookup(p[:8]) == idx.row_blocks[0][:1]          # 8 tokens: the second block holds the last one
    assert idx.lookup(p[:4] + [99] * 6) == idx.row_blocks[0][:1]
    # equal second-block tokens behind a different first block share nothing
    assert idx.lookup([50, 51, 52, 53] + p[4:]) == []


def test_waves_put_repeated_first_blocks_second():
    c = _Cache()
    idx = PrefixIndex(c)
    a, b = [1] * 5, [2] * 6
    assert idx.waves([a, b, a + [3], [7, 7], b + [4], [1] * 4]) == [[0, 1, 3, 5], [2, 4]]


def test_refs_idle_lru_eviction_and_conservation():
    c = _Cache()
    idx = PrefixIndex(c)
    sys_p = list(range(100, 112))  # 3 full blocks
    _prefill(c, idx, 0, sys_p + [1, 2])
    hits = _prefill(c, idx, 1, sys_p + [3])
    assert len(hits) == 3 and all(idx.refs[h] == 3 for h in hits)
    _prefill(c, idx, 2, list(range(200, 209)))
    _conserved(c, idx, [0, 1, 2])
    for s in (0, 1, 2):
        idx.release_rows([s])
        c.release(s)
    # every indexed block is idle now; row 0's blocks went idle first
    assert set(idx.idle) == set(idx.refs) and all(v == 1 for v in idx.refs.values())
    _conserved(c, idx, [])
    free0 = c.allocator.num_free
    lru = list(idx.idle)[:2]
    idx.make_room(free0 + 2, keep=[lru[0]])
    assert lru[0] in idx.idle and lru[1] not in idx.idle and c.allocator.num_free == free0 + 2
    assert c._blocks.free_stack[free0:free0 + 2].tolist()[0] == lru[1]
    assert idx.lookup(sys_p + [9]) == [lru[0]]  # kept; the chain breaks at the evicted second block
    _conserved(c, idx, [])
    idx.clear()
    assert not idx.idle and not idx.refs and not idx.by_key and c.allocator.num_free == NB
    _conserved(c, idx, [])


def test_truncate_inside_shared_block_copies_it():
    c = _Cache()
    idx = PrefixIndex(c)
    p = list(range(300, 313))  # 3 full blocks + 1
    _prefill(c, idx, 0, p)
    _prefill(c, idx, 1, p[:12] + [7, 8])
    shared = list(idx.row_blocks[1])
    # the row's own blocks first go back (the kernel truncate to the shared length)
    b = c._blocks
    own = b.block_table[1, 3: int(b.nblocks[1])].tolist()
    for j, blk in enumerate(own):
        top = c.allocator.num_free
        b.free_stack[top] = blk
        b.free_top.fill_(top + 1)
        b.block_free[blk] = 1
        b.block_table[1, 3 + j] = -1
    b.nblocks[1] = 3
    b.seq_len[1] = 12
    idx.truncate_shared(1, 6)
    new = int(b.block_table[1, 1])
    assert int(b.block_table[1, 0]) == shared[0] and new not in shared
    assert int(b.nblocks[1]) == 2 and int(b.seq_len[1]) == 6 and c._len_np[1] == 6
    assert torch.equal(c.k_pool[:, new], c.k_pool[:, shared[1]])
    assert torch.equal(c.v_pool[:, new], c.v_pool[:, shared[1]])
    assert idx.row_blocks[1] == shared[:1] and idx.refs[shared[0]] == 3 and idx.refs[shared[1]] == 2
    _conserved(c, idx, [0, 1])
