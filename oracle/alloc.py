"""Batched restatement of the reference free list (engine/paged_cache.py:32-56,
116-130, 140-160) in the form the device kernels use: an array stack plus an
exclusive prefix sum over the rows of one call, rows in call order.

Why the batched form equals the reference's sequential one:

* allocate is ``pop()`` from the stack top, rows processed in call order, each
  row's new blocks in table order (engine/paged_cache.py:120-124).  Row i's m-th
  new block is therefore the (off_i + m)-th pop, i.e. ``stack[top-1-(off_i+m)]``
  with ``off_i`` the exclusive prefix sum of the blocks the earlier rows need;
* truncate pushes a row's trailing blocks from the table end
  (engine/paged_cache.py:152-153): row i's m-th freed block is
  ``table[nb_i-1-m]`` and lands at ``stack[top + off_i + m]``;
* free_request pushes the table in forward order (engine/paged_cache.py:158-159):
  ``table[m]`` lands at ``stack[top + off_i + m]``.

Everything is integer arithmetic; the tests compare it bit for bit with a
sequential ``oracle.paged_cache.BlockAllocator`` replay and with the kernels.
"""
from __future__ import annotations

import numpy as np

OOM = 1
TABLE_OVERFLOW = 2
TRUNCATE_BEYOND_LENGTH = 4
DOUBLE_FREE = 8


def blocks_for(n_tokens, block_size: int):
    n = np.asarray(n_tokens, dtype=np.int64)
    return np.where(n == 0, 0, (n - 1) // block_size + 1)


class BlockState:
    """Host mirror of one cache's device bookkeeping."""

    def __init__(self, num_blocks: int, block_size: int, num_slots: int, max_blocks: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.stack = np.arange(num_blocks, dtype=np.int64)
        self.top = num_blocks
        self.block_free = np.ones(num_blocks, dtype=bool)
        self.table = np.full((num_slots, max_blocks), -1, dtype=np.int64)
        self.seq_len = np.zeros(num_slots, dtype=np.int64)
        self.nblocks = np.zeros(num_slots, dtype=np.int64)
        self.status = 0

    def free_list(self) -> list[int]:
        return self.stack[: self.top].tolist()

    def reserve(self, slots, width):
        """Make room for ``width`` more tokens in every row (an int, or one per
        row: one append per row in row order) and advance the rows' lengths;
        returns the lengths before the call.

        On exhaustion the state is the reference's after its ``MemoryError``
        (engine/paged_cache.py:46-47 raised inside the per-row append loop of
        engine/batched_forward.py:67-70): rows before the failing row are
        complete, the failing row keeps the blocks it got before the pool ran
        dry, its length and every later row are untouched."""
        slots = np.asarray(slots, dtype=np.int64)
        width = np.broadcast_to(np.asarray(width, dtype=np.int64), slots.shape)  # one width, or one per row
        base = self.seq_len[slots].copy()
        want = blocks_for(base + width, self.block_size)
        if np.any(want > self.table.shape[1]):
            self.status |= TABLE_OVERFLOW
            return base
        need = np.maximum(want - self.nblocks[slots], 0)
        off = np.concatenate([[0], np.cumsum(need)[:-1]]).astype(np.int64)
        got = np.clip(self.top - off, 0, need)
        complete = off + need <= self.top
        for i, s in enumerate(slots):
            for m in range(int(got[i])):
                blk = int(self.stack[self.top - 1 - (off[i] + m)])
                self.table[s, self.nblocks[s] + m] = blk
                self.block_free[blk] = False
            self.nblocks[s] += got[i]
            if complete[i]:
                self.seq_len[s] = base[i] + width[i]
        self.top -= int(got.sum())
        if not complete.all():
            self.status |= OOM
        return base

    def _push(self, blocks_per_row):
        total = sum(len(b) for b in blocks_per_row)
        pos = self.top
        for blocks in blocks_per_row:
            for blk in blocks:
                if self.block_free[blk]:
                    self.status |= DOUBLE_FREE
                self.block_free[blk] = True
                self.stack[pos] = blk
                pos += 1
        self.top += total

    def truncate(self, slots, new_len):
        slots = np.asarray(slots, dtype=np.int64)
        new_len = np.asarray(new_len, dtype=np.int64)
        freed = []
        for s, n in zip(slots, new_len):
            if n > self.seq_len[s]:
                self.status |= TRUNCATE_BEYOND_LENGTH
                freed.append([])
                continue
            keep = int(blocks_for(n, self.block_size))
            nb = int(self.nblocks[s])
            freed.append([int(self.table[s, b]) for b in range(nb - 1, keep - 1, -1)])
            self.nblocks[s] = keep
            self.seq_len[s] = n
        self._push(freed)

    def release(self, slots):
        slots = np.asarray(slots, dtype=np.int64)
        freed = [[int(self.table[s, b]) for b in range(int(self.nblocks[s]))] for s in slots]
        for s in slots:
            self.nblocks[s] = 0
            self.seq_len[s] = 0
        self._push(freed)

    def row_table(self, slot: int) -> list[int]:
        return self.table[slot, : self.nblocks[slot]].tolist()
