"""CPU restatement of the reference paged KV cache (engine/paged_cache.py).

Semantics kept exactly, because the device free list must reproduce them bit
for bit:

* the free list starts as ``[0, 1, ..., n-1]`` and ``allocate`` pops from the
  END, so the first block handed out is ``n-1`` (engine/paged_cache.py:39, 45-48);
* ``free`` pushes on the end and raises ``ValueError`` on a double free
  (engine/paged_cache.py:50-56);
* ``append`` allocates the missing blocks of a row, in table order, before
  writing (engine/paged_cache.py:116-136);
* ``truncate`` frees trailing blocks from the table END, i.e. in reverse table
  order (engine/paged_cache.py:151-153);
* ``free_request`` frees in FORWARD table order (engine/paged_cache.py:156-160).

Pools are per layer ``[num_blocks, n_heads, block_size, head_dim]``
(engine/paged_cache.py:83-88).
"""
from __future__ import annotations

import torch


class BlockAllocator:
    """LIFO stack of free block ids, engine/paged_cache.py:32-56."""

    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self._stack: list[int] = list(range(num_blocks))
        self._is_free = [True] * num_blocks

    @property
    def num_free(self) -> int:
        return len(self._stack)

    def free_list(self) -> list[int]:
        """Bottom-to-top copy of the stack (the reference's ``_free`` list)."""
        return list(self._stack)

    def allocate(self) -> int:
        if not self._stack:
            raise MemoryError(f"paged KV-cache exhausted: all {self.num_blocks} blocks in use")
        block = self._stack.pop()
        self._is_free[block] = False
        return block

    def free(self, block_id: int) -> None:
        if self._is_free[block_id]:
            raise ValueError(f"block {block_id} freed twice")
        self._is_free[block_id] = True
        self._stack.append(block_id)


class PagedKVCache:
    """engine/paged_cache.py:59-198."""

    def __init__(self, n_layers, n_heads, head_dim, block_size, num_blocks, dtype=torch.float32):
        self.n_layers = n_layers
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.allocator = BlockAllocator(num_blocks)
        shape = (num_blocks, n_heads, block_size, head_dim)
        self._k_pool = [torch.zeros(shape, dtype=dtype) for _ in range(n_layers)]
        self._v_pool = [torch.zeros(shape, dtype=dtype) for _ in range(n_layers)]
        self._tables: dict[str, list[int]] = {}
        self._lengths: dict[str, int] = {}

    # --- bookkeeping (engine/paged_cache.py:92-102) ---
    def create_request(self, request_id: str) -> None:
        if request_id in self._tables:
            raise ValueError(f"request {request_id} already exists in this cache")
        self._tables[request_id] = []
        self._lengths[request_id] = 0

    def length(self, request_id: str) -> int:
        return self._lengths[request_id]

    def num_blocks_in_use(self, request_id: str) -> int:
        return len(self._tables[request_id])

    def block_table(self, request_id: str) -> list[int]:
        return list(self._tables[request_id])

    def _blocks_for(self, n_tokens: int) -> int:
        return 0 if n_tokens == 0 else (n_tokens - 1) // self.block_size + 1

    # --- engine/paged_cache.py:104-138 ---
    def append(self, request_id, new_k, new_v) -> None:
        n_new = new_k[0].shape[1]
        table = self._tables[request_id]
        start = self._lengths[request_id]
        # Layer 0's pass allocates every block index the write reaches, in order.
        while len(table) < self._blocks_for(start + n_new):
            table.append(self.allocator.allocate())
        bs = self.block_size
        for layer in range(self.n_layers):
            for t in range(n_new):
                pos = start + t
                blk, off = table[pos // bs], pos % bs
                self._k_pool[layer][blk, :, off, :] = new_k[layer][:, t, :]
                self._v_pool[layer][blk, :, off, :] = new_v[layer][:, t, :]
        self._lengths[request_id] = start + n_new

    # --- engine/paged_cache.py:140-154 ---
    def truncate(self, request_id: str, new_length: int) -> None:
        old = self._lengths[request_id]
        if new_length > old:
            raise ValueError(f"truncate({new_length}) > current length {old}")
        table = self._tables[request_id]
        keep = self._blocks_for(new_length)
        while len(table) > keep:
            self.allocator.free(table.pop())
        self._lengths[request_id] = new_length

    # --- engine/paged_cache.py:156-160 ---
    def free_request(self, request_id: str) -> None:
        for block in self._tables.pop(request_id):
            self.allocator.free(block)
        del self._lengths[request_id]

    # --- engine/paged_cache.py:162-198 ---
    def gather(self, request_ids):
        lengths = torch.tensor([self._lengths[r] for r in request_ids], dtype=torch.long)
        max_len = int(lengths.max().item()) if len(lengths) else 0
        batch = len(request_ids)
        mask = torch.zeros(batch, max_len, dtype=torch.bool)
        for i, r in enumerate(request_ids):
            mask[i, : self._lengths[r]] = True
        k_out, v_out = [], []
        bs = self.block_size
        for layer in range(self.n_layers):
            dt = self._k_pool[layer].dtype
            kb = torch.zeros(batch, self.n_heads, max_len, self.head_dim, dtype=dt)
            vb = torch.zeros(batch, self.n_heads, max_len, self.head_dim, dtype=dt)
            for i, r in enumerate(request_ids):
                n = self._lengths[r]
                for j, blk in enumerate(self._tables[r]):
                    lo = j * bs
                    take = min(bs, n - lo)
                    if take <= 0:
                        break
                    kb[i, :, lo:lo + take] = self._k_pool[layer][blk, :, :take]
                    vb[i, :, lo:lo + take] = self._v_pool[layer][blk, :, :take]
            k_out.append(kb)
            v_out.append(vb)
        return k_out, v_out, mask, lengths
