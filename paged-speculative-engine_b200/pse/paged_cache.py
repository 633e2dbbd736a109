"""Device-resident paged KV cache with the reference's Python API
(engine/paged_cache.py:32-198).

Layout in HBM (one object per model):

* ``k_pool`` / ``v_pool``: ``[n_layers, num_blocks, n_heads, block_size,
  head_dim]`` in the cache dtype -- the reference's per-layer
  ``[num_blocks, n_heads, block_size, head_dim]`` pools stacked, so one
  block of one head is a contiguous ``block_size x head_dim`` tile;
* ``block_table`` ``[num_slots, max_blocks]`` int32, ``seq_len`` / ``nblocks``
  ``[num_slots]`` int32: one row (slot) per live request;
* ``free_stack`` ``[num_blocks]`` int32 + ``free_top``: the reference's LIFO
  free list (engine/paged_cache.py:39, 45-56), bit for bit;
* ``status``: the device error latch (see include/pse.h).

Request ids map to slots on the host.  Lengths are mirrored on the host
exactly (every length change is known there without a device read);
``num_blocks_in_use`` and ``allocator.num_free`` read the device.

A target cache driven by the speculative step can hold *pending* slots: the
row's last position (the step's final token) is reserved and counted, as the
reference's bonus append leaves it, but its K/V is written by the next step's
verify.  Tables, lengths and the free list are exact meanwhile; calls that
read or extend a row's K/V (``append``, ``truncate``, ``gather``,
``batched_forward_append``) first run the deferred target call for it.

Errors keep the reference's exception types: ``MemoryError`` on exhaustion,
``ValueError`` on a duplicate request, a truncate beyond the length or a
double free.  Device-detected errors (exhaustion inside a batched forward) are
raised at the next synchronisation point of the call that caused them; the
cache state then equals the reference's state after its exception.
"""
from __future__ import annotations

from collections.abc import Mapping

import numpy as np
import torch

from . import _native as N
from .prefix_cache import PrefixIndex


def _blocks_for(n: int, bs: int) -> int:
    return 0 if n == 0 else (n - 1) // bs + 1


class _DeviceBlocks:
    """Device bookkeeping arrays of one pool + the ctypes struct that points at them."""

    def __init__(self, num_blocks: int, block_size: int, num_slots: int, max_blocks: int, device):
        i32 = dict(dtype=torch.int32, device=device)
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_slots, self.max_blocks = num_slots, max_blocks
        self.block_table = torch.empty(num_slots, max_blocks, **i32)
        self.seq_len = torch.empty(num_slots, **i32)
        self.nblocks = torch.empty(num_slots, **i32)
        self.free_stack = torch.empty(max(num_blocks, 1), **i32)
        self.scalars = torch.zeros(4, **i32)  # [free_top, status, scratch id, pad]
        self.block_free = torch.empty(max(num_blocks, 1), dtype=torch.uint8, device=device)
        self.state = N.BlockState(
            self.block_table.data_ptr(), self.seq_len.data_ptr(), self.nblocks.data_ptr(),
            self.free_stack.data_ptr(), self.scalars.data_ptr(), self.block_free.data_ptr(),
            self.scalars.data_ptr() + 4, num_blocks, block_size, max_blocks, num_slots,
        )
        N.call("pse_block_init", self.state, N.stream_ptr())

    @property
    def free_top(self) -> torch.Tensor:
        return self.scalars[0:1]

    @property
    def status(self) -> torch.Tensor:
        return self.scalars[1:2]

    @property
    def scratch_id(self) -> torch.Tensor:
        return self.scalars[2:3]


class _LengthView(Mapping):
    """Read-only ``{request_id: length}`` over a cache's per-slot mirror."""

    def __init__(self, cache):
        self._c = cache

    def __getitem__(self, request_id):
        return int(self._c._len_np[self._c._slot[request_id]])

    def __iter__(self):
        return iter(self._c._slot)

    def __len__(self):
        return len(self._c._slot)


def _raise_for_status(bits: int, where: str) -> None:
    if bits & N.STATUS_OOM:
        raise MemoryError(f"paged KV-cache exhausted during {where}")
    if bits & N.STATUS_DOUBLE_FREE:
        raise ValueError(f"block freed twice during {where}")
    if bits & N.STATUS_TRUNCATE_LONG:
        raise ValueError(f"truncate beyond current length during {where}")
    if bits & N.STATUS_TABLE_OVERFLOW:
        raise RuntimeError(f"block table too narrow during {where}")
    if bits & N.STATUS_BAD_BLOCK:
        raise RuntimeError(f"corrupt block id during {where}")
    if bits & N.STATUS_TIMEOUT:
        raise RuntimeError(f"a bounded device wait expired during {where}")


class BlockAllocator:
    """Device free list over ``num_blocks`` ids (engine/paged_cache.py:32-56).

    ``allocate()``/``free()`` synchronise (they return or raise); the batched
    allocation of the engine never goes through them."""

    def __init__(self, num_blocks: int, device=None, _blocks: _DeviceBlocks | None = None) -> None:
        N.load()
        self.num_blocks = num_blocks
        dev = torch.device("cuda" if device is None else device)
        self._b = _blocks if _blocks is not None else _DeviceBlocks(num_blocks, 1, 1, 1, dev)

    @property
    def num_free(self) -> int:
        return int(self._b.free_top.item())

    def free_list(self) -> list[int]:
        top = self.num_free
        return self._b.free_stack[:top].tolist()

    def _check(self, where: str) -> None:
        bits = int(self._b.status.item())
        if bits:
            self._b.status.zero_()
            _raise_for_status(bits, where)

    def allocate(self) -> int:
        N.call("pse_block_alloc_one", self._b.state, self._b.scratch_id.data_ptr(), N.stream_ptr())
        self._check("allocate")
        return int(self._b.scratch_id.item())

    def free(self, block_id: int) -> None:
        if not 0 <= block_id < self.num_blocks:
            raise ValueError(f"block {block_id} out of range")
        self._b.scratch_id.fill_(int(block_id))
        N.call("pse_block_free_one", self._b.state, self._b.scratch_id.data_ptr(), N.stream_ptr())
        bits = int(self._b.status.item())
        if bits:
            self._b.status.zero_()
            if bits & N.STATUS_DOUBLE_FREE:
                raise ValueError(f"block {block_id} freed twice")
            _raise_for_status(bits, "free")


class PagedKVCache:
    """engine/paged_cache.py:59-198 on the device.

    Extra keyword arguments (all optional): ``dtype`` (pool dtype, float32 by
    default like the reference; bfloat16 for the bf16 engine), ``device``,
    ``max_requests`` (initial slot count; grows on demand),
    ``max_blocks_per_request`` (block-table width; grows on demand) and
    ``prefix_cache`` (share the blocks of common prompt prefixes between
    requests: see ``pse.prefix_cache``; off by default, which keeps the
    reference's allocation order bit for bit).
    """

    def __init__(self, n_layers: int, n_heads: int, head_dim: int, block_size: int, num_blocks: int, *,
                 dtype: torch.dtype = torch.float32, device=None, max_requests: int = 64,
                 max_blocks_per_request: int | None = None, prefix_cache: bool = False) -> None:
        N.load()
        self.n_layers, self.n_heads, self.head_dim = n_layers, n_heads, head_dim
        self.block_size, self.num_blocks = block_size, num_blocks
        self.dtype = dtype
        self.dtype_code = N.dtype_code(dtype)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        shape = (n_layers, num_blocks, n_heads, block_size, head_dim)
        self.k_pool = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v_pool = torch.zeros(shape, dtype=dtype, device=self.device)
        width = max_blocks_per_request or max(1, min(num_blocks, 256))
        self._blocks = _DeviceBlocks(num_blocks, block_size, max(1, max_requests), width, self.device)
        self.allocator = BlockAllocator(num_blocks, self.device, _blocks=self._blocks)
        self._slot: dict[str, int] = {}
        self._free_slots = list(range(self._blocks.num_slots - 1, -1, -1))
        # host mirror of the rows' lengths, one entry per slot (the device
        # seq_len is the truth; every mutation updates both)
        self._len_np = np.zeros(self._blocks.num_slots, dtype=np.int64)
        self.slot_version = 0  # bumped whenever a request id gets or loses a slot
        self.generation = 0  # bumped whenever device buffers move (captured graphs must be rebuilt)
        self._layer_structs = [self._layer_struct(l) for l in range(n_layers)]
        # last token id of each slot (for a pending slot: the token whose
        # position is reserved and counted but whose K/V the next step's
        # verify writes), the pending slots, the call that completes them
        # (set by the speculative step) and per-slot occupancy serials
        self.last_token = torch.zeros(self._blocks.num_slots, dtype=torch.int32, device=self.device)
        self.pending_slots: set[int] = set()
        self._flusher = None
        self._serial = np.zeros(self._blocks.num_slots, dtype=np.int64)
        self.prefix = PrefixIndex(self) if prefix_cache else None

    # ------------------------------------------------------------------ internals
    def _layer_struct(self, layer: int) -> N.KVLayer:
        return N.KVLayer(self.k_pool[layer].data_ptr(), self.v_pool[layer].data_ptr(),
                         self.n_heads, self.head_dim, self.dtype_code)

    @property
    def state(self) -> N.BlockState:
        return self._blocks.state

    def layer(self, layer: int) -> N.KVLayer:
        return self._layer_structs[layer]

    @property
    def max_blocks(self) -> int:
        return self._blocks.max_blocks

    def slot(self, request_id: str) -> int:
        return self._slot[request_id]

    def slots_tensor(self, request_ids) -> torch.Tensor:
        return torch.tensor([self._slot[r] for r in request_ids], dtype=torch.int32).to(self.device, non_blocking=True)

    def _grow(self, num_slots: int, max_blocks: int) -> None:
        """Reallocate the bookkeeping with more slots / a wider table, keeping
        every row and the free list."""
        old = self._blocks
        torch.cuda.current_stream().synchronize()
        new = _DeviceBlocks.__new__(_DeviceBlocks)
        i32 = dict(dtype=torch.int32, device=self.device)
        new.num_blocks, new.block_size = old.num_blocks, old.block_size
        new.num_slots, new.max_blocks = num_slots, max_blocks
        new.block_table = torch.full((num_slots, max_blocks), -1, **i32)
        new.block_table[: old.num_slots, : old.max_blocks] = old.block_table
        new.seq_len = torch.zeros(num_slots, **i32)
        new.seq_len[: old.num_slots] = old.seq_len
        new.nblocks = torch.zeros(num_slots, **i32)
        new.nblocks[: old.num_slots] = old.nblocks
        new.free_stack, new.scalars, new.block_free = old.free_stack, old.scalars, old.block_free
        new.state = N.BlockState(
            new.block_table.data_ptr(), new.seq_len.data_ptr(), new.nblocks.data_ptr(), new.free_stack.data_ptr(),
            new.scalars.data_ptr(), new.block_free.data_ptr(), new.scalars.data_ptr() + 4,
            new.num_blocks, new.block_size, max_blocks, num_slots,
        )
        self._free_slots = list(range(num_slots - 1, old.num_slots - 1, -1)) + self._free_slots
        self._blocks = new
        self.allocator._b = new
        last = torch.zeros(num_slots, dtype=torch.int32, device=self.device)
        last[: old.num_slots] = self.last_token
        self.last_token = last
        lens = np.zeros(num_slots, dtype=np.int64)
        lens[: old.num_slots] = self._len_np
        self._len_np = lens
        ser = np.zeros(num_slots, dtype=np.int64)
        ser[: old.num_slots] = self._serial
        self._serial = ser
        self.generation += 1

    def ensure_capacity(self, request_ids, extra_tokens: int) -> None:
        """Widen the block table if a row could outgrow it by ``extra_tokens``."""
        longest = max((self.length(r) for r in request_ids), default=0)
        self.ensure_capacity_len(longest + extra_tokens)

    def ensure_capacity_len(self, tokens: int) -> None:
        """Widen the block table so a row of ``tokens`` tokens fits."""
        need = _blocks_for(tokens, self.block_size)
        if need > self._blocks.max_blocks:
            width = self._blocks.max_blocks
            while width < need:
                width *= 2
            self._grow(self._blocks.num_slots, width)

    def check_status(self, where: str) -> None:
        """Synchronise and raise the reference's exception for a latched device error."""
        bits = int(self._blocks.status.item())
        if bits:
            self._resync_lengths()
            self._blocks.status.zero_()
            _raise_for_status(bits, where)

    def status_tensor(self) -> torch.Tensor:
        return self._blocks.status

    def _resync_lengths(self) -> None:
        self._len_np[:] = self._blocks.seq_len.cpu().numpy()

    @property
    def _lengths(self) -> "_LengthView":
        """request id -> length (a read-only mapping over the per-slot mirror)."""
        return _LengthView(self)

    def slots_np(self, request_ids) -> np.ndarray:
        return np.fromiter((self._slot[r] for r in request_ids), np.int32, len(request_ids))

    def lengths_np(self, slots: np.ndarray) -> np.ndarray:
        return self._len_np[slots]

    def note_lengths(self, request_ids, lengths) -> None:
        self._len_np[self.slots_np(request_ids)] = np.asarray(lengths, dtype=np.int64)

    def note_lengths_slots(self, slots: np.ndarray, lengths: np.ndarray) -> None:
        self._len_np[slots] = lengths

    def note_append(self, request_ids, width: int) -> None:
        self._len_np[self.slots_np(request_ids)] += width

    def slot_serial(self, slot: int) -> int:
        """Occupancy serial of ``slot`` (changes whenever a request takes or leaves it)."""
        return int(self._serial[slot])

    def flush_pending(self, slots=None) -> None:
        """Complete pending slots (all of them, or those of ``slots`` that are
        pending): run the target call the speculative step deferred, which
        writes the pending token's K/V and that slot's next-token logits."""
        if not self.pending_slots:
            return
        todo = sorted(self.pending_slots if slots is None else self.pending_slots.intersection(slots))
        if todo:
            self._flusher(self, todo)

    def _flush_ids(self, request_ids) -> None:
        if self.pending_slots:
            self.flush_pending([self._slot[r] for r in request_ids if r in self._slot])

    def note_last_tokens(self, slots: torch.Tensor, ids: torch.Tensor, rows: int, width: int) -> None:
        """Record the last token id each row appended (device op, stream-ordered)."""
        self.last_token.index_copy_(0, slots.long(), ids.view(rows, width)[:, width - 1].to(torch.int32))

    # ------------------------------------------------------------------ reference API
    def create_request(self, request_id: str) -> None:
        """engine/paged_cache.py:92-96."""
        if request_id in self._slot:
            raise ValueError(f"request {request_id} already exists in this cache")
        if not self._free_slots:
            self._grow(self._blocks.num_slots * 2, self._blocks.max_blocks)
        s = self._slot[request_id] = self._free_slots.pop()
        self._len_np[s] = 0
        self._serial[s] += 1
        self.slot_version += 1
        self.pending_slots.discard(s)

    def length(self, request_id: str) -> int:
        return int(self._len_np[self._slot[request_id]])

    def num_blocks_in_use(self, request_id: str) -> int:
        return int(self._blocks.nblocks[self._slot[request_id]].item())

    def block_table(self, request_id: str) -> list[int]:
        s = self._slot[request_id]
        n = int(self._blocks.nblocks[s].item())
        return self._blocks.block_table[s, :n].tolist()

    def append(self, request_id: str, new_k, new_v) -> None:
        """engine/paged_cache.py:104-138: new_k / new_v are per-layer [n_heads, n, head_dim]."""
        self._flush_ids([request_id])
        n = int(new_k[0].shape[1])
        self.ensure_capacity([request_id], n)
        slots = torch.tensor([self._slot[request_id]], dtype=torch.int32, device=self.device)
        base = torch.empty(1, dtype=torch.int32, device=self.device)
        st = N.stream_ptr()
        N.call("pse_kv_reserve", self.state, slots.data_ptr(), 1, n, base.data_ptr(), st)
        for layer in range(self.n_layers):
            k = new_k[layer].to(device=self.device, dtype=self.dtype).contiguous()
            v = new_v[layer].to(device=self.device, dtype=self.dtype).contiguous()
            N.call("pse_kv_append", self.state, self.layer(layer), k.data_ptr(), v.data_ptr(),
                   self.head_dim, n * self.head_dim, slots.data_ptr(), base.data_ptr(), 1, n, st)
        self._len_np[self._slot[request_id]] += n
        self.check_status("append")

    def truncate(self, request_id: str, new_length: int) -> None:
        """engine/paged_cache.py:140-154."""
        self._flush_ids([request_id])
        old = self.length(request_id)
        if new_length > old:
            raise ValueError(f"truncate({new_length}) > current length {old}")
        s = self._slot[request_id]
        shared = self.prefix.shared_tokens(s) if self.prefix is not None else 0
        slots = torch.tensor([s], dtype=torch.int32).to(self.device, non_blocking=True)
        lens = torch.tensor([max(new_length, shared)], dtype=torch.int32).to(self.device, non_blocking=True)
        N.call("pse_kv_truncate", self.state, slots.data_ptr(), 1, lens.data_ptr(), None, None, N.stream_ptr())
        self._len_np[s] = max(new_length, shared)
        if new_length < shared:
            # below the shared prefix: the row's own blocks are gone; the shared
            # ones past the new length leave its table, a partly kept one is copied
            self.prefix.truncate_shared(s, new_length)

    def free_request(self, request_id: str) -> None:
        """engine/paged_cache.py:156-160."""
        s = self._slot.pop(request_id)
        self._len_np[s] = 0
        self._serial[s] += 1
        self.slot_version += 1
        self.pending_slots.discard(s)
        if self.prefix is not None:
            self.prefix.release_rows([s])
        slots = torch.tensor([s], dtype=torch.int32).to(self.device, non_blocking=True)
        N.call("pse_kv_release", self.state, slots.data_ptr(), 1, N.stream_ptr())
        self._free_slots.append(s)

    def free_requests(self, request_ids) -> None:
        """Batched free_request, rows in the given order (one launch)."""
        if not request_ids:
            return
        slots = [self._slot.pop(r) for r in request_ids]
        self._len_np[slots] = 0
        self._serial[slots] += 1
        self.slot_version += 1
        self.pending_slots.difference_update(slots)
        if self.prefix is not None:
            self.prefix.release_rows(slots)
        t = torch.tensor(slots, dtype=torch.int32).to(self.device, non_blocking=True)
        N.call("pse_kv_release", self.state, t.data_ptr(), len(slots), N.stream_ptr())
        self._free_slots.extend(slots)

    def gather(self, request_ids):
        """engine/paged_cache.py:162-198: padded per-layer [B, H, max_len, hd]
        K and V, the [B, max_len] padding mask and the [B] lengths (device tensors)."""
        self._flush_ids(request_ids)
        lengths = torch.tensor([self.length(r) for r in request_ids], dtype=torch.long)
        max_len = int(lengths.max().item()) if len(lengths) else 0
        batch = len(request_ids)
        mask = torch.arange(max_len).view(1, -1) < lengths.view(-1, 1)
        k_out, v_out = [], []
        slots = self.slots_tensor(request_ids) if batch else None
        for layer in range(self.n_layers):
            kb = torch.empty(batch, self.n_heads, max_len, self.head_dim, dtype=self.dtype, device=self.device)
            vb = torch.empty_like(kb)
            if batch and max_len:
                N.call("pse_kv_gather", self.state, self.layer(layer), slots.data_ptr(), batch, max_len,
                       kb.data_ptr(), vb.data_ptr(), N.stream_ptr())
            k_out.append(kb)
            v_out.append(vb)
        return k_out, v_out, mask.to(self.device), lengths.to(self.device)
