"""Target next-token logits whose computation is deferred to the next step.

The reference's step ends with a width-1 target call over each row's final
token (engine/speculative.py:166-177) whose only product the scheduler uses is
``target_next_logits``, and the scheduler only ever hands those back to the
next step (engine/scheduler.py:100-113), which tests the first draft against
them (speculative.py:128-130).  The device step therefore skips that call:
the final token's position is reserved in the target cache exactly where the
reference's bonus append puts it (same block tables, lengths and free list),
its K/V is written by the next step's verify, which runs at width k+1 with
that token in column 0, and column 0's logits are the ``target_next_logits``
the reference would have returned.

What the step returns for such a row is a ``PendingLogits``: a tensor view of
the row's per-slot logits buffer that computes its values the first time
anything reads them.  Passing it back to the next step unchanged (as the
scheduler does) costs nothing; any torch operation on it (indexing, ``argmax``,
``.cpu()``, printing, arithmetic) first runs the skipped target call for every
pending row of that cache -- the same call the reference makes -- and then
proceeds on the real values.  Metadata (``shape``, ``dtype``, ``device``,
``data_ptr`` ...) is available without that.  Like every next-logits view the
step returns, it is overwritten by the next step of the same request; reading
it after its request was freed raises ``RuntimeError`` (the K/V it would need
is gone).
"""
from __future__ import annotations

import torch

# metadata that does not depend on the values: never triggers the deferred call
_META_GETTERS = frozenset({"shape", "dtype", "device", "ndim", "is_cuda", "requires_grad", "layout", "is_sparse",
                           "is_quantized", "is_meta", "grad_fn", "names", "itemsize", "nbytes"})
_META_METHODS = frozenset({"data_ptr", "numel", "dim", "size", "stride", "element_size", "__len__", "is_contiguous",
                           "storage_offset", "nelement", "get_device", "is_floating_point", "is_complex"})


def _is_meta(func) -> bool:
    name = getattr(func, "__name__", "")
    if name == "__get__":
        return getattr(getattr(func, "__self__", None), "__name__", "") in _META_GETTERS
    return name in _META_METHODS


def _collect(obj, out: list) -> None:
    if isinstance(obj, PendingLogits):
        out.append(obj)
    elif isinstance(obj, (list, tuple)):
        for o in obj:
            _collect(o, out)
    elif isinstance(obj, dict):
        for o in obj.values():
            _collect(o, out)


class PendingLogits(torch.Tensor):
    """A row of a target cache's next-logits buffer whose values may still be
    owed by a deferred target call (see the module docstring).  Instances are
    made by ``pending_view`` only."""

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if not _is_meta(func):
            found: list = []
            _collect(args, found)
            _collect(kwargs, found)
            for p in found:
                p._pse_materialize()
        with torch._C.DisableTorchFunctionSubclass():
            return func(*args, **kwargs)

    def _pse_materialize(self) -> None:
        cache, slot, serial = self.__dict__["_pse_owner"]
        if cache.slot_serial(slot) != serial:
            raise RuntimeError("these target logits belonged to a request that was freed before they were read; "
                               "read deferred logits before freeing the request")
        if slot in cache.pending_slots:
            cache.flush_pending()


def pending_view(row: torch.Tensor, cache, slot: int) -> PendingLogits:
    """``row`` (a view of ``cache``'s next-logits buffer for ``slot``) as a
    PendingLogits bound to the slot's current occupant."""
    p = row.as_subclass(PendingLogits)
    p.__dict__["_pse_owner"] = (cache, slot, cache.slot_serial(slot))
    return p
