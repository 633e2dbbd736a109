"""The C ABI's host-side argument checks (include/pse.h: "checked on the host
before anything is launched"): bad sizes, missing pointers and unsupported
combinations return PSE_EINVAL / PSE_EWORKSPACE, launch nothing and leave the
cache state as it was; the Python binding turns a non-zero code into an
exception.  GPU only (the binding refuses to load without a device)."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

EINVAL, EWORKSPACE = 10001, 10002


def _setup():
    import pse
    import pse._native as N
    lib = N.load()
    c = pse.PagedKVCache(1, 2, 64, 16, 32, dtype=torch.bfloat16, max_requests=4, max_blocks_per_request=8)
    return N, lib, c


def _snapshot(c):
    b = c._blocks
    torch.cuda.synchronize()
    return (b.block_table.cpu().clone(), b.seq_len.cpu().clone(), b.nblocks.cpu().clone(),
            b.free_stack.cpu().clone(), int(b.free_top.item()), int(b.status.item()))


def _same(a, b):
    return all(torch.equal(x, y) if torch.is_tensor(x) else x == y for x, y in zip(a, b))


def test_cache_entry_points_reject_bad_arguments_and_change_nothing():
    N, lib, c = _setup()
    st = c.state
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    base = torch.empty(2, dtype=torch.int32, device="cuda")
    widths = torch.tensor([3, 4], dtype=torch.int32, device="cuda")
    before = _snapshot(c)
    assert lib.pse_kv_reserve(st, slots.data_ptr(), -1, 4, base.data_ptr(), None) == EINVAL
    assert lib.pse_kv_reserve(st, slots.data_ptr(), 2, -1, base.data_ptr(), None) == EINVAL
    assert lib.pse_kv_reserve(st, None, 2, 4, base.data_ptr(), None) == EINVAL
    assert lib.pse_kv_reserve_rows(st, slots.data_ptr(), 2, None, base.data_ptr(), None) == EINVAL
    assert lib.pse_kv_truncate(st, slots.data_ptr(), 2, None, None, None, None) == EINVAL
    assert lib.pse_kv_release(st, None, 1, None) == EINVAL
    assert lib.pse_block_alloc_one(st, None, None) == EINVAL
    assert lib.pse_block_free_one(st, None, None) == EINVAL
    bad = N.BlockState.from_buffer_copy(st)
    bad.block_size = 0
    assert lib.pse_block_init(bad, None) == EINVAL
    assert lib.pse_kv_reserve_rows(bad, slots.data_ptr(), 2, widths.data_ptr(), base.data_ptr(), None) == EINVAL
    assert _same(before, _snapshot(c))
    # zero rows is a valid no-op
    assert lib.pse_kv_reserve(st, None, 0, 4, None, None) == 0
    assert lib.pse_kv_release(st, None, 0, None) == 0
    assert _same(before, _snapshot(c))
    with pytest.raises(RuntimeError, match=str(EINVAL)):
        N.call("pse_kv_reserve", st, slots.data_ptr(), -1, 4, base.data_ptr(), N.stream_ptr())


def test_attention_rejects_bad_shapes_and_short_workspaces():
    N, lib, c = _setup()
    st, kv = c.state, c.layer(0)
    rows, width, hq = 2, 1, 4
    q = torch.zeros(rows * width, hq * 64, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    base = torch.zeros(2, dtype=torch.int32, device="cuda")
    need = N.size_call("pse_paged_attention_workspace", rows, width, hq, 2, 64, 16)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")

    def attn(rows_=rows, q_heads=hq, max_ctx=16, wsp=ws.data_ptr(), wsb=ws.numel(), qp=q.data_ptr()):
        return lib.pse_paged_attention(st, kv, qp, hq * 64, out.data_ptr(), hq * 64, slots.data_ptr(),
                                       base.data_ptr(), rows_, width, q_heads, 0.125, max_ctx, None, wsp, wsb, None)

    assert attn(rows_=-1) == EINVAL
    assert attn(q_heads=3) == EINVAL            # not a multiple of the 2 KV heads
    assert attn(max_ctx=0) == EINVAL
    assert attn(qp=None) == EINVAL
    assert attn(wsp=None) == EWORKSPACE
    assert attn(wsb=need - 1) == EWORKSPACE if need > 0 else True
    assert attn(rows_=0) == 0                   # nothing to do
    big = N.KVLayer.from_buffer_copy(kv)
    big.head_dim = 512
    assert lib.pse_paged_attention(st, big, q.data_ptr(), hq * 64, out.data_ptr(), hq * 64, slots.data_ptr(),
                                   base.data_ptr(), rows, width, hq, 0.125, 16, None, ws.data_ptr(), ws.numel(),
                                   None) == EINVAL
    torch.cuda.synchronize()
    assert not out.any()  # nothing was launched


def test_sampling_and_model_ops_reject_bad_arguments():
    N, lib, _ = _setup()
    logits = torch.zeros(2, 8, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    keys = torch.zeros(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(2, 3, dtype=torch.float64, device="cuda")
    assert lib.pse_sample_tokens(logits.data_ptr(), 8, None, 2, 0, 0.0, None, 0, 0, out.data_ptr(), 1,
                                 None, 0, None) == EINVAL          # empty vocabulary
    assert lib.pse_sample_tokens(logits.data_ptr(), 8, None, 2, 8, 1.0, None, 0, 0, out.data_ptr(), 1,
                                 None, 0, None) == EINVAL          # T > 0 without uniforms
    assert lib.pse_philox_uniforms(1, keys.data_ptr(), keys.data_ptr(), -1, 3, u.data_ptr(), None) == EINVAL
    i32 = out.data_ptr()
    assert lib.pse_spec_accept(logits.data_ptr(), 8, None, logits.data_ptr(), 8, 8, None, 0, None, None, 0, 0,
                               i32, None, 0, 2, 0, 8, 0.0, i32, i32, i32, None) == EINVAL   # k = 0
    assert lib.pse_spec_accept(logits.data_ptr(), 8, None, logits.data_ptr(), 8, 8, None, 0, None, None, 0, 0,
                               i32, None, 0, 2, 2, 8, 1.0, i32, i32, i32, None) == EINVAL   # T > 0, no draft / u
    x = torch.zeros(2, 8, device="cuda")
    h = torch.zeros(2, 8, dtype=torch.bfloat16, device="cuda")
    assert lib.pse_add_norm(x.data_ptr(), 8, None, 0, None, 1, h.data_ptr(), None, 1, 2, 5000, 1e-5, 0,
                            h.data_ptr(), 8, 1, None) == EINVAL                        # d > 4096
    assert lib.pse_add_norm(x.data_ptr(), 8, None, 0, None, 0, h.data_ptr(), None, 1, 2, 8, 1e-5, 0,
                            h.data_ptr(), 8, 1, None) == EINVAL                        # mixed dtypes
    assert lib.pse_epilogue(3, h.data_ptr(), 8, None, None, 0, None, 0, 2, 8, 1, None) == EINVAL
    assert lib.pse_epilogue(2, h.data_ptr(), 8, None, None, 0, None, 0, 2, 4, 1, None) == EINVAL  # no y2
    assert lib.pse_rope(h.data_ptr(), 8, 2, 1, 1, 1, 7, keys.data_ptr(), 10000.0, 1, None) == EINVAL  # odd dim
    assert lib.pse_embed(keys.data_ptr(), keys.data_ptr(), 2, 1, h.data_ptr(), None, 0, 1, 8, 0,
                         x.data_ptr(), None) == EINVAL                                 # d = 0
    assert lib.pse_accept_select(4) == EINVAL and lib.pse_accept_select(-1) == EINVAL
    assert lib.pse_accept_select(0) == 0
    torch.cuda.synchronize()
    assert not out.any() and not x.any()
