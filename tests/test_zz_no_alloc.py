"""The allocation-free attention entry point, pse_paged_attention_noalloc.

Some hosts of this library cannot allocate device memory where they call it
(a runtime in another language that binds only the C ABI and has no CUDA
allocator, or a process whose device memory belongs to another allocator).
For them this entry point takes its split-KV scratch from a fixed array inside
the library.  These tests call it through the C ABI on shapes that do need
scratch (several KV splits) and check, over two calls in a row, that it returns
what the workspace-taking entry point returns; and that a shape whose scratch
would not fit is refused without a launch.  This file is collected last so a
failure here never hides the other tests' results.  GPU only."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2


def _setup(rows, width, hq, hk, hd, bs, max_len, dtype, seed):
    from pse import PagedKVCache
    from pse import _native as N
    N.load()
    rng = np.random.default_rng(seed)
    base = rng.integers(max_len // 2, max_len, size=rows)
    need = [(int(b) + width + bs - 1) // bs for b in base]
    nb = sum(need) + 3
    c = PagedKVCache(n_layers=1, n_heads=hk, head_dim=hd, block_size=bs, num_blocks=nb, dtype=dtype,
                     max_requests=rows, max_blocks_per_request=max(need))
    perm = rng.permutation(nb)
    o = 0
    for i, n in enumerate(need):
        c._blocks.block_table[i, :n] = torch.tensor(perm[o:o + n].tolist(), dtype=torch.int32)
        c._blocks.nblocks[i] = n
        o += n
    g = torch.Generator().manual_seed(seed)
    c.k_pool[0].copy_(torch.randn(nb, hk, bs, hd, generator=g).to(dtype))
    c.v_pool[0].copy_(torch.randn(nb, hk, bs, hd, generator=g).to(dtype))
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    base_d = torch.tensor(base, dtype=torch.int32, device="cuda")
    return N, c, slots, base_d, int(base.max()) + width


@pytest.mark.parametrize("shape", [
    (2, 1, 8, 8, 128, 16, 20000, torch.bfloat16),   # tensor-core kernel, many splits
    (3, 4, 16, 4, 64, 32, 6000, torch.bfloat16),    # GQA, block 32
    (1, 1, 4, 4, 128, 16, 9000, torch.float32),     # generic kernel, fp32 pools
])
def test_noalloc_matches_workspace_entry_point_twice(shape):
    rows, width, hq, hk, hd, bs, max_len, dtype = shape
    N, c, slots, base_d, max_ctx = _setup(rows, width, hq, hk, hd, bs, max_len, dtype, seed=11)
    ws_bytes = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    assert 0 < ws_bytes <= N.NOALLOC_SCRATCH_BYTES  # the shape really uses scratch
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    g = torch.Generator().manual_seed(5)
    st = N.stream_ptr()
    for call in range(2):  # two calls in a row: the shared array's leftovers must not matter
        q = torch.randn(rows * width, hq * hd, generator=g).to(dtype).cuda()
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        N.call("pse_paged_attention", c.state, c.layer(0), q.data_ptr(), hq * hd, want.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx,
               None, ws.data_ptr(), ws.numel(), st)
        N.call("pse_paged_attention_noalloc", c.state, c.layer(0), q.data_ptr(), hq * hd, got.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx, st)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), call
        assert (got.float() - want.float()).abs().max().item() < tol, call
    assert int(c._blocks.status.item()) == 0


def test_noalloc_refuses_scratch_beyond_its_array():
    rows, width, hq, hk, hd, bs = 36, 8, 32, 8, 128, 16
    N, c, slots, base_d, _ = _setup(rows, width, hq, hk, hd, bs, 64, torch.bfloat16, seed=3)
    max_ctx = 4096  # a bound that asks for two KV splits of a 36-row, 32-head, width-8 call
    need = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    assert need > N.NOALLOC_SCRATCH_BYTES
    q = torch.zeros(rows * width, hq * hd, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    lib = N.load()
    rc = lib.pse_paged_attention_noalloc(c.state, c.layer(0), q.data_ptr(), hq * hd, out.data_ptr(), hq * hd,
                                         slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 0.125, max_ctx,
                                         N.stream_ptr())
    assert rc == N.PSE_ESCRATCH


def test_noalloc_prompt_shaped_call_is_not_refused_for_size():
    """A wide (prompt-shaped) call runs the prefill kernel, which uses no
    split-KV scratch: it is served even when the split-KV formula's figure for
    the same shape exceeds the array, and returns what the workspace-taking
    entry point returns, on two calls in a row."""
    rows, width, hq, hk, hd, bs = 1, 256, 32, 32, 128, 16
    N, c, slots, base_d, _ = _setup(rows, width, hq, hk, hd, bs, 600, torch.bfloat16, seed=7)
    c._blocks.seq_len[:rows] = base_d + width  # the prompt's tokens lie inside the row
    max_ctx = 1024
    need = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    assert need > N.NOALLOC_SCRATCH_BYTES
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    g = torch.Generator().manual_seed(9)
    st = N.stream_ptr()
    for call in range(2):
        q = torch.randn(rows * width, hq * hd, generator=g).to(torch.bfloat16).cuda()
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        N.call("pse_paged_attention", c.state, c.layer(0), q.data_ptr(), hq * hd, want.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx,
               None, ws.data_ptr(), ws.numel(), st)
        N.call("pse_paged_attention_noalloc", c.state, c.layer(0), q.data_ptr(), hq * hd, got.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx, st)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), call
        assert want.float().abs().max().item() > 0, call  # the rows' keys were really read
        assert (got.float() - want.float()).abs().max().item() < BF16_TOL, call
    assert int(c._blocks.status.item()) == 0
