"""Truncate churn (the commit pattern of every speculative step,
engine/speculative.py:159-164 with the appends of engine/paged_cache.py:104-138):
each step reserves k + 1 = 8 tokens on every row, truncates each row back to
its length before the step plus that row's accepted count + 1, and reserves
1 more, many steps replayed from one CUDA graph.  The device block tables,
lengths and free list must equal a CPU replay of the reference allocator's
order (oracle.alloc) bit for bit.  GPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import alloc as OA

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,bs,steps,seed", [(256, 16, 200, 0), (97, 1, 60, 1), (130, 32, 120, 2)])
def test_churn_from_a_graph_is_bit_exact(rows, bs, steps, seed):
    import pse
    import pse._native as N
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 3000, size=rows)
    nb = int(((lens + 9 * steps + bs) // bs).sum()) + 64
    maxb = int((lens.max() + 9 * steps) // bs + 2)
    c = pse.PagedKVCache(1, 1, 1, bs, nb, dtype=torch.float32, max_requests=rows, max_blocks_per_request=maxb)
    ref = OA.BlockState(nb, bs, rows, maxb)
    # rows admitted in a shuffled slot order, each with its own initial length
    order = rng.permutation(rows).astype(np.int32)
    slots = torch.from_numpy(order).cuda()
    widths = torch.from_numpy(lens[order].astype(np.int32)).cuda()
    base = torch.empty(rows, dtype=torch.int32, device="cuda")
    base2 = torch.empty(rows, dtype=torch.int32, device="cuda")
    N.call("pse_kv_reserve_rows", c.state, slots.data_ptr(), rows, widths.data_ptr(), base.data_ptr(),
           N.stream_ptr())
    ref.reserve(order, lens[order])
    acc = rng.integers(0, 8, size=(steps, rows)).astype(np.int32)
    acc_d = torch.from_numpy(acc).cuda()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with N.graph_capture(g):
        st = N.stream_ptr()
        for j in range(steps):
            N.call("pse_kv_reserve", c.state, slots.data_ptr(), rows, 8, base.data_ptr(), st)
            N.call("pse_kv_truncate", c.state, slots.data_ptr(), rows, None, base.data_ptr(),
                   acc_d[j].data_ptr(), st)
            N.call("pse_kv_reserve", c.state, slots.data_ptr(), rows, 1, base2.data_ptr(), st)
    g.replay()
    torch.cuda.synchronize()
    for j in range(steps):
        b0 = ref.reserve(order, 8)
        ref.truncate(order, b0 + acc[j])
        ref.reserve(order, 1)
    b = c._blocks
    assert int(b.status.item()) == 0 and ref.status == 0
    top = int(b.free_top.item())
    assert b.free_stack[:top].cpu().tolist() == ref.free_list()
    nbk = b.nblocks.cpu().numpy()[:rows]
    assert nbk.tolist() == ref.nblocks.tolist()
    assert b.seq_len.cpu().numpy()[:rows].tolist() == ref.seq_len.tolist()
    assert (ref.seq_len[order] == lens[order] + acc.sum(0) + steps).all()
    table = b.block_table.cpu().numpy()
    for s in range(rows):
        assert table[s, :nbk[s]].tolist() == ref.row_table(s)
    del g
