"""Wide (prefill-shaped) paged attention on the tcgen05 kernel: every call
with at least 64 query rows per (row, KV head) on bf16 pools.  Checked against
the oracle (float64 restatement of engine/model.py:99-116 over the paged
layout) within the bf16 tolerance, against the mma.sync kernel the same calls
took before, and for the rows past a row's length (padding of a
length-grouped prefill) which must come out zero.  GPU only."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle.attention import paged_attention as oracle_attention

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2

CASES = [
    # rows, width, q_heads, kv_heads, head_dim, block_size, max_base
    (2, 200, 12, 12, 64, 16, 300),   # GPT-2-shaped heads, keys over several 128-key tiles
    (2, 160, 32, 8, 64, 32, 500),    # GQA 4: 640 query rows = 5 tiles
    (1, 300, 8, 8, 128, 16, 0),      # head_dim 128, prompt from position 0
    (3, 100, 16, 4, 128, 32, 1000),  # head_dim 128, GQA 4, long context before the prompt
    (2, 130, 4, 4, 64, 64, 200),     # block 64, a query tile of 2 rows
    (2, 70, 2, 2, 64, 128, 150),     # block 128 (one page per key tile)
    (1, 64, 1, 1, 64, 16, 0),        # exactly 64 query rows: the smallest call routed here
    (4, 33, 8, 2, 64, 16, 90),       # GQA 4 x width 33 = 132 rows: one full tile, one of 4 rows
    (2, 40, 16, 2, 64, 16, 100),     # GQA 8: 16 tokens per tile, last tile 8 tokens
    (1, 20, 32, 2, 128, 32, 50),     # GQA 16: 8 tokens per tile
    (1, 10, 64, 2, 64, 16, 50),      # GQA 32: not served by the tcgen05 kernel (falls back)
]


def _N():
    import pse._native as N
    N.load()
    return N


def _run(case, seed, ragged=False, select=0):
    import pse
    N = _N()
    rows, width, hq, hk, hd, bs, max_base = case
    rng = np.random.default_rng(seed)
    base = rng.integers(0, max_base + 1, size=rows)
    # ragged: a row holds only its first P_i <= width tokens (prefill of a
    # length-grouped batch padded to the longest prompt); the rest is padding
    plen = rng.integers(max(1, width // 3), width + 1, size=rows) if ragged else np.full(rows, width)
    seq = base + plen
    need = [(int(s) + bs - 1) // bs for s in seq]
    nb = sum(need) + 3
    c = pse.PagedKVCache(1, hk, hd, bs, nb, dtype=torch.bfloat16, max_requests=rows,
                         max_blocks_per_request=max(need))
    perm = rng.permutation(nb)
    tables, o = [], 0
    for i, n in enumerate(need):
        tables.append(perm[o:o + n].tolist())
        o += n
        c._blocks.block_table[i, :n] = torch.tensor(tables[-1], dtype=torch.int32)
        c._blocks.nblocks[i] = n
        c._blocks.seq_len[i] = int(seq[i])
    g = torch.Generator().manual_seed(seed + 1)
    kp = torch.randn(nb, hk, bs, hd, generator=g).to(torch.bfloat16)
    vp = torch.randn(nb, hk, bs, hd, generator=g).to(torch.bfloat16)
    c.k_pool[0].copy_(kp)
    c.v_pool[0].copy_(vp)
    q = torch.randn(rows * width, hq * hd, generator=g).to(torch.bfloat16)
    qd = q.cuda()
    out = torch.full_like(qd, float("nan"))
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    base_d = torch.tensor(base, dtype=torch.int32, device="cuda")
    max_ctx = int((base + width).max())
    ws_bytes = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    N.call("pse_attention_prefill_select", select)
    try:
        N.call("pse_paged_attention", c.state, c.layer(0), qd.data_ptr(), hq * hd, out.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx,
               None, ws.data_ptr(), ws.numel(), N.stream_ptr())
        torch.cuda.synchronize()
    finally:
        N.call("pse_attention_prefill_select", 0)
    assert int(c._blocks.status.item()) == 0
    got = out.float().cpu().view(rows, width, hq, hd).numpy()
    return got, q, kp, vp, tables, base, plen


@pytest.mark.parametrize("case", CASES)
def test_prefill_attention_matches_oracle(case):
    got, q, kp, vp, tables, base, _ = _run(case, seed=CASES.index(case))
    rows, width, hq, hk, hd, bs, _ = case
    want = oracle_attention(q.float().view(rows, width, hq, hd).numpy(), kp.float().numpy(), vp.float().numpy(),
                            tables, base)
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() < BF16_TOL


@pytest.mark.parametrize("case", CASES[:4])
def test_prefill_attention_padding_rows_are_zero(case):
    """Rows past the row's length get zero output; rows before it match the
    oracle, whose keys never reach past the length."""
    got, q, kp, vp, tables, base, plen = _run(case, seed=100 + CASES.index(case), ragged=True)
    rows, width, hq, hk, hd, bs, _ = case
    want = oracle_attention(q.float().view(rows, width, hq, hd).numpy(), kp.float().numpy(), vp.float().numpy(),
                            [t + [t[-1]] * 64 for t in tables], base)
    for i in range(rows):
        p = int(plen[i])
        assert np.abs(got[i, :p] - want[i, :p]).max() < BF16_TOL, i
        assert (got[i, p:] == 0).all(), i


@pytest.mark.parametrize("case", CASES[:3])
def test_prefill_attention_matches_previous_kernel(case):
    new = _run(case, seed=7)[0]
    old = _run(case, seed=7, select=1)[0]
    assert np.abs(new - old).max() < BF16_TOL


@pytest.mark.parametrize("case", [c for c in CASES if c[4] == 64])
def test_pair_and_single_tile_kernels_agree(case):
    """head_dim 64 runs two query tiles per CTA by default; the one-tile kernel
    (mode 2) must give the same rows, padding included."""
    pair = _run(case, seed=11, ragged=True)
    single = _run(case, seed=11, ragged=True, select=2)
    assert np.abs(pair[0] - single[0]).max() < BF16_TOL
    assert ((pair[0] == 0) == (single[0] == 0)).all()


def test_prefill_select_rejects_unknown_mode():
    N = _N()
    assert N.load().pse_attention_prefill_select(3) != 0
    assert N.load().pse_attention_prefill_select(-1) != 0
