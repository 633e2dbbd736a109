"""Kernel parity against the CPU oracle through the C ABI (libpse.so).

Integer work (free list, block tables, Philox, token choices) must match bit
for bit; floating-point outputs within the stated tolerances (1e-4 abs in
fp32, 2e-2 abs in bf16).  GPU only."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import alloc as OA
from oracle.accept import accept_row
from oracle.attention import paged_attention as oracle_attention
from oracle.philox import request_key, step_uniforms
from oracle.sampling import inverse_cdf, sample_with_uniform, weights

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2


def _N():
    from pse import _native as N
    N.load()
    return N


def _cache(**kw):
    from pse import PagedKVCache
    return PagedKVCache(**kw)


# ---------------------------------------------------------------- free list / tables
def _device_snapshot(cache):
    b = cache._blocks
    top = int(b.free_top.item())
    return (b.block_table.cpu().numpy(), b.nblocks.cpu().numpy(), b.seq_len.cpu().numpy(),
            b.free_stack[:top].cpu().numpy(), int(b.status.item()))


@pytest.mark.parametrize("seed", range(6))
def test_batched_reserve_truncate_release_bit_exact(seed):
    N = _N()
    rng = np.random.default_rng(seed)
    nb, bs, slots_n, width = int(rng.integers(8, 200)), int(rng.integers(1, 17)), 12, 64
    c = _cache(n_layers=1, n_heads=1, head_dim=2, block_size=bs, num_blocks=nb, max_requests=slots_n,
               max_blocks_per_request=width)
    ref = OA.BlockState(nb, bs, slots_n, width)
    live: list[int] = []
    st = N.stream_ptr()
    for _ in range(60):
        op = rng.choice(["reserve", "truncate", "release"], p=[0.5, 0.35, 0.15])
        if op == "reserve" or not live:
            free = [s for s in range(slots_n) if s not in live]
            pick = list(rng.choice(free, size=min(len(free), int(rng.integers(1, 5))), replace=False)) if free else []
            rows = [int(x) for x in pick] + ([int(x) for x in rng.choice(live, size=min(len(live), 3),
                                                                         replace=False)] if live else [])
            rng.shuffle(rows)
            ragged = bool(rng.integers(0, 2))  # pse_kv_reserve_rows: one width per row
            w = rng.integers(0, 12, size=len(rows)) if ragged else int(rng.integers(1, 12))
            if any((ref.seq_len[s] + ww + bs - 1) // bs > width for s, ww in zip(rows, np.broadcast_to(w, len(rows)))):
                continue
            ref.status = 0
            base_ref = ref.reserve(rows, w)
            slots = torch.tensor(rows, dtype=torch.int32, device="cuda")
            base = torch.empty(len(rows), dtype=torch.int32, device="cuda")
            if ragged:
                wd = torch.tensor(w.tolist(), dtype=torch.int32, device="cuda")
                N.call("pse_kv_reserve_rows", c.state, slots.data_ptr(), len(rows), wd.data_ptr(), base.data_ptr(), st)
            else:
                N.call("pse_kv_reserve", c.state, slots.data_ptr(), len(rows), w, base.data_ptr(), st)
            assert base.cpu().tolist() == base_ref.tolist()
            for s in rows:
                if s not in live:
                    live.append(s)
        elif op == "truncate":
            rows = [int(x) for x in rng.choice(live, size=min(len(live), int(rng.integers(1, 5))), replace=False)]
            new = [int(rng.integers(0, ref.seq_len[s] + 1)) for s in rows]
            ref.truncate(rows, new)
            slots = torch.tensor(rows, dtype=torch.int32, device="cuda")
            nl = torch.tensor(new, dtype=torch.int32, device="cuda")
            N.call("pse_kv_truncate", c.state, slots.data_ptr(), len(rows), nl.data_ptr(), None, None, st)
        else:
            rows = [int(x) for x in rng.choice(live, size=min(len(live), 2), replace=False)]
            ref.release(rows)
            slots = torch.tensor(rows, dtype=torch.int32, device="cuda")
            N.call("pse_kv_release", c.state, slots.data_ptr(), len(rows), st)
            live = [s for s in live if s not in rows]
        table, nbk, lens, stack, status = _device_snapshot(c)
        assert status == ref.status
        if status:
            c._blocks.status.zero_()
            ref.status = 0
        assert stack.tolist() == ref.free_list()
        assert nbk.tolist() == ref.nblocks.tolist()
        assert lens.tolist() == ref.seq_len.tolist()
        for s in range(slots_n):
            assert table[s, : nbk[s]].tolist() == ref.row_table(s)


def test_truncate_from_step_form_and_error_latch():
    N = _N()
    c = _cache(n_layers=1, n_heads=1, head_dim=2, block_size=4, num_blocks=16, max_requests=4)
    st = N.stream_ptr()
    slots = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    base = torch.empty(3, dtype=torch.int32, device="cuda")
    N.call("pse_kv_reserve", c.state, slots.data_ptr(), 3, 9, base.data_ptr(), st)
    acc = torch.tensor([0, 5, 9], dtype=torch.int32, device="cuda")
    base0 = torch.zeros(3, dtype=torch.int32, device="cuda")
    N.call("pse_kv_truncate", c.state, slots.data_ptr(), 3, None, base0.data_ptr(), acc.data_ptr(), st)
    assert c._blocks.seq_len[:3].tolist() == [0, 5, 9]
    assert c._blocks.nblocks[:3].tolist() == [0, 2, 3]
    # truncate beyond length latches the error; later mutations are no-ops until cleared
    bad = torch.tensor([7], dtype=torch.int32, device="cuda")
    N.call("pse_kv_truncate", c.state, slots[1:2].data_ptr(), 1, bad.data_ptr(), None, None, st)
    assert int(c._blocks.status.item()) & N.STATUS_TRUNCATE_LONG
    before = c._blocks.free_top.item()
    N.call("pse_kv_release", c.state, slots.data_ptr(), 3, st)
    assert c._blocks.free_top.item() == before
    c._blocks.status.zero_()


def test_reserve_exhaustion_matches_reference_partial_state():
    N = _N()
    c = _cache(n_layers=1, n_heads=1, head_dim=2, block_size=2, num_blocks=5, max_requests=4,
               max_blocks_per_request=8)
    ref = OA.BlockState(5, 2, 4, 8)
    st = N.stream_ptr()
    rows = [2, 0, 3]
    base = torch.empty(3, dtype=torch.int32, device="cuda")
    slots = torch.tensor(rows, dtype=torch.int32, device="cuda")
    N.call("pse_kv_reserve", c.state, slots.data_ptr(), 3, 4, base.data_ptr(), st)
    ref.reserve(rows, 4)
    table, nbk, lens, stack, status = _device_snapshot(c)
    assert status == ref.status == OA.OOM
    assert nbk.tolist() == ref.nblocks.tolist() and lens.tolist() == ref.seq_len.tolist()
    assert stack.tolist() == ref.free_list()
    c._blocks.status.zero_()


# ---------------------------------------------------------------- append / gather
def test_append_then_gather_roundtrip_bf16_and_f32():
    for dtype in (torch.float32, torch.bfloat16):
        c = _cache(n_layers=2, n_heads=3, head_dim=64, block_size=16, num_blocks=64, dtype=dtype)
        rng = torch.Generator().manual_seed(3)
        truth = {}
        for r, n in (("a", 5), ("b", 40), ("a", 17), ("c", 1), ("b", 3)):
            if r not in truth:
                c.create_request(r)
                truth[r] = [[], []]
            k = [torch.randn(3, n, 64, generator=rng).to(dtype) for _ in range(2)]
            v = [torch.randn(3, n, 64, generator=rng).to(dtype) for _ in range(2)]
            c.append(r, k, v)
            truth[r][0].append(k)
            truth[r][1].append(v)
        ko, vo, mask, lens = c.gather(["a", "b", "c"])
        for i, r in enumerate(["a", "b", "c"]):
            for layer in range(2):
                kk = torch.cat([t[layer] for t in truth[r][0]], dim=1)
                vv = torch.cat([t[layer] for t in truth[r][1]], dim=1)
                n = kk.shape[1]
                assert torch.equal(ko[layer][i, :, :n].cpu(), kk)
                assert torch.equal(vo[layer][i, :, :n].cpu(), vv)
                assert not ko[layer][i, :, n:].any()


# ---------------------------------------------------------------- paged attention
ATTN_CASES = [
    # rows, width, q_heads, kv_heads, head_dim, block_size, max_len, dtype
    (3, 1, 2, 2, 4, 4, 30, torch.float32),
    (4, 3, 2, 2, 6, 3, 25, torch.float32),
    (5, 5, 4, 4, 32, 16, 200, torch.float32),
    (2, 9, 2, 2, 8, 1, 40, torch.float32),
    (6, 1, 12, 12, 64, 16, 700, torch.bfloat16),
    (6, 6, 12, 12, 64, 16, 700, torch.bfloat16),
    (3, 8, 32, 8, 128, 16, 900, torch.bfloat16),
    (2, 4, 32, 8, 64, 32, 3000, torch.bfloat16),   # long context: split-KV path
    (1, 1, 4, 4, 128, 16, 9000, torch.float32),    # single row, many splits
    (1, 37, 2, 2, 16, 4, 60, torch.float32),       # prefill-like width, several query tiles
    (1, 40, 4, 4, 64, 16, 50, torch.bfloat16),     # prefill-like width on the tensor-core path (64-row items)
    (3, 23, 8, 2, 64, 32, 400, torch.bfloat16),    # GQA 4 x width 23 = 92 rows: two 64-row items, one padded
    (2, 33, 4, 4, 64, 16, 3000, torch.bfloat16),   # 33 rows just past a 32-row item, long context, splits
    (4, 1, 6, 6, 64, 64, 500, torch.bfloat16),     # block 64
    (2, 5, 12, 12, 64, 32, 2100, torch.bfloat16),  # block 32, splits
    (5, 6, 16, 4, 128, 16, 300, torch.bfloat16),   # GQA 4 x width 6 = 24 rows (two m-tiles, one padded)
    (2, 1, 8, 8, 128, 16, 20000, torch.bfloat16),  # very long context, many splits
]


@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("case", ATTN_CASES)
def test_paged_attention_matches_oracle(case, generic):
    N = _N()
    rows, width, hq, hk, hd, bs, max_len, dtype = case
    if generic and dtype == torch.float32:
        pytest.skip("fp32 pools always run the generic kernel")
    rng = np.random.default_rng(ATTN_CASES.index(case))
    base = rng.integers(0, max_len, size=rows)
    need = [(int(b) + width + bs - 1) // bs for b in base]
    nb = sum(need) + 5
    c = _cache(n_layers=1, n_heads=hk, head_dim=hd, block_size=bs, num_blocks=nb, dtype=dtype,
               max_requests=rows, max_blocks_per_request=max(need))
    perm = rng.permutation(nb)
    tables, o = [], 0
    for i, n in enumerate(need):
        tables.append(perm[o:o + n].tolist())
        o += n
        c._blocks.block_table[i, :n] = torch.tensor(tables[-1], dtype=torch.int32)
        c._blocks.nblocks[i] = n
        c._blocks.seq_len[i] = int(base[i]) + width
    g = torch.Generator().manual_seed(7)
    kp = torch.randn(nb, hk, bs, hd, generator=g)
    vp = torch.randn(nb, hk, bs, hd, generator=g)
    c.k_pool[0].copy_(kp.to(dtype))
    c.v_pool[0].copy_(vp.to(dtype))
    q = torch.randn(rows * width, hq * hd, generator=g).to(dtype)
    qd = q.cuda()
    out = torch.empty_like(qd)
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    base_d = torch.tensor(base, dtype=torch.int32, device="cuda")
    max_ctx = int(base.max()) + width
    ws_bytes = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    N.call("pse_attention_force_generic", 1 if generic else 0)
    try:
        # rows handed out longest-first (any permutation gives the same result)
        order = torch.from_numpy(np.argsort(-base, kind="stable").astype(np.int32)).cuda()
        N.call("pse_paged_attention", c.state, c.layer(0), qd.data_ptr(), hq * hd, out.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx,
               order.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_ptr())
        torch.cuda.synchronize()
    finally:
        N.call("pse_attention_force_generic", 0)
    assert int(c._blocks.status.item()) == 0
    want = oracle_attention(q.float().view(rows, width, hq, hd).numpy(), kp.to(dtype).float().numpy(),
                            vp.to(dtype).float().numpy(), tables, base)
    got = out.float().cpu().view(rows, width, hq, hd).numpy()
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert np.abs(got - want).max() < tol


TREE_ATTN_CASES = [
    # rows, branches, depth0, width, q_heads, kv_heads, head_dim, block_size, max_root, dtype
    (4, 2, 0, 8, 12, 12, 64, 16, 700, torch.bfloat16),     # verify of 2 x 4 nodes
    (4, 3, 2, 3, 12, 12, 64, 16, 700, torch.bfloat16),     # a draft call at depth 2
    (3, 4, 0, 16, 32, 8, 128, 16, 900, torch.bfloat16),    # GQA 4 x 16 nodes = 64 query rows
    (2, 4, 0, 20, 12, 12, 64, 32, 3000, torch.bfloat16),   # long root context: split-KV
    (3, 2, 0, 6, 4, 4, 8, 4, 50, torch.float32),
    (2, 2, 1, 2, 2, 2, 16, 3, 40, torch.float32),
    (2, 1, 0, 5, 4, 4, 16, 4, 30, torch.float32),          # one branch: the causal rule
]


@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("case", TREE_ATTN_CASES)
def test_paged_attention_tree_matches_oracle(case, generic):
    """pse_paged_attention_tree: each token-tree node sees the root context and
    its own branch, against the oracle's attention under the same mask."""
    N = _N()
    rows, b, d0, width, hq, hk, hd, bs, max_root, dtype = case
    if generic and dtype == torch.float32:
        pytest.skip("fp32 pools always run the generic kernel")
    rng = np.random.default_rng(100 + TREE_ATTN_CASES.index(case))
    root = rng.integers(1, max_root, size=rows)
    base = root + d0 * b
    need = [(int(x) + width + bs - 1) // bs for x in base]
    nb = sum(need) + 5
    c = _cache(n_layers=1, n_heads=hk, head_dim=hd, block_size=bs, num_blocks=nb, dtype=dtype,
               max_requests=rows, max_blocks_per_request=max(need))
    perm = rng.permutation(nb)
    tables, o = [], 0
    for i, n in enumerate(need):
        tables.append(perm[o:o + n].tolist())
        o += n
        c._blocks.block_table[i, :n] = torch.tensor(tables[-1], dtype=torch.int32)
        c._blocks.nblocks[i] = n
        c._blocks.seq_len[i] = int(base[i]) + width
    g = torch.Generator().manual_seed(11)
    kp = torch.randn(nb, hk, bs, hd, generator=g)
    vp = torch.randn(nb, hk, bs, hd, generator=g)
    c.k_pool[0].copy_(kp.to(dtype))
    c.v_pool[0].copy_(vp.to(dtype))
    q = torch.randn(rows * width, hq * hd, generator=g).to(dtype)
    qd = q.cuda()
    out = torch.empty_like(qd)
    slots = torch.arange(rows, dtype=torch.int32, device="cuda")
    base_d = torch.tensor(base, dtype=torch.int32, device="cuda")
    max_ctx = int(base.max()) + width
    ws_bytes = N.size_call("pse_paged_attention_workspace", rows, width, hq, hk, hd, max_ctx)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    N.call("pse_attention_force_generic", 1 if generic else 0)
    try:
        N.call("pse_paged_attention_tree", c.state, c.layer(0), qd.data_ptr(), hq * hd, out.data_ptr(), hq * hd,
               slots.data_ptr(), base_d.data_ptr(), rows, width, hq, 1.0 / math.sqrt(hd), max_ctx, None,
               ws.data_ptr(), ws.numel(), b, d0, N.stream_ptr())
        torch.cuda.synchronize()
    finally:
        N.call("pse_attention_force_generic", 0)
    assert int(c._blocks.status.item()) == 0
    want = oracle_attention(q.float().view(rows, width, hq, hd).numpy(), kp.to(dtype).float().numpy(),
                            vp.to(dtype).float().numpy(), tables, base, tree=(b, d0))
    got = out.float().cpu().view(rows, width, hq, hd).numpy()
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert np.abs(got - want).max() < tol


def test_kv_compact_moves_the_kept_nodes():
    """pse_kv_compact: per row, the tokens at root + src[m] land at root + m,
    the rest of the row untouched (fp32 and bf16 pools)."""
    N = _N()
    for dtype in (torch.float32, torch.bfloat16):
        rows, hk, hd, bs, k = 3, 2, 8, 4, 4
        c = _cache(n_layers=1, n_heads=hk, head_dim=hd, block_size=bs, num_blocks=40, dtype=dtype,
                   max_requests=rows, max_blocks_per_request=10)
        root = np.array([5, 0, 9])
        b = 3
        for i in range(rows):
            n = (int(root[i]) + b * k + bs - 1) // bs
            c._blocks.block_table[i, :n] = torch.arange(i * 12, i * 12 + n, dtype=torch.int32)
            c._blocks.nblocks[i] = n
            c._blocks.seq_len[i] = int(root[i]) + b * k
        c.k_pool.copy_(torch.randn_like(c.k_pool, dtype=torch.float32).to(dtype))
        c.v_pool.copy_(torch.randn_like(c.v_pool, dtype=torch.float32).to(dtype))
        before_k = c.k_pool.clone()
        before_v = c.v_pool.clone()
        branch = np.array([2, 0, 1])
        n_keep = np.array([3, 0, 4])
        src = (np.arange(k)[None, :] * b + branch[:, None]).astype(np.int32)
        # device arrays held in names until the launch is queued
        slots_d = torch.arange(rows, dtype=torch.int32).cuda()
        root_d = torch.tensor(root, dtype=torch.int32).cuda()
        src_d = torch.from_numpy(src).cuda()
        keep_d = torch.tensor(n_keep, dtype=torch.int32).cuda()
        N.call("pse_kv_compact", c.state, c.layer(0), slots_d.data_ptr(), root_d.data_ptr(), src_d.data_ptr(),
               keep_d.data_ptr(), rows, k, N.stream_ptr())
        torch.cuda.synchronize()
        assert int(c._blocks.status.item()) == 0

        def tok(pool, i, p):
            blk = int(c._blocks.block_table[i, p // bs])
            return pool[0, blk, :, p % bs]

        for i in range(rows):
            for p in range(int(root[i]) + b * k):
                m = p - int(root[i])
                if 0 <= m < n_keep[i]:
                    want_k = tok(before_k, i, int(root[i]) + int(src[i, m]))
                    want_v = tok(before_v, i, int(root[i]) + int(src[i, m]))
                else:
                    want_k, want_v = tok(before_k, i, p), tok(before_v, i, p)
                assert torch.equal(tok(c.k_pool, i, p), want_k) and torch.equal(tok(c.v_pool, i, p), want_v)


# ---------------------------------------------------------------- Philox, sampling, accept
def test_philox_uniforms_bit_exact():
    N = _N()
    keys = [request_key(f"r{i}") for i in range(37)]
    steps = list(range(5, 42))
    want = step_uniforms(0xDEADBEEF12345, keys, steps, 11)
    kd = torch.from_numpy(np.array(keys, dtype=np.uint32).view(np.int32)).cuda()
    sd = torch.tensor(steps, dtype=torch.int32, device="cuda")
    out = torch.empty(37, 11, dtype=torch.float64, device="cuda")
    N.call("pse_philox_uniforms", 0xDEADBEEF12345, kd.data_ptr(), sd.data_ptr(), 37, 11, out.data_ptr(),
           N.stream_ptr())
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("kern", [0, 1])
@pytest.mark.parametrize("vocab,temp", [(257, 0.0), (257, 1.0), (256, 1.0), (32000, 0.7), (128256, 1.0),
                                        (13, 1.0)])
def test_sample_tokens_matches_oracle(vocab, temp, kern):
    N = _N()
    rows = 48
    g = torch.Generator().manual_seed(vocab)
    logits = torch.randn(rows, vocab, generator=g) * 3
    logits[0, 5] = logits[0, 9] = logits[0].max() + 1  # greedy tie -> lowest index
    u = torch.rand(rows, 3, generator=g, dtype=torch.float64)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    ld, ud = logits.cuda(), u.cuda()
    N.load().pse_accept_select(2 * kern)  # 0: streaming sampler (vocab % 4 == 0), 2: the scalar one
    try:
        N.call("pse_sample_tokens", ld.data_ptr(), vocab, None, rows, vocab, temp, ud.data_ptr(), 3, 1,
               out.data_ptr(), 1, None, 0, N.stream_ptr())
        got = out.cpu().tolist()
    finally:
        N.load().pse_accept_select(0)
    want = [sample_with_uniform(logits[i].numpy(), temp, float(u[i, 1])) for i in range(rows)]
    assert got == want
    if temp == 0:
        assert got[0] == 5


def _accept_inputs(rows, k, vocab, temp, seed, agree):
    g = torch.Generator().manual_seed(seed)
    tgt = torch.randn(rows, k + 1, vocab, generator=g) * 3
    drf = tgt[:, :k] + torch.randn(rows, k, vocab, generator=g) * (3 * (1 - agree))
    u = torch.rand(rows, 2 * k + 1, generator=g, dtype=torch.float64)
    drafts = np.zeros((rows, k), dtype=np.int64)
    for i in range(rows):
        for j in range(k):
            if temp > 0:
                drafts[i, j] = sample_with_uniform(drf[i, j].numpy(), temp, float(u[i, j]))
            else:
                drafts[i, j] = int(torch.argmax(tgt[i, j])) if (i + j) % 3 else int(torch.argmax(drf[i, j]))
    return tgt, drf, u, drafts


def _run_accept(N, tgt, drf, u, drafts, temp):
    rows, kp1, vocab = tgt.shape
    k = kp1 - 1
    t0 = tgt[:, 0].contiguous().cuda()
    ver = tgt[:, 1:].contiguous().cuda()
    d0 = drf[:, 0].contiguous().cuda()
    dr = drf[:, 1:].transpose(0, 1).contiguous().cuda() if k > 1 else d0  # [k-1, rows, V]
    dd = torch.from_numpy(drafts.astype(np.int32)).cuda()
    ud = u.cuda()
    toks = torch.empty(rows, k + 1, dtype=torch.int32, device="cuda")
    nacc = torch.empty(rows, dtype=torch.int32, device="cuda")
    fin = torch.empty(rows, dtype=torch.int32, device="cuda")
    N.call("pse_spec_accept", t0.data_ptr(), vocab, None, ver.data_ptr(), k * vocab, vocab,
           d0.data_ptr(), vocab, None, dr.data_ptr(), vocab, rows * vocab, dd.data_ptr(), ud.data_ptr(),
           2 * k + 1, rows, k, vocab, temp, toks.data_ptr(), nacc.data_ptr(), fin.data_ptr(), N.stream_ptr())
    return toks.cpu().numpy(), nacc.cpu().numpy(), fin.cpu().numpy()


@pytest.mark.parametrize("k,vocab,temp,agree", [
    (1, 64, 0.0, 0.0), (4, 256, 0.0, 0.0), (8, 1000, 0.0, 0.0),
    (3, 64, 1.0, 0.9), (5, 1000, 1.0, 0.97), (8, 4096, 0.8, 0.99), (2, 32000, 1.0, 0.0),
    (1, 1000, 1.0, 0.9),     # one draft: no draft rows past the first
    (3, 1001, 1.0, 0.95),    # vocab not a multiple of 4: the scalar kernel takes the row
])
def test_accept_resample_matches_oracle(k, vocab, temp, agree):
    N = _N()
    rows = 64
    tgt, drf, u, drafts = _accept_inputs(rows, k, vocab, temp, seed=k * 1000 + vocab, agree=agree)
    toks, nacc, fin = _run_accept(N, tgt, drf, u, drafts, temp)
    seen = set()
    for i in range(rows):
        want, n = accept_row(tgt[i].numpy(), drf[i].numpy(), drafts[i], u[i].numpy(), k, temp)
        assert nacc[i] == n, (i, nacc[i], n)
        assert toks[i, : n + 1].tolist() == want and fin[i] == want[-1]
        seen.add(n)
    if temp > 0 and agree > 0.9:
        assert len(seen) > 1  # both accept and reject paths exercised


@pytest.mark.parametrize("rows,k,vocab,temp,agree", [
    (24, 4, 128256, 1.0, 0.97),   # cluster of 8 CTAs per row
    (16, 3, 100000, 0.7, 0.99),   # cluster of 7; streaming segments padded to 3200
    (300, 2, 32000, 1.0, 0.95),   # more rows than CTAs / clusters in flight: persistent
    (40, 8, 16388, 1.0, 0.98),    # just past a single cluster CTA's capacity
    (20, 3, 200000, 1.0, 0.97),   # beyond the cluster kernel's reach (it falls back to the scalar kernel)
])
def test_accept_kernels_match_oracle(rows, k, vocab, temp, agree):
    """T > 0 has four kernels (cluster-split streaming, the default; CTA-per-row
    scalar; one thread-block cluster per row holding the row on chip; streaming
    CTA per row).  Each must give the oracle's tokens exactly."""
    N = _N()
    tgt, drf, u, drafts = _accept_inputs(rows, k, vocab, temp, seed=rows + k + vocab, agree=agree)
    outs = []
    try:
        for kern in (0, 1, 2, 3):
            N.load().pse_accept_select(kern)
            outs.append(_run_accept(N, tgt, drf, u, drafts, temp))
    finally:
        N.load().pse_accept_select(0)
    seen = set()
    for i in range(rows):
        want, n = accept_row(tgt[i].numpy(), drf[i].numpy(), drafts[i], u[i].numpy(), k, temp)
        for toks, nacc, fin in outs:
            assert nacc[i] == n, (i, nacc[i], n)
            assert toks[i, : n + 1].tolist() == want and fin[i] == want[-1]
            assert (toks[i, n + 1:] == -1).all()
        seen.add(n)
    assert len(seen) > 1  # accepted runs, rejections (and bonus draws) all exercised


def test_accept_all_accepted_uses_bonus_position():
    N = _N()
    rows, k, vocab = 8, 3, 50
    tgt, _, u, _ = _accept_inputs(rows, k, vocab, 0.0, seed=1, agree=0)
    drafts = np.stack([[int(torch.argmax(tgt[i, j])) for j in range(k)] for i in range(rows)])
    toks, nacc, fin = _run_accept(N, tgt, tgt[:, :k].clone(), u, drafts, 0.0)
    assert (nacc == k).all()
    for i in range(rows):
        assert fin[i] == int(torch.argmax(tgt[i, k]))
    # T = 1 with identical draft and target: ratio is 1, every draft accepted
    drafts = np.stack([[sample_with_uniform(tgt[i, j].numpy(), 1.0, float(u[i, j])) for j in range(k)]
                       for i in range(rows)])
    toks, nacc, fin = _run_accept(N, tgt, tgt[:, :k].clone(), u, drafts, 1.0)
    assert (nacc == k).all()
    for i in range(rows):
        w, z = weights(tgt[i, k].numpy(), 1.0)
        assert fin[i] == inverse_cdf(w, float(z), float(u[i, 2 * k]))
