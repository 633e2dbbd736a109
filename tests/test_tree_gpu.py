"""Tree speculation (pse.tree; the reference's README lists it as future work)
on the device, against oracle/tree.py (itself checked on CPU: one branch is
the reference's linear rule, several keep the target's distribution).

* the accept kernel gives the oracle's tokens, accepted counts and branches
  exactly on random logits (T = 0 and T > 0, 1 to 8 branches, vocabularies up
  to 32000);
* a whole step (draft chains and verify with tree-masked attention, accept,
  the kept branch's K/V moved into place, the bonus call) gives the oracle's
  full-recomputation step draw for draw, and each request's cached K/V
  afterwards equals the reference model's K/V of its committed sequence;
* greedy tree decoding through the unchanged scheduler loop equals each
  request's solo ``generate_cached``, with the pool whole at the end;
* one branch is the linear step; T = 1 first tokens follow the target's
  softmax (chi-squared).
GPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from scipy.stats import chisquare

from oracle.generate import generate_cached
from oracle.model import ModelConfig, TinyGPT
from oracle.sampling import sample_with_uniform, weights
from oracle.tree import top_candidates, tree_accept_row, tree_step_row, tree_uniform_count

pytestmark = pytest.mark.gpu

CFG = ModelConfig(vocab_size=64, d_model=32, n_layers=2, n_heads=4, d_ff=64, max_seq_len=256)


def _N():
    import pse._native as N
    return N


def _tree_inputs(rows, b, k, V, T, agree, seed):
    g = torch.Generator().manual_seed(seed)
    p_root = torch.randn(rows, V, generator=g) * 3
    q_root = p_root + torch.randn(rows, V, generator=g) * (3 * (1 - agree))
    p_chain = torch.randn(rows, b, k, V, generator=g) * 3
    q_chain = p_chain[:, :, : max(k - 1, 0)] + torch.randn(rows, b, max(k - 1, 0), V, generator=g) * (3 * (1 - agree))
    U = tree_uniform_count(k, b)
    u = torch.rand(rows, U, generator=g, dtype=torch.float64)
    chain = np.zeros((rows, b, k), dtype=np.int64)
    for i in range(rows):
        cands = top_candidates(q_root[i].numpy(), b) if T <= 0 else \
            [sample_with_uniform(q_root[i].numpy(), T, float(u[i, j])) for j in range(b)]
        for j in range(b):
            chain[i, j, 0] = cands[j]
            for d in range(1, k):
                q = q_chain[i, j, d - 1].numpy()
                chain[i, j, d] = int(np.argmax(q)) if T <= 0 else sample_with_uniform(q, T, float(u[i, d * b + j]))
    if T <= 0:
        # greedy chains that sometimes agree with the target
        for i in range(rows):
            for j in range(b):
                if (i + j) % 3 == 0:
                    chain[i, j, 0] = int(torch.argmax(p_root[i]))
                    for d in range(1, k):
                        chain[i, j, d] = int(torch.argmax(p_chain[i, j, d - 1])) if (i + d) % 4 else chain[i, j, d]
    return p_root, q_root, p_chain, q_chain, u, chain


def _run_tree_accept(N, p_root, q_root, p_chain, q_chain, u, chain, b, k, T):
    rows, V = p_root.shape
    pr, qr = p_root.contiguous().cuda(), q_root.contiguous().cuda()
    ver = p_chain.reshape(rows * b, k, V).contiguous().cuda()
    dch = (q_chain.reshape(rows * b, k - 1, V).transpose(0, 1).contiguous().cuda() if k > 1
           else torch.zeros(1, rows * b, V, device="cuda"))
    ch = torch.from_numpy(chain.astype(np.int32)).cuda()
    ud = u.cuda()
    toks = torch.empty(rows, k + 1, dtype=torch.int32, device="cuda")
    res = torch.empty(3, rows, dtype=torch.int32, device="cuda")
    N.call("pse_tree_accept", pr.data_ptr(), V, None, qr.data_ptr(), V, None, ver.data_ptr(), b * k * V, k * V, V,
           dch.data_ptr(), b * V, V, rows * b * V, ch.data_ptr(), ud.data_ptr(), u.shape[1], rows, b, k, V, T,
           toks.data_ptr(), res[0].data_ptr(), res[1].data_ptr(), res[2].data_ptr(), N.stream_ptr())
    return toks.cpu().numpy(), res.cpu().numpy()


@pytest.mark.parametrize("rows,b,k,V,T,agree", [
    (48, 1, 3, 64, 1.0, 0.9), (48, 2, 4, 1000, 1.0, 0.7), (40, 4, 2, 257, 0.8, 0.7),
    (24, 3, 3, 32000, 1.0, 0.5), (32, 8, 2, 100, 1.0, 0.5), (48, 2, 1, 50, 1.0, 0.3),
    (48, 2, 4, 1000, 0.0, 0.0), (32, 3, 3, 257, 0.0, 0.0), (16, 1, 5, 64, 0.0, 0.0),
])
def test_tree_accept_kernel_matches_oracle(rows, b, k, V, T, agree):
    N = _N()
    p_root, q_root, p_chain, q_chain, u, chain = _tree_inputs(rows, b, k, V, T, agree, seed=rows * 7 + b + k + V)
    toks, res = _run_tree_accept(N, p_root, q_root, p_chain, q_chain, u, chain, b, k, T)
    seen_n, seen_b = set(), set()
    for i in range(rows):
        want, n, br = tree_accept_row(p_root[i].numpy(), q_root[i].numpy(), chain[i],
                                      [[p_chain[i, j, d].numpy() for d in range(k)] for j in range(b)],
                                      [[q_chain[i, j, d].numpy() for d in range(k - 1)] for j in range(b)],
                                      u[i].numpy(), k, b, T)
        assert (res[0, i], res[1, i], res[2, i]) == (n, br, want[-1]), i
        assert toks[i, : n + 1].tolist() == want and (toks[i, n + 1:] == -1).all()
        seen_n.add(n)
        seen_b.add(br)
    assert len(seen_n) > 1
    if b > 1:
        assert len(seen_b) > 1  # other branches than the first were kept


def _models(seed):
    torch.manual_seed(seed)
    return TinyGPT(CFG).eval(), TinyGPT(CFG).eval()


def _caches(bs, nb):
    import pse
    hd = CFG.d_model // CFG.n_heads
    return (pse.PagedKVCache(CFG.n_layers, CFG.n_heads, hd, bs, nb),
            pse.PagedKVCache(CFG.n_layers, CFG.n_heads, hd, bs, nb))


@pytest.mark.parametrize("b,k,T,bs", [(2, 3, 0.0, 4), (3, 2, 1.0, 4), (2, 4, 1.0, 3), (4, 3, 0.0, 16)])
def test_tree_step_matches_oracle_step_and_cache(b, k, T, bs):
    import pse
    d, t = _models(b * 10 + k)
    # a draft close to the target, so branches other than the first are taken
    with torch.no_grad():
        for pd, pt in zip(d.parameters(), t.parameters()):
            pd.copy_(pt + 0.02 * torch.randn_like(pt))
    rng = np.random.default_rng(b + k)
    prompts = [rng.integers(0, 64, size=int(rng.integers(2, 14))).tolist() for _ in range(6)]
    ids = [f"q{i}" for i in range(len(prompts))]
    dc, tc = _caches(bs, 400)
    out = pse.prefill_requests(d, t, dc, tc, ids, prompts)
    dn = {r: out[r][0] for r in ids}
    tn = {r: out[r][1] for r in ids}
    seqs = {r: list(p) for r, p in zip(ids, prompts)}
    U = tree_uniform_count(k, b)
    branches_seen = set()
    for step in range(3):
        u = rng.random((len(ids), U))
        res = pse.batched_tree_speculative_step(d, t, ids, dc, tc, dn, tn, k, b, T, uniforms=u)
        for i, r in enumerate(ids):
            want, n, br, _ = tree_step_row(d, t, seqs[r], k, b, T, u[i])
            assert res.accepted_tokens[r] == want, (step, r)
            assert res.num_draft_accepted[r] == n
            branches_seen.add(br)
            seqs[r].extend(want)
        dn, tn = res.draft_next_logits, res.target_next_logits
    assert b == 1 or len(branches_seen) > 1
    # every request's cached K/V is the reference model's K/V of its committed sequence
    for c, m in ((dc, d), (tc, t)):
        for r in ids:
            assert c.length(r) == len(seqs[r])
            ks, vs, _, _ = c.gather([r])
            with torch.no_grad():
                _, past = m(torch.tensor([seqs[r]]))
            for L in range(CFG.n_layers):
                assert torch.allclose(ks[L][0].cpu(), past[L][0][0], atol=1e-4)
                assert torch.allclose(vs[L][0].cpu(), past[L][1][0], atol=1e-4)
    for c in (dc, tc):
        for r in ids:
            c.free_request(r)
        assert sorted(c.allocator.free_list()) == list(range(400))


@pytest.mark.parametrize("b,k,bs,batch,prefix", [(2, 3, 4, 3, False), (3, 4, 16, 5, False), (2, 2, 1, 2, False),
                                                  (2, 3, 4, 4, True)])
def test_tree_scheduler_greedy_equals_solo(b, k, bs, batch, prefix):
    import pse
    d, t = _models(b + 31 * k)
    with torch.no_grad():
        for pd, pt in zip(d.parameters(), t.parameters()):
            pd.copy_(pt + 0.05 * torch.randn_like(pt))
    rng = np.random.default_rng(b * k)
    shared = rng.integers(0, 64, size=2 * bs + 1).tolist() if prefix else []
    reqs = [pse.Request(f"r{i}", shared + rng.integers(0, 64, size=int(rng.integers(1, 16))).tolist(),
                        int(rng.integers(1, 12))) for i in range(9)]
    nb = 500
    hd = CFG.d_model // CFG.n_heads
    dc, tc = (pse.PagedKVCache(CFG.n_layers, CFG.n_heads, hd, bs, nb, prefix_cache=prefix) for _ in range(2))
    res = pse.run_continuous_speculative_batches(d, t, reqs, dc, tc, batch, k=k, tree_branches=b)
    by = {r.request_id: r.output_ids for r in res}
    for q in reqs:
        assert by[q.request_id] == generate_cached(t, torch.tensor([q.prompt_ids]), q.max_new_tokens), q
    for c in (dc, tc):
        if prefix:
            assert c.prefix.stats()["hit_tokens"] > 0
            c.prefix.clear()
        assert sorted(c.allocator.free_list()) == list(range(nb))


def test_one_branch_is_the_linear_step():
    import pse
    d, t = _models(4)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 64, size=int(rng.integers(2, 10))).tolist() for _ in range(5)]
    ids = [f"x{i}" for i in range(5)]
    k = 3
    toks = []
    for tree in (False, True):
        dc, tc = _caches(4, 300)
        out = pse.prefill_requests(d, t, dc, tc, ids, prompts)
        dn = {r: out[r][0] for r in ids}
        tn = {r: out[r][1] for r in ids}
        got = []
        urng = np.random.default_rng(9)
        for _ in range(3):
            u = urng.random((5, 2 * k + 1))
            if tree:
                res = pse.batched_tree_speculative_step(d, t, ids, dc, tc, dn, tn, k, 1, 1.0, uniforms=u)
            else:
                res = pse.batched_speculative_step(d, t, ids, dc, tc, dn, tn, k, 1.0, uniforms=u, defer_bonus=False)
            got.append(res.accepted_tokens)
            dn, tn = res.draft_next_logits, res.target_next_logits
        toks.append(got)
    assert toks[0] == toks[1]


def test_tree_first_token_follows_the_target_softmax():
    import pse
    torch.manual_seed(8)
    cfg = ModelConfig(vocab_size=16, d_model=16, n_layers=1, n_heads=2, d_ff=32, max_seq_len=64)
    d, t = TinyGPT(cfg).eval(), TinyGPT(cfg).eval()
    hd = cfg.d_model // cfg.n_heads
    prompt = [1, 5, 2]
    n, b, k = 500, 3, 2
    counts = np.zeros(16)
    for rep in range(4):
        ids = [f"s{rep}_{i}" for i in range(n)]
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 8 * n)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_heads, hd, 4, 8 * n)
        out = pse.prefill_requests(d, t, dc, tc, ids, [prompt] * n)
        res = pse.batched_tree_speculative_step(d, t, ids, dc, tc, {r: out[r][0] for r in ids},
                                                {r: out[r][1] for r in ids}, k, b, 1.0)
        for r in ids:
            counts[res.accepted_tokens[r][0]] += 1
    with torch.no_grad():
        logits, _ = t(torch.tensor([prompt]))
    w, _ = weights(logits[0, -1].numpy(), 1.0)
    law = w.astype(np.float64) / w.astype(np.float64).sum()
    assert chisquare(counts, counts.sum() * law).pvalue > 0.001


def test_tree_step_llama_matches_oracle_step():
    """Llama-style pair (GQA, RoPE at the nodes' own positions): tree steps
    against the oracle's full recomputation, fp32, T = 0 and T = 1."""
    import pse
    from oracle.model import LlamaConfig, TinyLlama
    torch.manual_seed(21)
    cfg = LlamaConfig(vocab_size=64, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=96, max_seq_len=256)
    t = TinyLlama(cfg).eval()
    d = TinyLlama(cfg).eval()
    with torch.no_grad():
        for pd, pt in zip(d.parameters(), t.parameters()):
            pd.copy_(pt + 0.02 * torch.randn_like(pt))
    hd = cfg.d_model // cfg.n_heads
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 64, size=int(rng.integers(2, 12))).tolist() for _ in range(4)]
    ids = [f"l{i}" for i in range(4)]
    for T in (0.0, 1.0):
        dc = pse.PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, 4, 300)
        tc = pse.PagedKVCache(cfg.n_layers, cfg.n_kv_heads, hd, 4, 300)
        out = pse.prefill_requests(d, t, dc, tc, ids, prompts)
        dn = {r: out[r][0] for r in ids}
        tn = {r: out[r][1] for r in ids}
        seqs = {r: list(p) for r, p in zip(ids, prompts)}
        b, k = 3, 3
        for step in range(3):
            u = rng.random((4, tree_uniform_count(k, b)))
            res = pse.batched_tree_speculative_step(d, t, ids, dc, tc, dn, tn, k, b, T, uniforms=u)
            for i, r in enumerate(ids):
                want, n, _, _ = tree_step_row(d, t, seqs[r], k, b, T, u[i])
                assert res.accepted_tokens[r] == want, (T, step, r)
                seqs[r].extend(want)
            dn, tn = res.draft_next_logits, res.target_next_logits
        for r in ids:
            ks, _, _, _ = tc.gather([r])
            with torch.no_grad():
                _, past = t(torch.tensor([seqs[r]]))
            assert torch.allclose(ks[0][0].cpu(), past[0][0][0], atol=1e-4)
