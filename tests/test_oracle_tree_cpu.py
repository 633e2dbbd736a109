"""The tree-speculation rule of oracle/tree.py (the reference's README lists
tree-based speculation as future work, with no code): with one branch it is
the reference's linear rule (oracle.accept.accept_row, pinned to the
reference), the recursive rejection over several candidates leaves the first
committed token distributed exactly as the target's distribution (exact
enumeration and a Monte Carlo run of the oracle function itself), and greedy
trees commit the target's argmax.  No GPU."""
from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch
from scipy.stats import chisquare

from oracle.accept import accept_row
from oracle.model import ModelConfig, TinyGPT
from oracle.sampling import sample_with_uniform, weights
from oracle.tree import tree_accept_row, tree_generate, tree_step_row, tree_uniform_count
from oracle.generate import generate_cached


def _logits(rng, *shape):
    return (rng.standard_normal(shape) * 2).astype(np.float32)


@pytest.mark.parametrize("k,V,T", [(1, 7, 1.0), (3, 11, 0.8), (4, 50, 1.0), (3, 11, 0.0), (5, 40, 0.0)])
def test_single_branch_is_the_linear_rule(k, V, T):
    rng = np.random.default_rng(k * 100 + V)
    for trial in range(60):
        p = _logits(rng, k + 1, V)
        q = p[:k] + _logits(rng, k, V) * (0.3 if trial % 2 else 1.5)
        u = rng.random(2 * k + 1)
        drafts = [sample_with_uniform(q[j], T, u[j]) if T > 0 else int(np.argmax(q[j])) for j in range(k)]
        if T == 0 and trial % 3 == 0:
            drafts = [int(np.argmax(p[j])) for j in range(k)]
        want, n = accept_row(p, q, drafts, u, k, T)
        chain = np.array([drafts])
        p_chain = [[p[d + 1] for d in range(k)]]
        q_chain = [[q[d + 1] for d in range(k - 1)]]
        got, n2, br = tree_accept_row(p[0], q[0], chain, p_chain, q_chain, u, k, 1, T)
        assert (got, n2, br) == (want, n, 0)


def _first_token_law(p, q, b, T):
    """Exact law of the first committed token by enumerating the candidates
    (iid from q) and integrating the accept uniforms analytically."""
    V = len(p)
    wp, zp = weights(p, T)
    wq, zq = weights(q, T)
    qd = wq.astype(np.float64) / float(zq)
    law = np.zeros(V)
    for cands in itertools.product(range(V), repeat=b):
        w = np.prod([qd[x] for x in cands])
        P = wp.astype(np.float64) * (1.0 / float(zp))
        Q = wq.astype(np.float64) * (1.0 / float(zq))
        alive = 1.0
        last = None
        for x in cands:
            a = min(1.0, P[x] / Q[x]) if Q[x] > 0 else 0.0
            law[x] += w * alive * a
            alive *= 1.0 - a
            r = np.maximum(P - Q, 0.0)
            if r.sum() > 0:
                last = r / r.sum()
                P = r * (1.0 / r.sum())
        law += w * alive * (last if last is not None else wp / float(zp))
    return law


@pytest.mark.parametrize("b", [1, 2, 3])
def test_recursive_rejection_preserves_the_target_law(b):
    rng = np.random.default_rng(b)
    for _ in range(5):
        p, q = _logits(rng, 5), _logits(rng, 5)
        law = _first_token_law(p, q, b, 1.0)
        wp, zp = weights(p, 1.0)
        assert np.allclose(law, wp.astype(np.float64) / float(zp), atol=1e-12)


@pytest.mark.parametrize("b", [2, 3])
def test_oracle_tree_rule_samples_the_target_law(b):
    """Monte Carlo of tree_accept_row itself (k = 1): the first token's counts
    against the target's softmax."""
    rng = np.random.default_rng(10 + b)
    V, k, T = 6, 1, 1.0
    p, q = _logits(rng, V), _logits(rng, V) * 0.5
    p_chain = [[_logits(rng, V)] for _ in range(b)]
    counts = np.zeros(V)
    n = 6000
    for _ in range(n):
        u = rng.random(tree_uniform_count(k, b))
        chain = np.array([[sample_with_uniform(q, T, u[j])] for j in range(b)])
        toks, _, _ = tree_accept_row(p, q, chain, p_chain, [[] for _ in range(b)], u, k, b, T)
        counts[toks[0]] += 1
    wp, _ = weights(p, T)
    law = wp.astype(np.float64) / wp.astype(np.float64).sum()
    assert chisquare(counts, n * law).pvalue > 0.001


def test_greedy_tree_decode_is_the_target_greedy_decode():
    torch.manual_seed(0)
    cfg = ModelConfig(vocab_size=40, d_model=16, n_layers=2, n_heads=2, d_ff=32, max_seq_len=128)
    d, t = TinyGPT(cfg).eval(), TinyGPT(cfg).eval()
    for prompt, b, k in (([1, 2, 3], 2, 3), ([5], 3, 2), ([7, 8, 9, 10, 11], 1, 4)):
        want = generate_cached(t, torch.tensor([prompt]), 12)
        assert tree_generate(d, t, prompt, 12, k, b) == want
    # with draft = target every greedy branch-0 chain is accepted in full
    toks, n, br, _ = tree_step_row(t, t, [1, 2, 3], 4, 2, 0.0)
    assert n == 4 and br == 0 and len(toks) == 5
