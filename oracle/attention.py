"""Paged attention oracle: the masked softmax attention of
engine/model.py:99-116 evaluated directly on engine/paged_cache.py's block
layout (token p of a row lives in ``pool[table[p // bs], :, p % bs, :]``).

Query w of row i sits at absolute position ``base_len[i] + w`` and attends to
every key position ``<= base_len[i] + w`` (the causal rule of
engine/model.py:31-64 with the padding mask of engine/batched_forward.py:44);
its own K/V must already be in the pool.  Grouped query heads (Hq a multiple of
Hk) share key/value head ``h // (Hq // Hk)``.  Computed in float64.
"""
from __future__ import annotations

import numpy as np


def gather_row(pool: np.ndarray, table, n_tokens: int) -> np.ndarray:
    """pool [NB, Hk, bs, hd] -> [Hk, n_tokens, hd] for one row."""
    bs = pool.shape[2]
    nblk = (n_tokens + bs - 1) // bs
    blocks = pool[np.asarray(table[:nblk], dtype=np.int64)]  # [nblk, Hk, bs, hd]
    return blocks.transpose(1, 0, 2, 3).reshape(pool.shape[1], nblk * bs, pool.shape[3])[:, :n_tokens]


def visible(base: int, width: int, ctx: int, tree=None) -> np.ndarray:
    """[W, ctx] keys each query of a call sees.  Causal by default; ``tree=(b,
    d0)``: the call's tokens are token-tree nodes in depth-major order from
    depth d0 (query w is node n = d0*b + w at position L + n, L = base - d0*b),
    each seeing the keys below L and its own branch (n % b) at depths <= n // b
    (tree speculation: no reference counterpart)."""
    keys = np.arange(ctx)[None, :]
    if tree is None:
        return keys <= (base + np.arange(width))[:, None]
    b, d0 = tree
    n = d0 * b + np.arange(width)[:, None]
    L = base - d0 * b
    m = keys - L
    return (keys < L) | ((m >= 0) & (m % b == n % b) & (m // b <= n // b))


def paged_attention(q, k_pool, v_pool, tables, base_len, scale=None, tree=None):
    """q [R, W, Hq, hd] -> out [R, W, Hq, hd] (float64); ``tree`` as in ``visible``."""
    q = np.asarray(q, dtype=np.float64)
    rows, width, n_q, hd = q.shape
    n_kv = k_pool.shape[1]
    group = n_q // n_kv
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    out = np.zeros_like(q)
    for i in range(rows):
        ctx = int(base_len[i]) + width
        k = gather_row(np.asarray(k_pool, dtype=np.float64), tables[i], ctx)
        v = gather_row(np.asarray(v_pool, dtype=np.float64), tables[i], ctx)
        k = np.repeat(k, group, axis=0)  # [Hq, ctx, hd]
        v = np.repeat(v, group, axis=0)
        s = np.einsum("whd,htd->wht", q[i], k) * scale  # [W, Hq, ctx]
        allowed = visible(int(base_len[i]), width, ctx, tree)  # [W, ctx]
        s = np.where(allowed[:, None, :], s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[i] = np.einsum("wht,htd->whd", p, v)
    return out
