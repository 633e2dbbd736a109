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


def paged_attention(q, k_pool, v_pool, tables, base_len, scale=None):
    """q [R, W, Hq, hd] -> out [R, W, Hq, hd] (float64)."""
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
        pos = int(base_len[i]) + np.arange(width)
        allowed = np.arange(ctx)[None, :] <= pos[:, None]  # [W, ctx]
        s = np.where(allowed[:, None, :], s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[i] = np.einsum("wht,htd->whd", p, v)
    return out
