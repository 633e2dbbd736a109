"""Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
as 1, 2, 3", SC 2011), vectorised in numpy.

This is the uniform source of the explicit-uniform sampling mode.  The CUDA
kernel ``pse_philox_uniforms`` implements the same function; both map a
(seed, request key, step, slot) tuple to one float64 uniform in [0, 1), so the
accept/reject decisions of the GPU and of this oracle are comparable draw for
draw.

Keying (shared with the kernel):
    key     = (seed & 0xffffffff, seed >> 32)
    counter = (slot // 2, request_key, step, STREAM_TAG)
    words (x0, x1) -> uniform of the even slot, (x2, x3) -> the odd slot,
    u = ((x_hi << 32 | x_lo) >> 11) * 2**-53.
"""
from __future__ import annotations

import numpy as np

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
STREAM_TAG = 0x53504543  # "SPEC"
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, key: np.ndarray) -> np.ndarray:
    """ctr: [..., 4] uint32, key: [..., 2] uint32 -> [..., 4] uint32."""
    c = np.array(ctr, dtype=np.uint32, copy=True)
    k = np.array(key, dtype=np.uint32, copy=True)
    c0, c1, c2, c3 = (c[..., i].astype(np.uint64) for i in range(4))
    k0, k1 = k[..., 0].astype(np.uint64), k[..., 1].astype(np.uint64)
    for r in range(10):
        if r:
            k0 = (k0 + np.uint64(PHILOX_W0)) & _MASK32
            k1 = (k1 + np.uint64(PHILOX_W1)) & _MASK32
        p0 = PHILOX_M0 * c0
        p1 = PHILOX_M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def words_to_unit(hi: np.ndarray, lo: np.ndarray) -> np.ndarray:
    bits = (hi.astype(np.uint64) << np.uint64(32)) | lo.astype(np.uint64)
    return (bits >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def request_key(request_id: str) -> int:
    """32-bit FNV-1a of the request id's UTF-8 bytes (stable across runs)."""
    h = 0x811C9DC5
    for b in request_id.encode("utf-8"):
        h ^= b
        h = (h * 0x01000193) & 0xFFFFFFFF
    return h


def step_uniforms(seed: int, req_keys, steps, n: int) -> np.ndarray:
    """Uniforms [rows, n] float64 for rows keyed by (req_keys[i], steps[i])."""
    req_keys = np.asarray(req_keys, dtype=np.uint32).reshape(-1)
    steps = np.asarray(steps, dtype=np.uint32).reshape(-1)
    rows = req_keys.shape[0]
    pairs = (n + 1) // 2
    ctr = np.zeros((rows, pairs, 4), dtype=np.uint32)
    ctr[..., 0] = np.arange(pairs, dtype=np.uint32)[None, :]
    ctr[..., 1] = req_keys[:, None]
    ctr[..., 2] = steps[:, None]
    ctr[..., 3] = STREAM_TAG
    key = np.zeros((rows, pairs, 2), dtype=np.uint32)
    key[..., 0] = seed & 0xFFFFFFFF
    key[..., 1] = (seed >> 32) & 0xFFFFFFFF
    w = philox4x32_10(ctr, key)
    u = np.empty((rows, pairs * 2), dtype=np.float64)
    u[:, 0::2] = words_to_unit(w[..., 0], w[..., 1])
    u[:, 1::2] = words_to_unit(w[..., 2], w[..., 3])
    return u[:, :n]
