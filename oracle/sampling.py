"""Sampling helpers: the reference's (engine/sampling.py:10-23) and the
explicit-uniform forms the CUDA kernels implement.

Explicit-uniform arithmetic (shared with csrc/sampling.cu, stated once here):

* ``s_i = l_i / T`` in float32 (IEEE division), ``m = max_i s_i``;
* weight ``w_i = exp(s_i - m)`` rounded to float32;
* normaliser ``Z = sum_i w_i`` accumulated in float64;
* inverse CDF: with ``t = u * Z``, the token is the first ``i`` whose float64
  running sum of weights exceeds ``t``; if rounding leaves none, the last ``i``
  with ``w_i > 0``.

Greedy is ``argmax`` with ties to the lowest index, as ``torch.argmax``.
"""
from __future__ import annotations

import numpy as np
import torch


# --- engine/sampling.py:10-23 (torch, generator-driven) ---
def softmax_with_temperature(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    return torch.softmax(logits / temperature, dim=-1)


def sample_categorical(probs: torch.Tensor, generator=None) -> int:
    return int(torch.multinomial(probs, num_samples=1, generator=generator).item())


def greedy_token(logits: torch.Tensor) -> int:
    return int(logits.argmax(dim=-1).item())


# --- explicit-uniform forms ---
def weights(logits, temperature: float):
    """float32 weights and float64 normaliser of softmax(logits / T) along the
    last axis.  Works on [..., V]."""
    l = np.asarray(logits, dtype=np.float32)
    s = l / np.float32(temperature)
    m = s.max(axis=-1, keepdims=True)
    w = np.exp((s - m).astype(np.float64)).astype(np.float32)
    z = w.astype(np.float64).sum(axis=-1)
    return w, z


def inverse_cdf(w, total: float, u: float) -> int:
    """First index whose running float64 sum of ``w`` exceeds ``u * total``."""
    w64 = np.asarray(w, dtype=np.float64)
    run = np.cumsum(w64)
    hit = np.nonzero(run > u * total)[0]
    if hit.size:
        return int(hit[0])
    nz = np.nonzero(w64 > 0)[0]
    return int(nz[-1]) if nz.size else 0


def sample_with_uniform(logits, temperature: float, u: float) -> int:
    """Draw from softmax(logits / T) with one explicit uniform; T == 0 is greedy."""
    if temperature <= 0:
        return int(np.argmax(np.asarray(logits, dtype=np.float32)))
    w, z = weights(logits, temperature)
    return inverse_cdf(w, float(z), u)
