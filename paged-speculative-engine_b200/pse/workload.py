"""Seeded synthetic workloads with the shapes of the benchmark configurations.

Nothing here touches a GPU.  Prompts come from ``numpy.random.default_rng(seed)``
(PCG64) so every run, on every machine, sees the same requests.

=============  =================================================================
name           workload
=============  =================================================================
tiny           TinyGPT pair fp32 (target d128/4L/4H/ff512, draft d64/2L/2H/ff256,
               vocab 256, context 256); 8 prompts of U[8,32] tokens, 64 new,
               k=4, block 16, batch 4, greedy
tiny-sampled   same pair at T=1: 64 prompts of U[8,64], 128 new, k in {2,4,8}
gpt2-small     GPT-2-small-shaped pair bf16 (target d768/12L/12H/ff3072, draft
               d384/4L/6H/ff1536, vocab 32000); 256 prompts of U[128,1024],
               256 new, k=5, block 16, greedy
llama-1b       Llama-style pair bf16 (target d2048/16L/32q-8kv/SwiGLU 8192,
               draft d1024/2L/16q-4kv/SwiGLU 4096, vocab 32000); 2048 prompts
               lognormal(median 2048, sigma 0.8) clipped to [128, 8192],
               512 new, k=4, block 32
=============  =================================================================
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class PairSpec:
    """Shapes of one draft/target pair.  ``kind`` is "gpt" (TinyGPT layout) or
    "llama" (GQA/RoPE/SwiGLU layout)."""
    kind: str
    vocab: int
    target: dict
    draft: dict


TINY = PairSpec("gpt", 256,
                dict(d_model=128, n_layers=4, n_heads=4, d_ff=512, max_seq_len=256),
                dict(d_model=64, n_layers=2, n_heads=2, d_ff=256, max_seq_len=256))
GPT2_SMALL = PairSpec("gpt", 32000,
                      dict(d_model=768, n_layers=12, n_heads=12, d_ff=3072, max_seq_len=1536),
                      dict(d_model=384, n_layers=4, n_heads=6, d_ff=1536, max_seq_len=1536))
LLAMA_1B = PairSpec("llama", 32000,
                    dict(d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, d_ff=8192, max_seq_len=16384),
                    dict(d_model=1024, n_layers=2, n_heads=16, n_kv_heads=4, d_ff=4096, max_seq_len=16384))


@dataclass(frozen=True)
class Workload:
    name: str
    pair: PairSpec
    n_requests: int
    prompt_lo: int
    prompt_hi: int
    max_new_tokens: int
    k: int
    block_size: int
    max_batch_size: int
    temperature: float
    dtype: str
    lognormal_sigma: float = 0.0  # > 0: lognormal lengths with median sqrt(lo*hi)... see prompts()
    lognormal_median: float = 0.0


WORKLOADS = {
    "tiny": Workload("tiny", TINY, 8, 8, 32, 64, 4, 16, 4, 0.0, "float32"),
    "tiny-sampled": Workload("tiny-sampled", TINY, 64, 8, 64, 128, 4, 16, 64, 1.0, "float32"),
    "gpt2-small": Workload("gpt2-small", GPT2_SMALL, 256, 128, 1024, 256, 5, 16, 256, 0.0, "bfloat16"),
    "llama-1b": Workload("llama-1b", LLAMA_1B, 2048, 128, 8192, 512, 4, 32, 2048, 0.0, "bfloat16",
                         lognormal_sigma=0.8, lognormal_median=2048.0),
}


def prompts(w: Workload, seed: int = 0, n: int | None = None) -> list[list[int]]:
    """The workload's prompts (first ``n`` if given), token ids uniform over the
    vocabulary, lengths U[lo, hi] or clipped lognormal."""
    rng = np.random.default_rng(seed)
    count = w.n_requests if n is None else n
    if w.lognormal_sigma > 0:
        lengths = rng.lognormal(math.log(w.lognormal_median), w.lognormal_sigma, size=count)
        lengths = np.clip(np.rint(lengths), w.prompt_lo, w.prompt_hi).astype(np.int64)
    else:
        lengths = rng.integers(w.prompt_lo, w.prompt_hi + 1, size=count)
    return [rng.integers(0, w.pair.vocab, size=int(L)).tolist() for L in lengths]


def request_ids(n: int, prefix: str = "r") -> list[str]:
    return [f"{prefix}{i}" for i in range(n)]


def lpt_shards(costs, n_shards: int) -> list[list[int]]:
    """Longest-processing-time assignment of items (by cost) to shards; returns
    the item indices of each shard, each list in ascending item order."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * n_shards
    shards: list[list[int]] = [[] for _ in range(n_shards)]
    for i in order:
        s = min(range(n_shards), key=lambda j: (loads[j], j))
        shards[s].append(i)
        loads[s] += costs[i]
    return [sorted(s) for s in shards]
