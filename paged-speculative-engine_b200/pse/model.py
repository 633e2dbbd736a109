"""Model definitions the engine runs: parameter layouts and configs only.

``TinyGPT`` has the reference's module tree and parameter names
(engine/model.py:21-28, 67-74, 121-129, 145-156), so ``torch.manual_seed(s);
TinyGPT(cfg)`` draws the same weights as the reference constructor and either
state_dict loads into the other.  The engine accepts any module with this
layout -- the reference's own ``TinyGPT`` objects included -- and reads only its
parameters; it never calls ``forward``.

``TinyLlama`` is the GQA / RoPE / SwiGLU / RMSNorm layout of the Llama-style
workload (no reference counterpart): fused ``qkv`` (q heads, then k heads, then
v heads, no bias), ``out``, ``gate_up`` (gate rows first), ``down``, norms
``norm1``/``norm2``/``norm_f`` and an untied ``lm_head``.

Neither class has a forward: the only compute path is the paged CUDA engine
(``pse.batched_forward_append`` and the speculative step).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn


@dataclass
class ModelConfig:
    vocab_size: int = 256
    d_model: int = 64
    n_layers: int = 4
    n_heads: int = 4
    d_ff: int = 256
    max_seq_len: int = 512


class _Attention(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model)
        self.out = nn.Linear(cfg.d_model, cfg.d_model)


class _Block(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = _Attention(cfg)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.mlp = nn.Sequential(nn.Linear(cfg.d_model, cfg.d_ff), nn.GELU(), nn.Linear(cfg.d_ff, cfg.d_model))


class TinyGPT(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.pos_emb = nn.Embedding(cfg.max_seq_len, cfg.d_model)
        self.blocks = nn.ModuleList([_Block(cfg) for _ in range(cfg.n_layers)])
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)


@dataclass
class LlamaConfig:
    vocab_size: int = 32000
    d_model: int = 2048
    n_layers: int = 16
    n_heads: int = 32
    n_kv_heads: int = 8
    d_ff: int = 8192
    max_seq_len: int = 16384
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5


class _RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class _LlamaAttention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0 and cfg.n_heads % cfg.n_kv_heads == 0
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.theta = cfg.rope_theta
        self.qkv = nn.Linear(cfg.d_model, (cfg.n_heads + 2 * cfg.n_kv_heads) * self.head_dim, bias=False)
        self.out = nn.Linear(cfg.n_heads * self.head_dim, cfg.d_model, bias=False)


class _LlamaBlock(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.norm1 = _RMSNorm(cfg.d_model, cfg.norm_eps)
        self.attn = _LlamaAttention(cfg)
        self.norm2 = _RMSNorm(cfg.d_model, cfg.norm_eps)
        self.gate_up = nn.Linear(cfg.d_model, 2 * cfg.d_ff, bias=False)
        self.down = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)


class TinyLlama(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.blocks = nn.ModuleList([_LlamaBlock(cfg) for _ in range(cfg.n_layers)])
        self.norm_f = _RMSNorm(cfg.d_model, cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
