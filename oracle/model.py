"""CPU restatement of the reference model (engine/model.py) plus the Llama-style
model of the GQA/RoPE workload.

TinyGPT keeps the reference's module tree and parameter names exactly
(engine/model.py:145-156, 121-129, 67-74): with the same ``torch.manual_seed``
the constructor draws the same random numbers in the same order, so its weights
are bit-identical to the reference's and its state_dict loads either way.
That layout is a format both sides must share; the arithmetic below is this
oracle's own statement of engine/model.py:31-206.

The Llama-style model has no counterpart in the reference.  It is written to
the same ``forward(input_ids, past_kv, position_offset, padding_mask,
key_positions)`` contract (engine/model.py:158-206) so the reference-shaped
batched forward and ``generate_cached`` drive it unchanged.  Its conventions
(rotate-half RoPE with theta 10000, RMSNorm eps 1e-5, SwiGLU with the gate rows
first in ``gate_up``) are the ones the CUDA kernels implement.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

LayerKV = tuple[torch.Tensor, torch.Tensor]


@dataclass
class ModelConfig:
    """engine/model.py:21-28."""
    vocab_size: int = 256
    d_model: int = 64
    n_layers: int = 4
    n_heads: int = 4
    d_ff: int = 256
    max_seq_len: int = 512


def build_causal_mask(seq_len, total_len, position_offset, device, key_positions=None):
    """Absolute-position causal mask, engine/model.py:31-64.

    Query i of row b sits at position_offset[b] + i; it may attend key j iff
    its position is >= key_positions[b, j] (key_positions defaults to 0..total-1).
    """
    if key_positions is None:
        key_positions = torch.arange(total_len, device=device)
    if isinstance(position_offset, torch.Tensor):
        qpos = position_offset.view(-1, 1) + torch.arange(seq_len, device=device).view(1, -1)
        if key_positions.dim() == 1:
            key_positions = key_positions.view(1, -1).expand(position_offset.shape[0], -1)
        return qpos[:, :, None] >= key_positions[:, None, :]
    qpos = torch.arange(position_offset, position_offset + seq_len, device=device)
    return qpos[:, None] >= key_positions[None, :]


def _masked_attention(q, k, v, seq_len, position_offset, padding_mask, key_positions):
    """softmax(q k^T / sqrt(hd), masked) v -- engine/model.py:99-116.

    q: [B, Hq, S, hd]; k, v: [B, Hk, T, hd] with Hq a multiple of Hk (grouped
    query heads share a key/value head).
    """
    batch, n_q, _, hd = q.shape
    n_kv = k.shape[1]
    if n_kv != n_q:
        rep = n_q // n_kv
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    total = k.shape[2]
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(hd)
    allowed = build_causal_mask(seq_len, total, position_offset, q.device, key_positions)
    allowed = allowed.view(batch, 1, seq_len, total) if allowed.dim() == 3 else allowed.view(1, 1, seq_len, total)
    if padding_mask is not None:
        allowed = allowed & padding_mask.view(batch, 1, 1, total)
    weights = F.softmax(scores.masked_fill(~allowed, float("-inf")), dim=-1)
    return weights @ v


class CausalSelfAttention(nn.Module):
    """engine/model.py:67-118 (fused qkv Linear with bias, out Linear)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model)
        self.out = nn.Linear(cfg.d_model, cfg.d_model)

    def forward(self, x, past_kv, position_offset, padding_mask, key_positions=None):
        batch, seq_len, _ = x.shape
        heads = [t.view(batch, seq_len, self.n_heads, self.head_dim).transpose(1, 2)
                 for t in self.qkv(x).chunk(3, dim=-1)]
        q, k, v = heads
        if past_kv is not None:
            k = torch.cat([past_kv[0], k], dim=2)
            v = torch.cat([past_kv[1], v], dim=2)
        o = _masked_attention(q, k, v, seq_len, position_offset, padding_mask, key_positions)
        o = o.transpose(1, 2).reshape(batch, seq_len, self.n_heads * self.head_dim)
        return self.out(o), (k, v)


class Block(nn.Module):
    """Pre-LN block with GELU MLP, engine/model.py:121-142."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = CausalSelfAttention(cfg)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.mlp = nn.Sequential(nn.Linear(cfg.d_model, cfg.d_ff), nn.GELU(), nn.Linear(cfg.d_ff, cfg.d_model))

    def forward(self, x, past_kv, position_offset, padding_mask, key_positions=None):
        a, kv = self.attn(self.ln1(x), past_kv, position_offset, padding_mask, key_positions)
        x = x + a
        return x + self.mlp(self.ln2(x)), kv


class TinyGPT(nn.Module):
    """engine/model.py:145-206: learned positions, untied lm_head without bias."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.pos_emb = nn.Embedding(cfg.max_seq_len, cfg.d_model)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layers)])
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)

    def _positions(self, input_ids, position_offset):
        seq_len = input_ids.shape[1]
        steps = torch.arange(seq_len, device=input_ids.device)
        if isinstance(position_offset, torch.Tensor):
            return position_offset.view(-1, 1) + steps.view(1, -1)
        return (position_offset + steps).unsqueeze(0)

    def forward(self, input_ids, past_kv=None, position_offset=0, padding_mask=None, key_positions=None):
        seq_len = input_ids.shape[1]
        x = self.token_emb(input_ids) + self.pos_emb(self._positions(input_ids, position_offset))
        # engine/model.py:183-201: padded query rows are zeroed after every block.
        valid = padding_mask[:, -seq_len:].unsqueeze(-1) if padding_mask is not None else None
        if valid is not None:
            x = x * valid
        new_kv = []
        for i, block in enumerate(self.blocks):
            x, kv = block(x, None if past_kv is None else past_kv[i], position_offset, padding_mask, key_positions)
            if valid is not None:
                x = x * valid
            new_kv.append(kv)
        return self.lm_head(self.ln_f(x)), new_kv


# ---------------------------------------------------------------------------
# Llama-style model (GQA + RoPE + SwiGLU + RMSNorm); no reference counterpart.
# ---------------------------------------------------------------------------

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


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


def rope_rotate(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half RoPE.  x: [B, H, S, hd]; positions: [B, S] (absolute)."""
    hd = x.shape[-1]
    half = hd // 2
    inv_freq = theta ** (-torch.arange(0, half, dtype=torch.float64) * 2.0 / hd)
    ang = positions.to(torch.float64)[..., None] * inv_freq  # [B, S, half]
    cos = torch.cos(ang).to(torch.float32)[:, None]
    sin = torch.sin(ang).to(torch.float32)[:, None]
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


class LlamaAttention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0 and cfg.n_heads % cfg.n_kv_heads == 0
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.theta = cfg.rope_theta
        self.qkv = nn.Linear(cfg.d_model, (cfg.n_heads + 2 * cfg.n_kv_heads) * self.head_dim, bias=False)
        self.out = nn.Linear(cfg.n_heads * self.head_dim, cfg.d_model, bias=False)

    def forward(self, x, past_kv, position_offset, padding_mask, key_positions=None):
        batch, seq_len, _ = x.shape
        hd = self.head_dim
        qkv = self.qkv(x)
        nq, nk = self.n_heads * hd, self.n_kv_heads * hd
        q = qkv[..., :nq].view(batch, seq_len, self.n_heads, hd).transpose(1, 2)
        k = qkv[..., nq:nq + nk].view(batch, seq_len, self.n_kv_heads, hd).transpose(1, 2)
        v = qkv[..., nq + nk:].view(batch, seq_len, self.n_kv_heads, hd).transpose(1, 2)
        if isinstance(position_offset, torch.Tensor):
            pos = position_offset.view(-1, 1) + torch.arange(seq_len).view(1, -1)
        else:
            pos = (position_offset + torch.arange(seq_len)).view(1, -1).expand(batch, -1)
        q = rope_rotate(q, pos, self.theta)
        k = rope_rotate(k, pos, self.theta)
        if past_kv is not None:
            k = torch.cat([past_kv[0], k], dim=2)
            v = torch.cat([past_kv[1], v], dim=2)
        o = _masked_attention(q, k, v, seq_len, position_offset, padding_mask, key_positions)
        o = o.transpose(1, 2).reshape(batch, seq_len, self.n_heads * hd)
        return self.out(o), (k, v)


class LlamaBlock(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.norm1 = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.attn = LlamaAttention(cfg)
        self.norm2 = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.gate_up = nn.Linear(cfg.d_model, 2 * cfg.d_ff, bias=False)
        self.down = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)

    def forward(self, x, past_kv, position_offset, padding_mask, key_positions=None):
        a, kv = self.attn(self.norm1(x), past_kv, position_offset, padding_mask, key_positions)
        x = x + a
        gate, up = self.gate_up(self.norm2(x)).chunk(2, dim=-1)
        return x + self.down(F.silu(gate) * up), kv


class TinyLlama(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.blocks = nn.ModuleList([LlamaBlock(cfg) for _ in range(cfg.n_layers)])
        self.norm_f = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)

    def forward(self, input_ids, past_kv=None, position_offset=0, padding_mask=None, key_positions=None):
        seq_len = input_ids.shape[1]
        x = self.token_emb(input_ids)
        valid = padding_mask[:, -seq_len:].unsqueeze(-1) if padding_mask is not None else None
        if valid is not None:
            x = x * valid
        new_kv = []
        for i, block in enumerate(self.blocks):
            x, kv = block(x, None if past_kv is None else past_kv[i], position_offset, padding_mask, key_positions)
            if valid is not None:
                x = x * valid
            new_kv.append(kv)
        return self.lm_head(self.norm_f(x)), new_kv
