"""Device copy of a model's weights in the engine's compute dtype.

Accepts any module with the TinyGPT layout (engine/model.py:145-156; the
reference's own objects included) or the TinyLlama layout of ``pse.model``.
Weights are snapshotted on first use per (dtype, device); call
``refresh(model)`` after changing a model's parameters.
"""
from __future__ import annotations

import weakref
from dataclasses import dataclass, field

import torch


@dataclass
class DeviceLayer:
    norm1_w: torch.Tensor
    norm1_b: torch.Tensor | None
    qkv_w: torch.Tensor
    qkv_b: torch.Tensor | None
    out_w: torch.Tensor
    out_b: torch.Tensor | None
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor | None
    up_w: torch.Tensor          # GELU MLP: [d_ff, d]; SwiGLU: gate_up [2*d_ff, d]
    up_b: torch.Tensor | None
    down_w: torch.Tensor
    down_b: torch.Tensor | None


@dataclass(eq=False)
class DeviceModel:
    kind: str                   # "gpt" | "llama"
    vocab: int
    d_model: int
    n_layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    d_ff: int
    max_seq_len: int
    eps: float
    rope_theta: float
    dtype: torch.dtype
    device: torch.device
    tok_emb: torch.Tensor
    pos_emb: torch.Tensor | None
    layers: list = field(default_factory=list)
    normf_w: torch.Tensor | None = None
    normf_b: torch.Tensor | None = None
    lm_w: torch.Tensor | None = None

    @property
    def qkv_width(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim

    @property
    def kv_bytes_per_token(self) -> int:
        return 2 * self.n_layers * self.kv_heads * self.head_dim * torch.finfo(self.dtype).bits // 8

    def weight_bytes(self, lm_head: bool = True) -> int:
        n = 0
        for L in self.layers:
            for t in (L.qkv_w, L.qkv_b, L.out_w, L.out_b, L.up_w, L.up_b, L.down_w, L.down_b,
                      L.norm1_w, L.norm1_b, L.norm2_w, L.norm2_b):
                if t is not None:
                    n += t.numel() * t.element_size()
        if lm_head and self.lm_w is not None:
            n += self.lm_w.numel() * self.lm_w.element_size()
        return n


_cache: "weakref.WeakKeyDictionary[torch.nn.Module, dict]" = weakref.WeakKeyDictionary()


def _cvt(t, dtype, device):
    return None if t is None else t.detach().to(device=device, dtype=dtype).contiguous()


def _build(model: torch.nn.Module, dtype: torch.dtype, device: torch.device) -> DeviceModel:
    cfg = model.cfg
    blocks = list(model.blocks)
    if hasattr(model, "pos_emb"):
        a0 = blocks[0].attn
        dm = DeviceModel(
            kind="gpt", vocab=cfg.vocab_size, d_model=cfg.d_model, n_layers=len(blocks),
            q_heads=a0.n_heads, kv_heads=a0.n_heads, head_dim=a0.head_dim, d_ff=cfg.d_ff,
            max_seq_len=cfg.max_seq_len, eps=blocks[0].ln1.eps, rope_theta=0.0, dtype=dtype, device=device,
            tok_emb=_cvt(model.token_emb.weight, dtype, device), pos_emb=_cvt(model.pos_emb.weight, dtype, device),
        )
        for b in blocks:
            dm.layers.append(DeviceLayer(
                _cvt(b.ln1.weight, dtype, device), _cvt(b.ln1.bias, dtype, device),
                _cvt(b.attn.qkv.weight, dtype, device), _cvt(b.attn.qkv.bias, dtype, device),
                _cvt(b.attn.out.weight, dtype, device), _cvt(b.attn.out.bias, dtype, device),
                _cvt(b.ln2.weight, dtype, device), _cvt(b.ln2.bias, dtype, device),
                _cvt(b.mlp[0].weight, dtype, device), _cvt(b.mlp[0].bias, dtype, device),
                _cvt(b.mlp[2].weight, dtype, device), _cvt(b.mlp[2].bias, dtype, device),
            ))
        dm.normf_w = _cvt(model.ln_f.weight, dtype, device)
        dm.normf_b = _cvt(model.ln_f.bias, dtype, device)
    else:
        a0 = blocks[0].attn
        dm = DeviceModel(
            kind="llama", vocab=cfg.vocab_size, d_model=cfg.d_model, n_layers=len(blocks),
            q_heads=a0.n_heads, kv_heads=a0.n_kv_heads, head_dim=a0.head_dim, d_ff=cfg.d_ff,
            max_seq_len=cfg.max_seq_len, eps=cfg.norm_eps, rope_theta=cfg.rope_theta, dtype=dtype, device=device,
            tok_emb=_cvt(model.token_emb.weight, dtype, device), pos_emb=None,
        )
        for b in blocks:
            dm.layers.append(DeviceLayer(
                _cvt(b.norm1.weight, dtype, device), None,
                _cvt(b.attn.qkv.weight, dtype, device), None,
                _cvt(b.attn.out.weight, dtype, device), None,
                _cvt(b.norm2.weight, dtype, device), None,
                _cvt(b.gate_up.weight, dtype, device), None,
                _cvt(b.down.weight, dtype, device), None,
            ))
        dm.normf_w = _cvt(model.norm_f.weight, dtype, device)
    dm.lm_w = _cvt(model.lm_head.weight, dtype, device)
    return dm


def device_model(model: torch.nn.Module, dtype: torch.dtype, device) -> DeviceModel:
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if isinstance(model, DeviceModel):
        return model
    per = _cache.get(model)
    if per is None:
        per = {}
        _cache[model] = per
    key = (dtype, device)
    dm = per.get(key)
    if dm is None:
        with torch.no_grad():
            dm = _build(model, dtype, device)
        per[key] = dm
    return dm


def refresh(model: torch.nn.Module) -> None:
    _cache.pop(model, None)
