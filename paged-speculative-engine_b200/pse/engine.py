"""The paged forward and the device-resident speculative step.

One forward of width W over B rows (engine/batched_forward.py:27-72 and
engine/model.py:158-206, re-planned for the device):

    reserve blocks for W tokens per row (pse_kv_reserve, rows in call order)
    x = tok_emb[ids] + pos_emb[len + w]                       (pse_embed)
    per layer:
        h = norm1(x)                                          (pse_norm)
        qkv = h Wqkv^T + b                                    (GEMM)
        [rope on q, k]                                        (pse_rope, Llama layout)
        K, V -> their blocks                                  (pse_kv_append)
        a = paged attention of q over the row's blocks        (pse_paged_attention)
        x += a Wo^T + bo                                      (GEMM + pse_epilogue)
        h = norm2(x); u = act(h W1^T + b1); x += u W2^T + b2  (GEMM + pse_epilogue)
    logits = norm_f(x) Wlm^T                                  (GEMM, fp32 out)

The residual stream is fp32; GEMM operands, K/V and attention run in the
cache dtype (fp32 or bf16).  No step synchronises the host.

The speculative step (engine/speculative.py:77-177) runs k width-1 draft
forwards with a sampling kernel between them, one width-k verify forward,
the fused accept kernel, the batched truncate of both caches and the two
width-1 bonus forwards -- all on the device, optionally replayed from a CUDA
graph -- and returns with one device->host copy of the accepted tokens.
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from .device_model import DeviceModel


class Scratch:
    """Activation buffers of one model, grown on demand (never inside a capture)."""

    def __init__(self, dm: DeviceModel):
        self.dm = dm
        self.cap = 0
        self.generation = 0  # bumped on every reallocation (captured graphs hold the old pointers)
        self.ws = torch.empty(0, dtype=torch.uint8, device=dm.device)
        self.base_len = torch.empty(0, dtype=torch.int32, device=dm.device)

    def ensure(self, tokens: int) -> None:
        if tokens <= self.cap:
            return
        cap = max(tokens, 2 * self.cap, 16)
        dm, dev, dt = self.dm, self.dm.device, self.dm.dtype
        self.x = torch.empty(cap, dm.d_model, dtype=torch.float32, device=dev)
        self.h = torch.empty(cap, dm.d_model, dtype=dt, device=dev)
        self.qkv = torch.empty(cap, dm.qkv_width, dtype=dt, device=dev)
        self.attn = torch.empty(cap, dm.q_heads * dm.head_dim, dtype=dt, device=dev)
        self.tmp = torch.empty(cap, dm.d_model, dtype=dt, device=dev)
        up = 2 * dm.d_ff if dm.kind == "llama" else dm.d_ff
        self.up = torch.empty(cap, up, dtype=dt, device=dev)
        self.act = torch.empty(cap, dm.d_ff, dtype=dt, device=dev) if dm.kind == "llama" else self.up
        self.cap = cap
        self.generation += 1

    def ensure_ws(self, nbytes: int) -> None:
        if nbytes > self.ws.numel():
            # zeroed: its first 256 bytes are the attention kernel's work counters (left zero by every call)
            self.ws = torch.zeros(max(nbytes, 2 * self.ws.numel()), dtype=torch.uint8, device=self.dm.device)
            self.generation += 1


def scratch_for(dm: DeviceModel) -> Scratch:
    """The shared scratch of a device model (prefill and plain forwards)."""
    s = dm.__dict__.get("_scratch")
    if s is None:
        s = dm.__dict__["_scratch"] = Scratch(dm)
    return s


# bf16 projections on the tcgen05 GEMM (pse_gemm_bf16): False (cuBLAS), True
# (every projection), or "gelu" (only the MLP up-projections, whose GELU the
# GEMM applies in its epilogue instead of a separate kernel after cuBLAS)
USE_TC_GEMM = False
TC_GEMM_MAX_ROWS = 1 << 30  # with USE_TC_GEMM: only GEMMs of at most this many rows


def _tc_ok(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, gelu: bool = False) -> bool:
    """pse_gemm_bf16 takes bf16 operands, k in whole 64-element slabs, row
    pitches in 16-byte units and 16-byte aligned bases."""
    if not USE_TC_GEMM or (USE_TC_GEMM == "gelu" and not gelu):
        return False
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or a.shape[0] > TC_GEMM_MAX_ROWS:
        return False
    k = a.shape[1]
    esz = out.element_size()
    return (k % 64 == 0 and a.stride(1) == 1 and w.stride(1) == 1 and out.stride(1) == 1
            and a.stride(0) % 8 == 0 and w.stride(0) % 8 == 0 and (out.stride(0) * esz) % 16 == 0
            and a.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0 and out.data_ptr() % 16 == 0)


def _mm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, bias: torch.Tensor | None = None,
        gelu: bool = False) -> bool:
    """out = a @ w^T (+ bias).  With ``gelu`` the tensor-core path also applies
    GELU; returns whether it did (the cuBLAS fallback never does)."""
    if _tc_ok(a, w, out, gelu):
        N.call("pse_gemm_bf16", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), N.ptr(bias), out.data_ptr(),
               out.stride(0), a.shape[0], w.shape[0], a.shape[1], 1 if gelu else 0,
               1 if out.dtype == torch.float32 else 0, None, N.stream_ptr())
        return gelu
    if bias is not None:
        torch.addmm(bias, a, w.t(), out=out)
    else:
        torch.mm(a, w.t(), out=out)
    return False


def lm_head(dm: DeviceModel, h: torch.Tensor, out: torch.Tensor) -> None:
    """fp32 logits from the final normed hidden rows."""
    if dm.dtype == torch.float32:
        torch.mm(h, dm.lm_w.t(), out=out)
    elif _tc_ok(h, dm.lm_w, out):
        _mm(h, dm.lm_w, out)
    else:
        torch.mm(h, dm.lm_w.t(), out_dtype=torch.float32, out=out)  # bf16 in, fp32 logits out, no temporary


def forward(dm: DeviceModel, cache, slots: torch.Tensor, ids: torch.Tensor, rows: int, width: int,
            base_len: torch.Tensor, max_ctx: int, logits_out: torch.Tensor | None, last_only: bool = False,
            scratch: Scratch | None = None, row_order: torch.Tensor | None = None, reserve: bool = True,
            tree: tuple | None = None) -> None:
    """One paged forward.  ``slots`` int32 [rows]; ``ids`` int32 [rows*width];
    ``base_len`` int32 [rows] receives the rows' lengths before the call;
    ``max_ctx`` >= every row's length after it.  ``logits_out`` fp32
    [rows*width, V] (or [rows, V] with ``last_only``) or None.  With
    ``reserve=False`` nothing is allocated: ``base_len`` gives each row's first
    position, and K/V of positions in blocks the row does not hold are dropped.
    ``tree=(b, d0)``: the call's tokens are token-tree nodes of b branches in
    depth-major order from depth d0 (``pse_paged_attention_tree``): node
    positions are the row's root length plus the node's depth, and each node
    attends to the root context and its own branch.  The final normed hidden
    rows stay in the scratch's ``h``."""
    T = rows * width
    sc = scratch or scratch_for(dm)
    sc.ensure(T)
    st = N.stream_ptr()
    state = cache.state
    dt = N.dtype_code(dm.dtype)
    d, hd = dm.d_model, dm.head_dim
    nq, nk = dm.q_heads * hd, dm.kv_heads * hd
    if reserve:
        N.call("pse_kv_reserve", state, slots.data_ptr(), rows, width, base_len.data_ptr(), st)
    x, h, qkv, attn, tmp, up, act = (sc.x[:T], sc.h[:T], sc.qkv[:T], sc.attn[:T], sc.tmp[:T], sc.up[:T],
                                      sc.act[:T])
    pos = None
    if tree is not None:
        tb, td0 = tree
        off = (td0 * tb + torch.arange(width, device=base_len.device)) // tb - td0 * tb
        pos = (base_len.view(-1, 1).long() + off.view(1, -1)).to(torch.int32).reshape(-1)
        N.call("pse_embed_pos", ids.data_ptr(), pos.data_ptr(), rows, width, dm.tok_emb.data_ptr(),
               None if dm.pos_emb is None else dm.pos_emb.data_ptr(), d, dt, dm.vocab,
               0 if dm.pos_emb is None else dm.pos_emb.shape[0], x.data_ptr(), st)
    else:
        N.call("pse_embed", ids.data_ptr(), base_len.data_ptr(), rows, width, dm.tok_emb.data_ptr(),
               None if dm.pos_emb is None else dm.pos_emb.data_ptr(), d, dt, dm.vocab,
               0 if dm.pos_emb is None else dm.pos_emb.shape[0], x.data_ptr(), st)
    ws_bytes = N.size_call("pse_paged_attention_workspace", rows, width, dm.q_heads, dm.kv_heads, hd, max_ctx)
    sc.ensure_ws(ws_bytes)
    scale = 1.0 / math.sqrt(hd)
    rms = 1 if dm.kind == "llama" else 0
    L0 = dm.layers[0]
    N.call("pse_add_norm", x.data_ptr(), d, None, 0, None, dt, L0.norm1_w.data_ptr(), N.ptr(L0.norm1_b), dt, T, d,
           dm.eps, rms, h.data_ptr(), d, dt, st)
    n_layers = len(dm.layers)
    for li, L in enumerate(dm.layers):
        _mm(h, L.qkv_w, qkv, L.qkv_b)
        if dm.kind == "llama" and pos is not None:
            N.call("pse_rope_pos", qkv.data_ptr(), qkv.stride(0), rows, width, dm.q_heads, dm.kv_heads, hd,
                   pos.data_ptr(), dm.rope_theta, dt, st)
        elif dm.kind == "llama":
            N.call("pse_rope", qkv.data_ptr(), qkv.stride(0), rows, width, dm.q_heads, dm.kv_heads, hd,
                   base_len.data_ptr(), dm.rope_theta, dt, st)
        kvl = cache.layer(li)
        N.call("pse_kv_append", state, kvl, qkv.data_ptr() + nq * qkv.element_size(),
               qkv.data_ptr() + (nq + nk) * qkv.element_size(), qkv.stride(0), hd, slots.data_ptr(),
               base_len.data_ptr(), rows, width, st)
        if tree is not None:
            N.call("pse_paged_attention_tree", state, kvl, qkv.data_ptr(), qkv.stride(0), attn.data_ptr(),
                   attn.stride(0), slots.data_ptr(), base_len.data_ptr(), rows, width, dm.q_heads, scale, max_ctx,
                   N.ptr(row_order), sc.ws.data_ptr(), sc.ws.numel(), tree[0], tree[1], st)
        else:
            N.call("pse_paged_attention", state, kvl, qkv.data_ptr(), qkv.stride(0), attn.data_ptr(),
                   attn.stride(0), slots.data_ptr(), base_len.data_ptr(), rows, width, dm.q_heads, scale, max_ctx,
                   N.ptr(row_order), sc.ws.data_ptr(), sc.ws.numel(), st)
        _mm(attn, L.out_w, tmp, L.out_b)
        # x += attn-out (bias already added by the GEMM); h = norm2(x)
        N.call("pse_add_norm", x.data_ptr(), d, tmp.data_ptr(), d, None, dt, L.norm2_w.data_ptr(),
               N.ptr(L.norm2_b), dt, T, d, dm.eps, rms, h.data_ptr(), d, dt, st)
        if dm.kind == "llama":
            _mm(h, L.up_w, up)
            N.call("pse_epilogue", 2, up.data_ptr(), up.stride(0), None, None, 0, act.data_ptr(), act.stride(0),
                   T, dm.d_ff, dt, st)
        elif not _mm(h, L.up_w, up, L.up_b, gelu=True):
            N.call("pse_epilogue", 0, up.data_ptr(), up.stride(0), None, None, 0, None, 0, T, dm.d_ff, dt, st)
        _mm(act, L.down_w, tmp, L.down_b)
        # x += mlp-out (+ bias); h = next layer's norm1(x), or the final norm after the last layer
        if li + 1 < n_layers:
            nw, nb = dm.layers[li + 1].norm1_w, dm.layers[li + 1].norm1_b
        else:
            nw, nb = dm.normf_w, dm.normf_b
        N.call("pse_add_norm", x.data_ptr(), d, tmp.data_ptr(), d, None, dt, nw.data_ptr(), N.ptr(nb), dt, T, d,
               dm.eps, rms, h.data_ptr(), d, dt, st)
    if logits_out is None:
        return
    hf = h.view(rows, width, d)[:, width - 1] if last_only else h
    lm_head(dm, hf, logits_out)
