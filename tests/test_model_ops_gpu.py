"""Model-piece kernels against plain PyTorch fp32 references.  GPU only.

``pse_add_norm`` (fused residual add + LayerNorm / RMSNorm, engine/model.py:
139-142 pre-LN blocks): the bf16 vector path (8 columns per thread), the
scalar path (fp32, and bf16 rows whose stride rules the vector path out), with
and without the residual input, bias and beta.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
F32_TOL = 1e-4


def _N():
    from pse import _native as N
    N.load()
    return N


def _ref(x, y, bias, gamma, beta, eps, rms):
    v = x.clone()
    if y is not None:
        v = v + (y.float() + (bias.float() if bias is not None else 0.0))
    if rms:
        o = v * torch.rsqrt((v * v).mean(-1, keepdim=True) + eps) * gamma.float()
    else:
        o = torch.nn.functional.layer_norm(v, (v.shape[-1],), gamma.float(),
                                           beta.float() if beta is not None else None, eps)
    return v, o


@pytest.mark.parametrize("d", [64, 384, 768, 1000, 2048, 4096])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("variant", ["full", "no_residual", "rms", "padded_rows"])
def test_add_norm_matches_torch(d, dtype, variant):
    N = _N()
    g = torch.Generator().manual_seed(d)
    rows = 37
    rms = variant == "rms"
    pad = 8 if variant == "padded_rows" else 0
    if pad and dtype == torch.bfloat16:
        pad = 3  # odd stride: the scalar path
    x = torch.randn(rows, d + pad, generator=g).cuda()
    xv = x[:, :d]
    y = None if variant == "no_residual" else (torch.randn(rows, d + pad, generator=g) * 2).to(dtype).cuda()[:, :d]
    bias = None if variant in ("no_residual", "rms") else torch.randn(d, generator=g).to(dtype).cuda()
    gamma = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype).cuda()
    beta = None if rms else (0.1 * torch.randn(d, generator=g)).to(dtype).cuda()
    out = torch.full((rows, d + pad), float("nan"), dtype=dtype, device="cuda")
    want_x, want = _ref(xv.clone(), y, bias, gamma, beta, 1e-5, rms)
    dt = N.PSE_BF16 if dtype == torch.bfloat16 else N.PSE_F32
    N.call("pse_add_norm", xv.data_ptr(), x.stride(0), None if y is None else y.data_ptr(),
           0 if y is None else y.stride(0), None if bias is None else bias.data_ptr(), dt, gamma.data_ptr(),
           None if beta is None else beta.data_ptr(), dt, rows, d, 1e-5, int(rms), out.data_ptr(), out.stride(0),
           dt, N.stream_ptr())
    torch.cuda.synchronize()
    tol = BF16_TOL if dtype == torch.bfloat16 else F32_TOL
    assert (xv - want_x).abs().max().item() <= 1e-6  # the residual stream: same fp32 additions
    got = out[:, :d].float()
    assert torch.isfinite(got).all()
    assert (got - want).abs().max().item() < tol
    if pad:
        assert torch.isnan(out[:, d:].float()).all()  # nothing written past the row


@pytest.mark.parametrize("d,pos,dtype", [(768, True, torch.bfloat16), (2048, False, torch.bfloat16),
                                         (100, True, torch.bfloat16), (384, True, torch.float32)])
def test_embed_matches_torch(d, pos, dtype):
    """``pse_embed`` / ``pse_embed_pos`` (engine/model.py:175-181: token plus
    learned position embedding) equal the fp32 sum of the table rows exactly:
    the bf16 vector path (d a multiple of 8), the scalar path (other d, fp32
    tables); ids and positions out of range read as zero rows."""
    N = _N()
    g = torch.Generator(device="cuda").manual_seed(d)
    vocab, n_pos, rows, width = 1000, 300, 37, 3
    tok = torch.randn(vocab, d, device="cuda", generator=g).to(dtype)
    pe = torch.randn(n_pos, d, device="cuda", generator=g).to(dtype) if pos else None
    ids = torch.randint(0, vocab, (rows * width,), device="cuda", generator=g, dtype=torch.int32)
    ids[5] = vocab + 7  # out of range: no token row
    base = torch.randint(0, n_pos - width, (rows,), device="cuda", generator=g, dtype=torch.int32)
    base[3] = n_pos  # every position of row 3 out of range: no position row
    x = torch.full((rows * width, d), float("nan"), device="cuda")
    dt = N.dtype_code(dtype)
    N.call("pse_embed", ids.data_ptr(), base.data_ptr(), rows, width, tok.data_ptr(),
           None if pe is None else pe.data_ptr(), d, dt, vocab, n_pos, x.data_ptr(), N.stream_ptr())
    positions = (base.view(-1, 1).long() + torch.arange(width, device="cuda").view(1, -1)).reshape(-1)
    want = torch.where((ids.long() < vocab).view(-1, 1), tok.float()[ids.long().clamp(max=vocab - 1)],
                       torch.zeros((), device="cuda"))
    if pe is not None:
        ok = (positions < n_pos).view(-1, 1)
        want = want + torch.where(ok, pe.float()[positions.clamp(max=n_pos - 1)], torch.zeros((), device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(x, want)
    x2 = torch.full_like(x, float("nan"))
    pos32 = positions.to(torch.int32)
    N.call("pse_embed_pos", ids.data_ptr(), pos32.data_ptr(), rows, width, tok.data_ptr(),
           None if pe is None else pe.data_ptr(), d, dt, vocab, n_pos, x2.data_ptr(), N.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(x2, want)
