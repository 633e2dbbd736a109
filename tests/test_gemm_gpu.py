"""tcgen05 projection GEMM (pse_gemm_bf16) against a torch fp32 reference of
the same bf16 operands.  Tolerance: the bf16 rounding of the output (relative
2^-8) plus fp32 accumulation-order noise.  GPU only."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [
    # m, n, k, bias, act, out_f32
    (128, 128, 64, False, 0, False),     # one tile, one k-slab
    (256, 1152, 384, True, 0, False),    # draft qkv
    (1536, 2304, 768, True, 0, False),   # target verify qkv (width 6 x 256 rows)
    (300, 200, 128, True, 0, False),     # ragged m and n
    (1280, 3072, 768, True, 1, False),   # MLP up + bias + GELU
    (256, 768, 3072, False, 0, False),   # MLP down, long k
    (96, 32000, 768, False, 0, True),    # lm_head, fp32 logits
    (17, 16384, 2048, False, 0, False),  # few rows, wide n
]


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_matches_fp32_reference(shape):
    from pse import _native as N
    N.load()
    m, n, k, has_bias, act, out_f32 = shape
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    a = (torch.randn(m, k, device="cuda", generator=g) / k ** 0.5).bfloat16()
    w = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    bias = torch.randn(n, device="cuda", generator=g).bfloat16() if has_bias else None
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32 if out_f32 else torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.call("pse_gemm_bf16", a.data_ptr(), k, w.data_ptr(), k, N.ptr(bias), c.data_ptr(), n, m, n, k, act,
           1 if out_f32 else 0, status.data_ptr(), N.stream_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = a.float() @ w.float().t()
    if bias is not None:
        ref = ref + bias.float()
    if act == 1:
        ref = torch.nn.functional.gelu(ref)
    got = c.float()
    assert torch.isfinite(got).all()
    tol = 1e-3 + (0 if out_f32 else 1) * 8e-3 * ref.abs()
    assert ((got - ref).abs() <= tol + 2e-3).all(), (got - ref).abs().max().item()


def test_gemm_rejects_unsupported_shapes():
    from pse import _native as N
    lib = N.load()
    a = torch.zeros(8, 48, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 48, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(8, 8, device="cuda", dtype=torch.bfloat16)
    rc = lib.pse_gemm_bf16(a.data_ptr(), 48, w.data_ptr(), 48, None, c.data_ptr(), 8, 8, 8, 48, 0, 0, None,
                           N.stream_ptr())
    assert rc == 10001  # k not a multiple of 64
