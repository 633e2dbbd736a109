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
    (1536, 768, 768, True, 0, False),    # verify out projection: 64-column tiles
    (1536, 768, 3072, True, 0, False),   # verify MLP down: 64-column tiles, long k
    (512, 1536, 384, True, 1, False),    # draft width-2 call, MLP up + GELU
    (1536, 32000, 768, False, 0, True),  # verify lm_head: ~10 tiles per CTA, both accumulators in turn
    (2560, 16384, 2048, False, 0, False),  # Llama-style gate+up
]


@pytest.fixture(params=[1, 0], ids=["pair-tiles", "single-cta"])
def pair_tiles(request):
    from pse import _native as N
    lib = N.load()
    lib.pse_gemm_pair_tiles(request.param)
    yield request.param
    lib.pse_gemm_pair_tiles(1)


@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_matches_fp32_reference(shape, pair_tiles):
    """Wide shapes run the two-SM kernel when pair tiles are on and the
    single-CTA kernel when off; both must match."""
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


def test_gemm_chain_reads_the_previous_output(pair_tiles):
    """Back-to-back calls on one stream, each reading the previous call's
    output: the second call may start while the first finishes (programmatic
    dependent launch) and must still see all of its output."""
    from pse import _native as N
    N.load()
    g = torch.Generator(device="cuda").manual_seed(3)
    m, d, f = 1536, 768, 3072
    x = (torch.randn(m, d, device="cuda", generator=g) / d ** 0.5).bfloat16()
    w1 = (torch.randn(f, d, device="cuda", generator=g) / d ** 0.5).bfloat16()
    w2 = (torch.randn(d, f, device="cuda", generator=g) / f ** 0.5).bfloat16()
    h = torch.full((m, f), float("nan"), device="cuda", dtype=torch.bfloat16)
    y = torch.full((m, d), float("nan"), device="cuda", dtype=torch.bfloat16)
    st = N.stream_ptr()
    for _ in range(3):
        N.call("pse_gemm_bf16", x.data_ptr(), d, w1.data_ptr(), d, None, h.data_ptr(), f, m, f, d, 1, 0, None, st)
        N.call("pse_gemm_bf16", h.data_ptr(), f, w2.data_ptr(), f, None, y.data_ptr(), d, m, d, f, 0, 0, None, st)
    torch.cuda.synchronize()
    ref_h = torch.nn.functional.gelu(x.float() @ w1.float().t()).bfloat16()
    ref = ref_h.float() @ w2.float().t()
    assert ((h.float() - ref_h.float()).abs() <= 1e-3 + 8e-3 * ref_h.float().abs()).all()
    assert ((y.float() - ref).abs() <= 3e-3 + 8e-3 * ref.abs()).all(), (y.float() - ref).abs().max().item()
