"""SSM prefill front end (SiLU + depthwise causal conv + split, conv-context capture)
against the reference's own code (golden vectors from its ``SSM.conv`` layer and
``SSMCache.build_conv_ctx``) and the CPU restatement ``oracle/ssm_front_ref.py``.

Tolerances: fp32 rel 1e-4 (assert_fp32_close); 16-bit atol 2e-2 / rel 1e-2
(assert_bf16_close); the conv context is a copy of inputs and must match exactly."""
import pytest
import torch

from conftest import assert_bf16_close, assert_close_for, assert_fp32_close, load_golden
from oracle import ssm_front_ref

FRONT_CASES = ["ssm_front_fp32", "ssm_front_fp32_short", "ssm_front_bf16"]


@pytest.mark.parametrize("case", FRONT_CASES)
def test_oracle_matches_reference_golden(case):
    g = load_golden(case)
    hBC = g["hBC"]
    act = None if hBC.dtype == torch.float32 else hBC.dtype
    x, B, C, ctx = ssm_front_ref.prefill_front(hBC, g["weight"], g["bias"], g["inner"], g["gn"], g["lengths"],
                                               act_dtype=act)
    close = assert_close_for(hBC.dtype)
    close(x, g["x"].float(), f"{case} x")
    close(B, g["B"].float(), f"{case} B")
    close(C, g["C"].float(), f"{case} C")
    assert torch.equal(ctx, g["conv_ctx"])


def _run(hBC, weight, bias, inner, gn, lengths=None, build_ctx=True):
    from selective_attention_b200 import kernels

    out = kernels.ssm_conv_prefill(hBC, weight, bias, inner, gn, lengths=lengths, build_ctx=build_ctx)
    torch.cuda.synchronize()
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("case", FRONT_CASES)
def test_kernel_matches_reference_golden(case):
    g = load_golden(case)
    lengths = None if g["lengths"] is None else g["lengths"].cuda()
    x, B, C, ctx = _run(g["hBC"].cuda(), g["weight"].cuda(), g["bias"].cuda(), g["inner"], g["gn"], lengths)
    close = assert_close_for(g["hBC"].dtype)
    close(x.float(), g["x"].float(), f"{case} x")
    close(B.float(), g["B"].float(), f"{case} B")
    close(C.float(), g["C"].float(), f"{case} C")
    assert torch.equal(ctx.cpu(), g["conv_ctx"])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_kernel_on_projection_slice_vs_oracle(dtype):
    """c1-like widths (inner 1536, G*N 128, K 4) read from a slice of a wider projection
    output (token stride > conv_dim), ragged lengths for the conv context."""
    g = torch.Generator().manual_seed(3)
    b, L, inner, gn, K = 3, 700, 1536, 128, 4
    conv_dim = inner + 2 * gn
    proj = torch.randn(b, L, conv_dim + inner + 24, generator=g).to(dtype)
    hBC = proj[..., :conv_dim]
    w = torch.randn(conv_dim, 1, K, generator=g) * 0.5
    bias = torch.randn(conv_dim, generator=g) * 0.1
    lengths = torch.tensor([700, 513, 2])
    x, B, C, ctx = _run(proj.cuda()[..., :conv_dim], w.cuda(), bias.cuda(), inner, gn, lengths.cuda())
    act = None if dtype == torch.float32 else dtype
    xr, Br, Cr, ctxr = ssm_front_ref.prefill_front(hBC, w, bias, inner, gn, lengths, act_dtype=act)
    close = assert_close_for(dtype)
    assert x.dtype == dtype and x.shape == (b, L, inner) and B.shape == (b, L, gn) and x.is_contiguous()
    close(x.float(), xr, f"{dtype} x")
    close(B.float(), Br, f"{dtype} B")
    close(C.float(), Cr, f"{dtype} C")
    assert torch.equal(ctx.cpu(), ctxr)


@pytest.mark.gpu
def test_kernel_scalar_path_odd_widths_short_kernel():
    """Widths that do not split on 8 bytes take the one-channel-per-thread path; K = 2;
    no bias, no lengths."""
    g = torch.Generator().manual_seed(4)
    b, L, inner, gn, K = 2, 77, 30, 5, 2
    hBC = torch.randn(b, L, inner + 2 * gn, generator=g).to(torch.bfloat16)
    w = torch.randn(inner + 2 * gn, K, generator=g)
    x, B, C, ctx = _run(hBC.cuda(), w.cuda(), None, inner, gn)
    xr, Br, Cr, ctxr = ssm_front_ref.prefill_front(hBC, w, None, inner, gn, None, act_dtype=torch.bfloat16)
    assert_bf16_close(x.float(), xr, "x")
    assert_bf16_close(B.float(), Br, "B")
    assert_bf16_close(C.float(), Cr, "C")
    assert torch.equal(ctx.cpu(), ctxr)


@pytest.mark.gpu
def test_errors_before_launch():
    from selective_attention_b200 import kernels

    hBC = torch.randn(1, 8, 20, device="cuda")
    with pytest.raises(ValueError):
        kernels.ssm_conv_prefill(hBC, torch.randn(20, 1, 4, device="cuda"), None, 10, 4)  # 10 + 8 != 20
    with pytest.raises(ValueError):
        kernels.ssm_conv_prefill(hBC, torch.randn(20, 1, 9, device="cuda"), None, 12, 4)  # K > 8


DECODE_CASES = ["ssm_decode_fp32", "ssm_decode_bf16"]


@pytest.mark.parametrize("case", DECODE_CASES)
def test_decode_oracle_matches_reference_golden(case):
    g = load_golden(case)
    ctx = g["ctx0"].clone()
    for hBC, o in zip(g["hBC"], g["out"]):
        x, B, C, ctx = ssm_front_ref.decode_front(hBC, ctx, g["weight"], g["bias"], g["inner"], g["gn"])
        close = assert_close_for(hBC.dtype)
        close(x.float(), o["x"].float(), f"{case} x")
        close(B.float(), o["B"].float(), f"{case} B")
        close(C.float(), o["C"].float(), f"{case} C")
        assert torch.equal(ctx, o["conv_ctx"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", DECODE_CASES)
def test_decode_kernel_matches_reference_golden(case):
    """Two steps in a row: the cache is updated in place and carried to the next step."""
    from selective_attention_b200 import kernels

    g = load_golden(case)
    ctx = g["ctx0"].cuda().contiguous()
    for hBC, o in zip(g["hBC"], g["out"]):
        x, B, C = kernels.ssm_conv_decode(hBC.cuda(), ctx, g["weight"].cuda(), g["bias"].cuda(), g["inner"], g["gn"])
        torch.cuda.synchronize()
        close = assert_close_for(hBC.dtype)
        close(x.float(), o["x"].float(), f"{case} x")
        close(B.float(), o["B"].float(), f"{case} B")
        close(C.float(), o["C"].float(), f"{case} C")
        assert torch.equal(ctx.cpu(), o["conv_ctx"])


@pytest.mark.gpu
def test_decode_step_front_end_then_ssu_vs_oracle():
    """A whole decode step of the SSM layer below the projections: the front end reads a
    slice of a projection-shaped row, its x/B/C feed the SSU with D and the z gate
    (modules/ssm.py:162-202), against the oracle composition."""
    import math

    from selective_attention_b200 import kernels
    from oracle import ssd_ref

    g = torch.Generator().manual_seed(11)
    b, H, P, N, G, K = 5, 8, 64, 128, 1, 4
    inner, gn = H * P, G * N
    conv_dim = inner + 2 * gn
    proj = torch.randn(b, conv_dim + inner + H, generator=g).to(torch.bfloat16)
    hBC, z, dr = proj[:, :conv_dim], proj[:, conv_dim:conv_dim + inner], proj[:, conv_dim + inner:].float() - 4.0
    ctx0 = torch.randn(b, conv_dim, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(conv_dim, 1, K, generator=g) * 0.5).to(torch.bfloat16)
    bias = (torch.randn(conv_dim, generator=g) * 0.1).to(torch.bfloat16)
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    db = 0.1 * torch.randn(H, generator=g)
    D = torch.randn(inner, generator=g)
    h0 = 0.1 * torch.randn(b, H, P, N, generator=g)

    ctx = ctx0.cuda().contiguous()
    x, B, C = kernels.ssm_conv_decode(proj.cuda()[:, :conv_dim], ctx, w.cuda(), bias.cuda(), inner, gn)
    h = h0.cuda().contiguous()
    y, _ = kernels.ssu_forward(x.view(b, H, P), A.cuda(), B.view(b, G, N), C.view(b, G, N), dr.cuda(), db.cuda(), h,
                               True, (0.0, float("inf")), D.cuda(), z.cuda().contiguous())
    torch.cuda.synchronize()

    xr, Br, Cr, ctxr = ssm_front_ref.decode_front(hBC, ctx0, w, bias, inner, gn)
    yr, hr = ssd_ref.ssu_forward(xr.view(b, H, P).float(), A, Br.view(b, G, N).float(), Cr.view(b, G, N).float(),
                                 dr, db, h0)
    yr = ssd_ref.gate_epilogue(yr.reshape(b, 1, H, P), xr.view(b, 1, H, P), D, z.reshape(b, 1, inner)).view(b, H, P)
    assert torch.equal(ctx.cpu(), ctxr)
    assert_bf16_close(x.float(), xr.float(), "front x")
    assert_bf16_close(y.float(), yr, "decode y")
    assert_bf16_close(h, hr, "decode h")
