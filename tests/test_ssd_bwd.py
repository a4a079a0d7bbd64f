"""SSD backward: the CPU oracle against the reference's golden gradients, and the
CUDA backward (C-ABI ``ssd_scan_bwd`` through ``kernels.ssd_scan_backward`` and
``SSDScanFn`` autograd) against both.

Golden vectors: ``tests/golden/make_golden_bwd.py`` runs the reference's own
backward kernels (``triton_kernels/ssd_scan/backward.py``) under the Triton
interpreter. Tolerances: fp32 problems rel 1e-4 (``assert_fp32_close``); for 16-bit
inputs, a gradient returned in a 16-bit type atol 2e-2 / rel 1e-2 (``assert_bf16_close``)
and one returned in fp32 rel 1e-2 plus 5e-3 of its largest magnitude
(``assert_bf16_operand_close``: the state-side products run on tensor cores with 16-bit
operands).
"""
import math

import pytest
import torch

from conftest import assert_bf16_close, assert_bf16_operand_close, assert_fp32_close, load_golden
from oracle import ssd_bwd_ref, ssd_ref

INF = float("inf")
BWD_CASES = ["ssd_bwd_c0_fp32", "ssd_bwd_ragged_fp32", "ssd_bwd_clamp_fp32", "ssd_bwd_nosoftplus_fp32",
             "ssd_bwd_p64_bf16", "ssd_bwd_p64_groups_ragged_bf16"]
IN_NAMES = ("u", "A", "B", "C", "delta_raw", "delta_bias", "h_init")
GRAD_NAMES = tuple(n + "_grad" for n in IN_NAMES)


def assert_token_sum_close(actual, expected, terms, what=""):
    """delta_bias_grad[h] is the sum over tokens of delta_raw_grad[t, h] (the bias enters as
    raw + bias): held to rel 1e-4 of the summed terms' magnitudes, the bound that rel 1e-4 on
    every term gives; a head whose terms cancel has a small sum with that absolute error."""
    a, e = actual.double().cpu(), expected.double().cpu()
    mag = terms.double().cpu().abs().reshape(-1, e.numel()).sum(0)
    tol = 1e-4 * mag + 1e-5 * e.abs().max().item() + 1e-12
    err = (a - e).abs()
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {e.numel()} sums outside rel 1e-4 of their terms "
                           f"(max abs err {err.max().item():.3e})")


def check_grads(out, ref, case, u_dtype):
    for name, a, e in zip(GRAD_NAMES, out, [ref[n] for n in GRAD_NAMES]):
        if e is None:
            assert a is None, f"{case}: {name} should be None"
            continue
        if name == "delta_bias_grad" and a.dtype == torch.float32 and u_dtype == torch.float32:
            assert_token_sum_close(a.float(), e, ref["delta_raw_grad"], f"{case} {name}")
            continue
        # a gradient returned in a 16-bit type (u_grad for 16-bit u; every 16-bit leaf
        # through autograd, which casts to the leaf's dtype) carries one rounding of it; an
        # fp32 gradient of a 16-bit problem comes from 16-bit tensor-core operands
        if a.dtype != torch.float32:
            close = assert_bf16_close
        elif u_dtype != torch.float32:
            close = assert_bf16_operand_close
        else:
            close = assert_fp32_close
        close(a.float(), e, f"{case} {name}")


def oracle_args(g):
    return ([g[k] for k in IN_NAMES] + [g["y_grad"], g["h_last_grad"], g["length"], g["chunk_size"],
                                        g["use_delta_softplus"], g["delta_limit"]])


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("case", BWD_CASES)
def test_oracle_matches_reference_golden(case):
    g = load_golden(case)
    out = ssd_bwd_ref.ssd_scan_backward(*oracle_args(g), dtype=torch.float32)
    check_grads(out, g, case, torch.float32)


def test_golden_equals_autograd_of_the_forward():
    """Pin independent of the reference: on full-length rows (no clamps active) the
    reference backward is the exact derivative of its forward."""
    g = load_golden("ssd_bwd_c0_fp32")
    leaves = {k: g[k].double().clone().requires_grad_(True) for k in IN_NAMES}
    y, h = ssd_ref.ssd_scan_forward(*[leaves[k] for k in IN_NAMES], g["length"], g["chunk_size"],
                                    g["use_delta_softplus"], g["delta_limit"], True, dtype=torch.float64)
    torch.autograd.backward([y, h], [g["y_grad"].double(), g["h_last_grad"].double()])
    for k in IN_NAMES:
        assert_fp32_close(leaves[k].grad, g[k + "_grad"], f"autograd {k}")


@pytest.mark.parametrize("case", BWD_CASES)
def test_golden_bias_grad_is_the_token_sum_of_raw_grad(case):
    """The bias enters as raw + bias, so the reference's delta_bias_grad is the sum over tokens
    of its delta_raw_grad: the identity the fp32 bias-gradient tolerance rests on."""
    g = load_golden(case)
    db = g.get("delta_bias_grad")
    if db is None:
        pytest.skip("no delta_bias in this case")
    dr = g["delta_raw_grad"].double().reshape(-1, db.numel())
    assert ((dr.sum(0) - db.double()).abs() <= 1e-6 * dr.abs().sum(0) + 1e-12).all()


def test_oracle_ignores_y_grad_past_length():
    """The reference masks every backward stage at ``length``: y_grad there changes nothing."""
    g = load_golden("ssd_bwd_ragged_fp32")
    yg = g["y_grad"].clone()
    for r, n in enumerate(g["length"].tolist()):
        yg[r, n:] = 1e3
    args = oracle_args(g)
    args[7] = yg
    out = ssd_bwd_ref.ssd_scan_backward(*args)
    check_grads(out, g, "ragged y_grad past length", torch.float32)


def test_oracle_varlen_matches_padded():
    torch.manual_seed(0)
    H, P, N, G, cs = 2, 32, 16, 1, 64
    lens = [70, 130, 33]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.long)
    u = torch.randn(1, T, H, P)
    B = torch.randn(1, T, G, N) / 4
    C = torch.randn(1, T, G, N) / 4
    dr = torch.randn(1, T, H) - 4
    A = -torch.rand(H) * 4 - 0.5
    yg = torch.randn(1, T, H, P)
    out = ssd_bwd_ref.ssd_scan_backward_varlen(u, A, B, C, dr, None, cu, yg, None, cs)
    # row by row through the padded oracle
    for i, n in enumerate(lens):
        s = slice(int(cu[i]), int(cu[i]) + n)
        r = ssd_bwd_ref.ssd_scan_backward(u[:, s], A, B[:, s], C[:, s], dr[:, s], None, None, yg[:, s], None,
                                          None, cs)
        torch.testing.assert_close(out[0][:, s], r[0])
        torch.testing.assert_close(out[2][:, s], r[2])


# ----------------------------------------------------------------------------- GPU
def dev(t):
    return None if t is None else t.cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("case", BWD_CASES)
def test_kernel_matches_reference_golden(case):
    import selective_attention_b200 as sab
    from selective_attention_b200 import kernels

    g = load_golden(case)
    out = kernels.ssd_scan_backward(*[dev(g[k]) for k in IN_NAMES], dev(g["y_grad"]), dev(g["h_last_grad"]),
                                    dev(g["length"]), g["chunk_size"], g["use_delta_softplus"], g["delta_limit"])
    sab.check_device_error()
    assert out[0].dtype == g["u"].dtype and out[4].dtype == g["delta_raw"].dtype
    check_grads([None if t is None else t.cpu() for t in out], g, case, g["u"].dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["ssd_bwd_c0_fp32", "ssd_bwd_p64_groups_ragged_bf16"])
def test_autograd_through_ssdscanfn(case):
    import selective_attention_b200 as sab

    g = load_golden(case)
    leaves = {k: (None if g[k] is None else dev(g[k]).clone().requires_grad_(True)) for k in IN_NAMES}
    y, h = sab.SSDScanFn.apply(*[leaves[k] for k in IN_NAMES], dev(g["length"]), g["chunk_size"],
                               g["use_delta_softplus"], g["delta_limit"], True)
    torch.autograd.backward([y, h], [dev(g["y_grad"]), dev(g["h_last_grad"])])
    out = [None if leaves[k] is None else leaves[k].grad.cpu() for k in IN_NAMES]
    check_grads(out, g, case + " autograd", g["u"].dtype)


def make_inputs(seed, b, L, H, P, N, G, dtype, *, h_init=False, bias=False):
    gen = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=gen)  # noqa: E731
    inp = {
        "u": rn(b, L, H, P).to(dtype),
        "A": -torch.exp(torch.rand(H, generator=gen) * math.log(16.0)),
        "B": (rn(b, L, G, N) / math.sqrt(N)).to(dtype),
        "C": (rn(b, L, G, N) / math.sqrt(N)).to(dtype),
        "delta_raw": rn(b, L, H) - 4.0,
        "delta_bias": 0.1 * rn(H) if bias else None,
        "h_init": 0.1 * rn(b, H, P, N) if h_init else None,
    }
    return inp, rn(b, L, H, P), 0.1 * rn(b, H, P, N)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_kernel_matches_oracle_c1_heads(dtype):
    """config-1 head shape (P64 N128 cs256) over 4 chunks, a ragged row, 6 heads in 2 groups."""
    from selective_attention_b200 import kernels

    inp, yg, hlg = make_inputs(3, 2, 1024, 6, 64, 128, 2, dtype, h_init=True, bias=True)
    length = torch.tensor([1024, 777])
    out = kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg), dev(hlg), dev(length), 256)
    ref = ssd_bwd_ref.ssd_scan_backward(*[inp[k] for k in IN_NAMES], yg, hlg, length, 256)
    check_grads([None if t is None else t.cpu() for t in out], dict(zip(GRAD_NAMES, ref)), "c1 heads", dtype)


@pytest.mark.gpu
def test_kernel_y_grad_in_16_bits_and_no_h_last_grad():
    from selective_attention_b200 import kernels

    inp, yg, _ = make_inputs(4, 1, 512, 2, 64, 128, 1, torch.bfloat16)
    yg16 = yg.to(torch.bfloat16)
    out = kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg16), None, None, 256)
    ref = ssd_bwd_ref.ssd_scan_backward(*[inp[k] for k in IN_NAMES], yg16.float(), None, None, 256)
    check_grads([None if t is None else t.cpu() for t in out], dict(zip(GRAD_NAMES, ref)), "bf16 y_grad",
                torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kernel_packed_rows_match_oracle(dtype):
    """Packed rows whose chunks end inside a chunk; fp32 inputs take the split-bf16 products."""
    from selective_attention_b200 import kernels

    H, P, N, G, cs = 4, 64, 128, 1, 256
    lens = [300, 513, 64, 700]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    inp, yg, _ = make_inputs(5, 1, T, H, P, N, G, dtype, bias=True)
    hlg = 0.1 * torch.randn(len(lens), H, P, N)
    out = kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg), dev(hlg), None, cs,
                                    cu_seqlens=dev(cu))
    ref = ssd_bwd_ref.ssd_scan_backward_varlen(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"],
                                               inp["delta_bias"], cu.long(), yg, hlg, cs)
    check_grads([None if t is None else t.cpu() for t in out], dict(zip(GRAD_NAMES, ref)), "packed", dtype)


@pytest.mark.gpu
def test_kernel_rejects_unsupported_shapes():
    from selective_attention_b200 import kernels

    inp, yg, _ = make_inputs(6, 1, 256, 2, 128, 16, 1, torch.float32)
    with pytest.raises(ValueError):  # headdim 128 > 64
        kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg), None, None, 64)
    inp, yg, _ = make_inputs(6, 1, 256, 2, 32, 16, 1, torch.float32)
    with pytest.raises(ValueError):  # chunk size not a multiple of 32
        kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg), None, None, 48)
    with pytest.raises(ValueError):  # y_grad shape
        kernels.ssd_scan_backward(*[dev(inp[k]) for k in IN_NAMES], dev(yg[:, :10]), None, None, 64)
