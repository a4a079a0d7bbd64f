"""Selective attention (row f4): the decode step and the inference prefill. The CPU oracle
against golden vectors made with the reference's own cache, compression and softmax code,
and the CUDA kernels (C-ABI ``sattn_decode_step``, ``sattn_prefill_fwd``) against both.

Golden vectors: ``tests/golden/make_golden_sattn.py``. Tolerances: fp32 rel 1e-4
(``assert_fp32_close``); 16-bit outputs atol 2e-2 / rel 1e-2 (``assert_bf16_close``).
"""
import math
import types

import pytest
import torch

from conftest import assert_bf16_close, assert_fp32_close, load_golden
from oracle import sattn_ref

CASES = ["sattn_decode_dropped_fp32", "sattn_decode_fresh_d128_fp32", "sattn_decode_long_fp32"]


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_golden(case):
    g = load_golden(case)
    k, v, lg, w = g["k0"].clone(), g["v0"].clone(), g["lg0"].clone(), g["w0"]
    for i in range(g["q"].shape[0]):
        out, w = sattn_ref.decode_step(g["q"][i], g["k"][i], g["v"][i], g["lg"][i], k, v, lg, w, g["scale"])
        assert_fp32_close(out, g["out"][i], f"{case} step {i}")
    assert w == g["w_end"]
    assert torch.equal(k, g["k_end"]) and torch.equal(v, g["v_end"]) and torch.equal(lg, g["lg_end"])


# ----------------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_kernel_matches_reference_golden(case):
    import selective_attention_b200 as sab
    from selective_attention_b200 import kernels

    g = load_golden(case)
    k, v, lg, w = g["k0"].cuda(), g["v0"].cuda(), g["lg0"].cuda(), g["w0"]
    for i in range(g["q"].shape[0]):
        out = kernels.sattn_decode_step(g["q"][i].cuda(), g["k"][i].cuda(), g["v"][i].cuda(), g["lg"][i].cuda(),
                                        k, v, lg, w, g["scale"])
        w += 1
        assert_fp32_close(out.cpu(), g["out"][i], f"{case} step {i}")
    sab.check_device_error()
    assert torch.equal(k.cpu(), g["k_end"]) and torch.equal(v.cpu(), g["v_end"])
    assert torch.equal(lg.cpu(), g["lg_end"])


@pytest.mark.gpu
def test_cache_object_step_advances_write_idx():
    from selective_attention_b200 import kernels

    g = load_golden("sattn_decode_dropped_fp32")
    cache = types.SimpleNamespace(k_rot=g["k0"].cuda(), v=g["v0"].cuda(), log_gate=g["lg0"].cuda(),
                                  write_idx=g["w0"])
    for i in range(g["q"].shape[0]):
        out = kernels.selective_attn_step(cache, g["q"][i].cuda(), g["k"][i].cuda(), g["v"][i].cuda(),
                                          g["lg"][i].cuda(), g["scale"])
        assert out.shape == (g["q"].shape[1], g["q"].shape[2] * g["q"].shape[3])
        assert_fp32_close(out.view_as(g["out"][i]).cpu(), g["out"][i], f"object step {i}")
    assert cache.write_idx == g["w_end"]


def random_cache(seed, b, H, D, cap, w, dtype, p_zero=0.1):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(b, H, cap, D, generator=gen).to(dtype)
    v = torch.randn(b, H, cap, D, generator=gen).to(dtype)
    lg = torch.log(torch.sigmoid(torch.randn(b, H, cap, generator=gen) + 2.0)) * 2.0
    lg = torch.where(torch.rand(b, H, cap, generator=gen) < p_zero, torch.full_like(lg, -math.inf), lg)
    q = torch.randn(b, H, D, generator=gen).to(dtype)
    kn = torch.randn(b, H, D, generator=gen).to(dtype)
    vn = torch.randn(b, H, D, generator=gen).to(dtype)
    lgn = torch.log(torch.sigmoid(torch.randn(b, H, generator=gen) + 2.0)) * 2.0
    return q, kn, vn, lgn, k, v, lg


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 32),
                                     (torch.float32, 256), (torch.bfloat16, 8)])
def test_kernel_matches_oracle_long_cache(dtype, D):
    from selective_attention_b200 import kernels

    b, H, cap, w = 4, 6, 3000, 2411
    q, kn, vn, lgn, k, v, lg = random_cache(7, b, H, D, cap, w, dtype)
    kd, vd, lgd = k.cuda(), v.cuda(), lg.cuda()
    out = kernels.sattn_decode_step(q.cuda(), kn.cuda(), vn.cuda(), lgn.cuda(), kd, vd, lgd, w)
    ref, _ = sattn_ref.decode_step(q.float(), kn.float(), vn.float(), lgn, k.float(), v.float(), lg, w, D ** -0.5)
    close = assert_fp32_close if dtype == torch.float32 else assert_bf16_close
    close(out.float().cpu(), ref, f"{dtype} D{D}")
    assert torch.equal(kd[:, :, w].cpu(), kn) and torch.equal(vd[:, :, w].cpu(), vn)
    assert torch.equal(lgd[:, :, w].cpu(), lgn)


@pytest.mark.gpu
def test_first_step_returns_the_value():
    """With one cached key (the token) the weight is exactly 1, as the reference's early
    return ``out_proj(v * out_gate)`` (``modules/selective_attention.py:392-393``) assumes."""
    from selective_attention_b200 import kernels

    q, kn, vn, lgn, k, v, lg = random_cache(8, 2, 3, 64, 16, 0, torch.float32)
    out = kernels.sattn_decode_step(q.cuda(), kn.cuda(), vn.cuda(), lgn.cuda(), k.cuda(), v.cuda(), lg.cuda(), 0)
    assert torch.equal(out.cpu(), vn)


@pytest.mark.gpu
def test_kernel_rejects_bad_arguments():
    from selective_attention_b200 import kernels

    q, kn, vn, lgn, k, v, lg = random_cache(9, 1, 2, 64, 16, 0, torch.float32)
    args = [t.cuda() for t in (q, kn, vn, lgn, k, v, lg)]
    with pytest.raises(ValueError):  # no free slot
        kernels.sattn_decode_step(*args, 16)
    q2, kn2, vn2, lgn2, k2, v2, lg2 = random_cache(9, 1, 2, 48, 16, 0, torch.float32)
    with pytest.raises(ValueError):  # head_dim 48 is not a supported power of two
        kernels.sattn_decode_step(*[t.cuda() for t in (q2, kn2, vn2, lgn2, k2, v2, lg2)], 3)


# ----------------------------------------------------------------------------- prefill
PREFILL_CASES = ["sattn_prefill_dropped_fp32", "sattn_prefill_padded_d32_fp32", "sattn_prefill_kept_d128_fp32"]


@pytest.mark.parametrize("case", PREFILL_CASES)
def test_prefill_oracle_matches_reference_golden(case):
    g = load_golden(case)
    out = sattn_ref.prefill_attention(g["q"], g["k"], g["v"], g["log_gate"], g["scale"])
    assert_fp32_close(out, g["out"], case)


@pytest.mark.gpu
@pytest.mark.parametrize("case", PREFILL_CASES)
def test_prefill_kernel_matches_reference_golden(case):
    import selective_attention_b200 as sab
    from selective_attention_b200 import kernels

    g = load_golden(case)
    out = kernels.sattn_prefill(g["q"].cuda(), g["k"].cuda(), g["v"].cuda(), g["log_gate"].cuda(), g["scale"])
    sab.check_device_error()
    assert_fp32_close(out.cpu(), g["out"], case)


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["auto", "simt"])
@pytest.mark.parametrize("dtype,D,L", [(torch.bfloat16, 128, 1000), (torch.float16, 64, 777),
                                       (torch.bfloat16, 64, 130), (torch.float16, 128, 64),
                                       (torch.float32, 16, 300)])
def test_prefill_kernel_matches_oracle(dtype, D, L, impl):
    """``auto`` takes the tensor-core kernel for 16-bit inputs with head_dim 64 / 128."""
    from selective_attention_b200 import kernels

    gen = torch.Generator().manual_seed(11)
    b, H = 2, 3
    q, k, v = (torch.randn(b, H, L, D, generator=gen).to(dtype) for _ in range(3))
    lg = torch.log(torch.sigmoid(torch.randn(b, H, L, generator=gen) + 2.0)) * 2.0
    lg = torch.where(torch.rand(b, H, L, generator=gen) < 0.1, torch.full_like(lg, -math.inf), lg)
    out = kernels.sattn_prefill(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), impl=impl)
    ref = sattn_ref.prefill_attention(q.float(), k.float(), v.float(), lg, D ** -0.5)
    close = assert_fp32_close if dtype == torch.float32 else assert_bf16_close
    close(out.float().cpu(), ref, f"prefill {dtype} D{D} L{L}")


@pytest.mark.gpu
def test_prefill_rejects_bad_arguments():
    from selective_attention_b200 import kernels

    q = torch.randn(1, 2, 10, 48, device="cuda")
    with pytest.raises(ValueError):  # head_dim 48 unsupported
        kernels.sattn_prefill(q, q, q, torch.zeros(1, 2, 10, device="cuda"))
    q = torch.randn(1, 2, 10, 64, device="cuda")
    with pytest.raises(ValueError):  # log_gate shape
        kernels.sattn_prefill(q, q, q, torch.zeros(1, 2, 9, device="cuda"))
    with pytest.raises(ValueError):  # the tensor-core kernel takes 16-bit inputs
        kernels.sattn_prefill(q, q, q, torch.zeros(1, 2, 10, device="cuda"), impl="tc")


def _prefill_inputs(b, H, L, D, dtype, seed, drop=0.1):
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(b, H, L, D, generator=gen).to(dtype) for _ in range(3))
    lg = torch.log(torch.sigmoid(torch.randn(b, H, L, generator=gen) + 2.0)) * 2.0
    lg = torch.where(torch.rand(b, H, L, generator=gen) < drop, torch.full_like(lg, -math.inf), lg)
    return q, k, v, lg


@pytest.mark.gpu
@pytest.mark.parametrize("L", [1, 127, 128, 255, 256, 257, 600, 2048])
def test_prefill_tc_head64_tile_edges(L):
    """The pipelined head_dim-64 kernel (two 128-query tiles per CTA, 128-key tiles in a
    TMA ring) at lengths around its tile edges: a missing second query tile, a partial
    key tile, one token."""
    from selective_attention_b200 import kernels

    q, k, v, lg = _prefill_inputs(2, 3, L, 64, torch.bfloat16, 40 + L)
    out = kernels.sattn_prefill(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), impl="tc")
    ref = sattn_ref.prefill_attention(q.float(), k.float(), v.float(), lg, 64 ** -0.5)
    assert_bf16_close(out.float().cpu(), ref, f"prefill tc D64 L{L}")


@pytest.mark.gpu
def test_prefill_tc_head64_growing_scores_and_dropped_prefix():
    """Scores that grow along the keys (the running max rises tile after tile, so the
    output accumulator is rescaled) and a prefix of 300 dropped keys (rows past it see
    only -inf scores in their first key tiles)."""
    from selective_attention_b200 import kernels

    b, H, L, D = 1, 2, 1100, 64
    q, k, v, lg = _prefill_inputs(b, H, L, D, torch.bfloat16, 5, drop=0.0)
    ramp = torch.linspace(0.0, 6.0, L).view(1, 1, L, 1)
    k = (k.float() * 0.2 + ramp).to(torch.bfloat16)
    q = (q.float() * 0.2 + 1.0).to(torch.bfloat16)
    lg2 = lg.clone()
    lg2[..., :300] = -math.inf
    for lgx in (lg, lg2):
        out = kernels.sattn_prefill(q.cuda(), k.cuda(), v.cuda(), lgx.cuda(), impl="tc")
        ref = sattn_ref.prefill_attention(q.float(), k.float(), v.float(), lgx, D ** -0.5)
        assert_bf16_close(out.float().cpu(), ref, "prefill tc D64 growing scores")


@pytest.mark.gpu
def test_prefill_tc_repeated_runs_are_bit_identical():
    """The pipelined kernel has no atomics and a fixed MMA order: 20 runs on the same
    inputs must match the first bit for bit (a missing wait between its warp roles shows
    up here first)."""
    from selective_attention_b200 import kernels

    q, k, v, lg = (t.cuda() for t in _prefill_inputs(2, 16, 2048, 64, torch.bfloat16, 9))
    out0 = kernels.sattn_prefill(q, k, v, lg, impl="tc")
    differ = 0
    for _ in range(20):
        out = kernels.sattn_prefill(q, k, v, lg, impl="tc")
        differ += int(not torch.equal(out, out0))
    torch.cuda.synchronize()
    assert differ == 0, f"{differ} of 20 runs differ from the first"
