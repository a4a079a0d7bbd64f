"""Training-mode selective attention (``modules/selective_attention.py:232-280`` with
``self.training``) and its backward: the CPU oracle against golden vectors from the
reference's own ``SelectiveMHA`` (``tests/golden/make_golden_sattn_train.py``), and the CUDA
op (C-ABI ``sattn_train_fwd`` / ``sattn_train_bwd`` through ``SelectiveAttnTrainFn``) against
both. Tolerances: fp32 rel 1e-4 (``assert_fp32_close``); 16-bit inputs atol 2e-2 / rel 1e-2
against the oracle run in fp32 on the same rounded inputs (``assert_bf16_close``).
"""
import pytest
import torch

from conftest import assert_bf16_close, assert_fp32_close, load_golden
from oracle import sattn_ref

CASES = ["sattn_train_causal_ragged_fp32", "sattn_train_bidir_ragged_fp32", "sattn_train_causal_d64_fp32"]
GRADS = ("q_rot", "k_rot", "v", "select_gate")


def _oracle_with_grads(g, dtype=torch.float32):
    leaves = {n: g[n].to(dtype).clone().requires_grad_(True) for n in GRADS}
    out, std = sattn_ref.train_attention(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                         g["log_gate_penalty"], g["lengths"], g["is_causal"], g["scale"], dtype)
    out.backward(g["dout"].to(dtype))
    return out.detach(), std.detach(), {n: leaves[n].grad for n in GRADS}


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_golden(case):
    g = load_golden(case)
    out, std, grads = _oracle_with_grads(g)
    assert_fp32_close(out, g["out"], f"{case} out")
    assert_fp32_close(std, g["std"], f"{case} std")
    for n in GRADS:
        assert_fp32_close(grads[n], g[n + "_grad"], f"{case} d{n}")


def test_oracle_std_path_matters():
    """The gradient through the score std is not negligible in these cases: dropping it
    (std detached) moves dq away from the reference's."""
    g = load_golden("sattn_train_causal_ragged_fp32")
    q = g["q_rot"].clone().requires_grad_(True)
    out, std = sattn_ref.train_attention(q, g["k_rot"], g["v"], g["select_gate"], g["log_gate_penalty"],
                                         g["lengths"], True, g["scale"])
    (dq_full,) = torch.autograd.grad(out, q, g["dout"])
    assert (dq_full - g["q_rot_grad"]).abs().max() < 1e-4 * g["q_rot_grad"].abs().max() + 1e-6
    # a copy of the oracle with std detached
    import oracle.sattn_ref as sr
    orig = torch.Tensor.sqrt
    try:
        torch.Tensor.sqrt = lambda t: orig(t).detach()
        q2 = g["q_rot"].clone().requires_grad_(True)
        out2, _ = sr.train_attention(q2, g["k_rot"], g["v"], g["select_gate"], g["log_gate_penalty"], g["lengths"],
                                     True, g["scale"])
        (dq_nostd,) = torch.autograd.grad(out2, q2, g["dout"])
    finally:
        torch.Tensor.sqrt = orig
    assert (dq_nostd - g["q_rot_grad"]).abs().max() > 1e-3 * g["q_rot_grad"].abs().max()


# ----------------------------------------------------------------------------- GPU
def _dev(g):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in g.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_kernel_matches_reference_golden(case):
    import selective_attention_b200 as sab

    g = load_golden(case)
    d = _dev(g)
    leaves = {n: d[n].clone().requires_grad_(True) for n in GRADS}
    out, std = sab.SelectiveAttnTrainFn.apply(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                              d["lengths"], g["log_gate_penalty"], g["is_causal"], g["scale"])
    out.backward(d["dout"])
    sab.check_device_error()
    assert_fp32_close(out.detach().cpu(), g["out"], f"{case} out")
    assert_fp32_close(std.cpu(), g["std"], f"{case} std")
    for n in GRADS:
        assert_fp32_close(leaves[n].grad.cpu(), g[n + "_grad"], f"{case} d{n}")


@pytest.mark.gpu
def test_forward_outputs_lse_and_log_gate():
    from selective_attention_b200 import kernels

    g = load_golden("sattn_train_bidir_ragged_fp32")
    d = _dev(g)
    out, lse, lg, stats = kernels.sattn_train_forward(d["q_rot"], d["k_rot"], d["v"], d["select_gate"],
                                                      g["log_gate_penalty"], d["lengths"], False, g["scale"])
    b, H, L, D = g["q_rot"].shape
    pad = torch.arange(L)[None] >= g["lengths"][:, None]
    exp_lg = torch.log(g["select_gate"]) * (g["std"][None, :, None] * g["log_gate_penalty"])
    exp_lg = exp_lg.masked_fill(pad[:, None, :], float("-inf"))
    fin = torch.isfinite(exp_lg)
    assert torch.equal(torch.isfinite(lg.cpu()), fin)
    assert_fp32_close(lg.cpu()[fin], exp_lg[fin], "log_gate")
    s = (g["q_rot"] @ g["k_rot"].transpose(-2, -1)) * g["scale"]
    diag = torch.arange(L)
    dd = s[:, :, diag, diag]
    s = s + exp_lg.unsqueeze(2)
    s[:, :, diag, diag] = dd
    assert_fp32_close(lse.cpu(), torch.logsumexp(s, -1), "lse")
    valid = (~pad[:, :, None] & ~pad[:, None, :]).sum().float()
    assert torch.all(stats[:, 2].cpu() == valid)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [True, False])
def test_kernel_matches_oracle_at_size(causal):
    """b 2, H 4, L 300 (five 64-token tiles, ragged), D 64, fp32 against the oracle."""
    import selective_attention_b200 as sab

    gen = torch.Generator().manual_seed(11 + causal)
    b, H, L, D = 2, 4, 300, 64
    q, k, v = (torch.randn(b, H, L, D, generator=gen) for _ in range(3))
    sel = torch.sigmoid(torch.randn(b, H, L, generator=gen) + 1.0)
    lengths = torch.tensor([300, 217])
    dout = torch.randn(b, H, L, D, generator=gen)
    g = {"q_rot": q, "k_rot": k, "v": v, "select_gate": sel, "lengths": lengths, "log_gate_penalty": 1.5,
         "is_causal": causal, "scale": D ** -0.5, "dout": dout}
    ref_out, ref_std, ref_grads = _oracle_with_grads(g)
    leaves = {n: g[n].cuda().requires_grad_(True) for n in GRADS}
    out, std = sab.selective_attn_train(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                        lengths.cuda(), 1.5, causal)
    out.backward(dout.cuda())
    assert_fp32_close(out.detach().cpu(), ref_out, "out")
    assert_fp32_close(std.cpu(), ref_std, "std")
    for n in GRADS:
        assert_fp32_close(leaves[n].grad.cpu(), ref_grads[n], f"d{n}")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_kernel_16bit_matches_oracle(dtype):
    import selective_attention_b200 as sab

    gen = torch.Generator().manual_seed(21)
    b, H, L, D = 2, 2, 200, 32
    q, k, v = (torch.randn(b, H, L, D, generator=gen).to(dtype) for _ in range(3))
    sel = torch.sigmoid(torch.randn(b, H, L, generator=gen) + 1.0).to(dtype)
    dout = torch.randn(b, H, L, D, generator=gen).to(dtype)
    lengths = torch.tensor([200, 150])
    g = {"q_rot": q, "k_rot": k, "v": v, "select_gate": sel, "lengths": lengths, "log_gate_penalty": 1.0,
         "is_causal": True, "scale": D ** -0.5, "dout": dout}
    ref_out, ref_std, ref_grads = _oracle_with_grads(g, torch.float32)
    leaves = {n: g[n].cuda().requires_grad_(True) for n in GRADS}
    out, std = sab.selective_attn_train(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                        lengths.cuda(), 1.0, True)
    out.backward(dout.cuda())
    assert out.dtype == dtype and leaves["q_rot"].grad.dtype == dtype
    assert_bf16_close(out.detach().float().cpu(), ref_out, "out")
    assert_fp32_close(std.cpu(), ref_std, "std")  # fp32 statistics of the same rounded inputs
    for n in GRADS:
        assert_bf16_close(leaves[n].grad.float().cpu(), ref_grads[n], f"d{n}")


@pytest.mark.gpu
def test_rejects_unsupported_head_dim():
    from selective_attention_b200 import kernels

    q = torch.randn(1, 1, 64, 48, device="cuda")
    with pytest.raises(ValueError):
        kernels.sattn_train_forward(q, q, q, torch.rand(1, 1, 64, device="cuda"), 1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_path_matches_oracle(causal, dtype):
    """16-bit inputs with head_dim 64 run on tcgen05 (impl "tc"): b 2, H 3, L 300 (three
    128-token tiles, the last partial), ragged lengths, against the oracle in fp32 on the
    same rounded inputs. Probabilities and dS enter the products in 16 bits."""
    import selective_attention_b200 as sab

    gen = torch.Generator().manual_seed(31 + causal)
    b, H, L, D = 2, 3, 300, 64
    q, k, v = (torch.randn(b, H, L, D, generator=gen).to(dtype) for _ in range(3))
    sel = torch.sigmoid(torch.randn(b, H, L, generator=gen) + 1.0).to(dtype)
    dout = torch.randn(b, H, L, D, generator=gen).to(dtype)
    lengths = torch.tensor([300, 190])
    g = {"q_rot": q, "k_rot": k, "v": v, "select_gate": sel, "lengths": lengths, "log_gate_penalty": 1.0,
         "is_causal": causal, "scale": D ** -0.5, "dout": dout}
    ref_out, ref_std, ref_grads = _oracle_with_grads(g, torch.float32)
    leaves = {n: g[n].cuda().requires_grad_(True) for n in GRADS}
    out, std = sab.selective_attn_train(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                        lengths.cuda(), 1.0, causal, impl="tc")
    out.backward(dout.cuda())
    sab.check_device_error()
    assert_bf16_close(out.detach().float().cpu(), ref_out, "out")
    assert_fp32_close(std.cpu(), ref_std, "std")
    for n in GRADS:
        assert_bf16_close(leaves[n].grad.float().cpu(), ref_grads[n], f"d{n}")


@pytest.mark.gpu
def test_tensor_core_path_rejects_fp32():
    from selective_attention_b200 import kernels

    q = torch.randn(1, 1, 128, 64, device="cuda")
    with pytest.raises(ValueError):
        kernels.sattn_train_forward(q, q, q, torch.rand(1, 1, 128, device="cuda"), 1.0, impl="tc")


@pytest.mark.gpu
def test_tensor_core_path_short_sequence():
    """L = 100 (one partial 128-token tile; TMA boxes reach past the end), bidirectional."""
    import selective_attention_b200 as sab

    gen = torch.Generator().manual_seed(41)
    b, H, L, D = 1, 2, 100, 64
    q, k, v = (torch.randn(b, H, L, D, generator=gen).bfloat16() for _ in range(3))
    sel = torch.sigmoid(torch.randn(b, H, L, generator=gen) + 1.0).bfloat16()
    dout = torch.randn(b, H, L, D, generator=gen).bfloat16()
    g = {"q_rot": q, "k_rot": k, "v": v, "select_gate": sel, "lengths": None, "log_gate_penalty": 1.0,
         "is_causal": False, "scale": D ** -0.5, "dout": dout}
    ref_out, ref_std, ref_grads = _oracle_with_grads(g, torch.float32)
    leaves = {n: g[n].cuda().requires_grad_(True) for n in GRADS}
    out, std = sab.selective_attn_train(leaves["q_rot"], leaves["k_rot"], leaves["v"], leaves["select_gate"],
                                        None, 1.0, False, impl="tc")
    out.backward(dout.cuda())
    sab.check_device_error()
    assert_bf16_close(out.detach().float().cpu(), ref_out, "out")
    assert_fp32_close(std.cpu(), ref_std, "std")
    for n in GRADS:
        assert_bf16_close(leaves[n].grad.float().cpu(), ref_grads[n], f"d{n}")
