"""The reference's own SSM layer running on the B200 kernels through ``shim.install()``.

The reference package (pure Python + Triton) is installed without its dependencies into
``baseline/_ref`` by ``baseline/install_reference.sh``; these tests import it from there
and skip when it is absent. ``shim.install()`` rebinds ``SSDScanFn`` / ``SSUFn`` inside
it, so ``SSM.forward`` (``modules/ssm.py:136-139``) and ``SSM.step`` (``:195-197``) call
the CUDA library unchanged.

GPU tests:
- prefill of padded rows with a cache, then 16 decode steps, on the GPU under the shim,
  against the same layer on the CPU with both ops bound to the oracle restatement;
- the reference's own consistency check (``tests/test_causal_lm.py:55-133``, here at the
  layer): a prefill of L tokens followed by k steps gives the outputs of one forward over
  L + k tokens.
"""
import copy
import os
import sys

import pytest
import torch

from conftest import ROOT, assert_fp32_close

REF_DIR = os.path.join(ROOT, "baseline", "_ref")
INF = float("inf")


def _reference():
    if not os.path.isdir(os.path.join(REF_DIR, "selective_attention")):
        pytest.skip("reference package not installed in baseline/_ref (run baseline/install_reference.sh)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import selective_attention.modules.ssm as ssm_mod
    from selective_attention.inference import SSMCache

    return ssm_mod, SSMCache


def test_install_raises_for_a_missing_package():
    from selective_attention_b200 import shim

    with pytest.raises(ImportError):
        shim.install("no_such_selective_attention_package")
    assert not shim.installed()


def test_install_rebinds_and_uninstall_restores():
    ssm_mod, _ = _reference()
    import selective_attention.ops as ref_ops

    import selective_attention_b200 as sab
    from selective_attention_b200 import shim

    orig = (ssm_mod.SSDScanFn, ssm_mod.SSUFn, ref_ops.SSDScanFn, ref_ops.SSUFn)
    shim.install()
    try:
        assert ssm_mod.SSDScanFn is sab.SSDScanFn and ssm_mod.SSUFn is sab.SSUFn
        assert ref_ops.SSDScanFn is sab.SSDScanFn and ref_ops.SSUFn is sab.SSUFn
    finally:
        shim.uninstall()
    assert (ssm_mod.SSDScanFn, ssm_mod.SSUFn, ref_ops.SSDScanFn, ref_ops.SSUFn) == orig


class _OracleSSD:
    """``SSDScanFn`` bound to the CPU restatement (same positional signature)."""

    @staticmethod
    def apply(u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None, chunk_size=256,
              use_delta_softplus=True, delta_limit=(0.0, INF), is_causal=True):
        from oracle import ssd_ref

        return ssd_ref.ssd_scan_forward(u.float(), A.float(), B.float(), C.float(), delta_raw.float(),
                                        None if delta_bias is None else delta_bias.float(), h_init, length,
                                        chunk_size, use_delta_softplus, delta_limit)


class _OracleSSU:
    """``SSUFn`` bound to the CPU restatement: state updated in place, y in u's dtype."""

    @staticmethod
    def forward(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus=True, delta_limit=(0.0, INF)):
        from oracle import ssd_ref

        y, h_new = ssd_ref.ssu_forward(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus, delta_limit)
        h.copy_(h_new)
        return y.to(u.dtype), h


def _layer(ssm_mod, seed=0):
    torch.manual_seed(seed)
    layer = ssm_mod.SSM(0, model_dim=256, state_dim=128, head_dim=64, num_groups=1, chunk_size=256,
                        device="cpu").eval()
    with torch.no_grad():  # the default init leaves D at 1 and the conv bias small: spread them
        layer.D.normal_()
        layer.conv.bias.normal_(0.0, 0.1)
    return layer


def _run(layer, ssm_mod, SSMCache, ssd_op, ssu_op, x, lengths, steps):
    saved = (ssm_mod.SSDScanFn, ssm_mod.SSUFn)
    ssm_mod.SSDScanFn, ssm_mod.SSUFn = ssd_op, ssu_op
    try:
        with torch.no_grad():
            cache = SSMCache()
            out, h_last = layer(x, lengths, None, cache)
            outs = [layer.step(s, cache) for s in steps]
        return out, h_last, torch.stack(outs, 1)
    finally:
        ssm_mod.SSDScanFn, ssm_mod.SSUFn = saved


@pytest.fixture
def no_tf32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


@pytest.mark.gpu
def test_ssm_layer_prefill_and_decode_through_shim_vs_oracle(no_tf32):
    ssm_mod, SSMCache = _reference()
    import selective_attention_b200 as sab
    from selective_attention_b200 import shim

    cpu = _layer(ssm_mod)
    gpu = copy.deepcopy(cpu).cuda()
    g = torch.Generator().manual_seed(1)
    b, L, k = 3, 300, 16
    x = torch.randn(b, L, 256, generator=g)
    lengths = torch.tensor([300, 211, 64], dtype=torch.long)
    steps = [torch.randn(b, 256, generator=g) for _ in range(k)]

    ref_out, ref_h, ref_steps = _run(cpu, ssm_mod, SSMCache, _OracleSSD, _OracleSSU, x, lengths, steps)

    shim.install()
    try:
        assert ssm_mod.SSDScanFn is sab.SSDScanFn
        with torch.no_grad():
            cache = SSMCache()
            out, h_last = gpu(x.cuda(), lengths.cuda(), None, cache)
            outs = torch.stack([gpu.step(s.cuda(), cache) for s in steps], 1)
        torch.cuda.synchronize()
        sab.check_device_error()
    finally:
        shim.uninstall()
    for r in range(b):  # positions past a row's length are the layer's padding outputs
        n = int(lengths[r])
        assert_fp32_close(out[r, :n].cpu(), ref_out[r, :n], f"SSM.forward row {r}")
    assert_fp32_close(h_last.cpu(), ref_h, "SSM.forward h_last")
    assert_fp32_close(outs.cpu(), ref_steps, "SSM.step outputs")


@pytest.mark.gpu
def test_ssm_layer_prefill_plus_steps_equals_full_forward_through_shim(no_tf32):
    ssm_mod, SSMCache = _reference()
    from selective_attention_b200 import shim

    gpu = _layer(ssm_mod, seed=2).cuda()
    g = torch.Generator().manual_seed(3)
    b, L, k = 2, 280, 12
    x = torch.randn(b, L + k, 256, generator=g).cuda()
    shim.install()
    try:
        with torch.no_grad():
            full, h_full = gpu(x)
            cache = SSMCache()
            pre, _ = gpu(x[:, :L], None, None, cache)
            outs = torch.stack([gpu.step(x[:, L + i], cache) for i in range(k)], 1)
    finally:
        shim.uninstall()
    assert_fp32_close(pre.cpu(), full[:, :L].cpu(), "prefill vs full forward")
    assert_fp32_close(outs.cpu(), full[:, L:].cpu(), "decode steps vs full forward")
    assert_fp32_close(cache.h.cpu(), h_full.cpu(), "state after the steps vs full forward")
