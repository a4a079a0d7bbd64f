"""Selective state update (decode) on the GPU against golden vectors and the oracle.

Tolerances: fp32 rel 1e-4, bf16 atol 2e-2 / rel 1e-2 (conftest.py). The state is
fp32 in the reference's path, so h is also checked at fp32 tolerance.
"""
import pytest
import torch

from conftest import SSU_CASES, assert_bf16_close, assert_fp32_close, load_golden
from oracle import ssd_ref

pytestmark = pytest.mark.gpu


def dev(t):
    return None if t is None else t.cuda()


@pytest.mark.parametrize("case", SSU_CASES)
def test_ssu_matches_reference_golden(case):
    import selective_attention_b200 as sab

    g = load_golden(case)
    i = g["inputs"]
    limit = g.get("limit", (0.0, float("inf")))
    h = dev(i["h"])
    y, h_out = sab.SSUFn.forward(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]),
                                 dev(i["delta_bias"]), h, True, limit)
    sab.check_device_error()
    assert h_out.data_ptr() == h.data_ptr(), "state must be updated in place"
    assert y.dtype == i["u"].dtype
    assert_fp32_close(h_out, g["h_new"], f"{case} h")
    if y.dtype == torch.float32:
        assert_fp32_close(y, g["y"], f"{case} y")
    else:
        assert_bf16_close(y.float(), g["y"].float(), f"{case} y")


def test_ssu_fused_gate_vs_oracle():
    import selective_attention_b200 as sab

    g = load_golden("ssu_bf16")
    i = g["inputs"]
    y, h = sab.SSUFn.forward(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]),
                             dev(i["delta_bias"]), dev(i["h"]), True, (0.0, float("inf")), dev(i["D"]), dev(i["z"]))
    sab.check_device_error()
    y_ref, _ = ssd_ref.ssu_forward(i["u"].float(), i["A"], i["B"].float(), i["C"].float(), i["delta_raw"],
                                   i["delta_bias"], i["h"])
    b, H, P = i["u"].shape
    gated = (y_ref + i["D"].view(H, P) * i["u"].float()) * torch.nn.functional.silu(i["z"].float().view(b, H, P))
    assert_bf16_close(y.float(), gated, "gated ssu y")


@pytest.mark.parametrize("N", [16, 48, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_ssu_shapes_and_dtypes_vs_oracle(N, dtype):
    import selective_attention_b200 as sab
    from selective_attention_b200 import workloads

    cfg = workloads.SSU_CONFIGS["c3"]
    inp = workloads.make_ssu_inputs(cfg, seed=N, batch=5, nheads=6, ngroups=3, dstate=N, headdim=40,
                                    dtype={torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[dtype])
    h = dev(inp["h"])
    y, h = sab.SSUFn.forward(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                             dev(inp["delta_bias"]), h, True, (0.0, float("inf")), dev(inp["D"]), dev(inp["z"]))
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssu_forward(inp["u"].float(), inp["A"], inp["B"].float(), inp["C"].float(),
                                       inp["delta_raw"], inp["delta_bias"], inp["h"])
    b, H, P = inp["u"].shape
    y_ref = (y_ref + inp["D"].view(H, P) * inp["u"].float()) * torch.nn.functional.silu(inp["z"].float().view(b, H, P))
    assert_fp32_close(h, h_ref, "h")
    if dtype == torch.float32:
        assert_fp32_close(y, y_ref, "y")
    else:
        assert_bf16_close(y.float(), y_ref, "y")


def test_ssu_bf16_state():
    import selective_attention_b200 as sab
    from selective_attention_b200 import workloads

    inp = workloads.make_ssu_inputs(workloads.SSU_CONFIGS["c3"], seed=3, batch=4, nheads=8)
    h16 = dev(inp["h"]).bfloat16()
    y, h16 = sab.SSUFn.forward(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                               dev(inp["delta_bias"]), h16)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssu_forward(inp["u"].float(), inp["A"], inp["B"].float(), inp["C"].float(),
                                       inp["delta_raw"], inp["delta_bias"], inp["h"].bfloat16().float())
    assert_bf16_close(h16.float(), h_ref, "bf16 state")
    assert_bf16_close(y.float(), y_ref, "y")


def test_ssu_c3_full_size_vs_oracle():
    """Benchmark config c3: b256 H80 P64 N128, fp32 state in place, bf16 x/B/C/z, dt_bias, D + z."""
    import selective_attention_b200 as sab
    from selective_attention_b200 import workloads

    inp = workloads.make_ssu_inputs(workloads.SSU_CONFIGS["c3"], seed=0)
    h = dev(inp["h"])
    y, h = sab.SSUFn.forward(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                             dev(inp["delta_bias"]), h, True, (0.0, float("inf")), dev(inp["D"]), dev(inp["z"]))
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssu_forward(inp["u"].float(), inp["A"], inp["B"].float(), inp["C"].float(),
                                       inp["delta_raw"], inp["delta_bias"], inp["h"])
    b, H, P = inp["u"].shape
    y_ref = (y_ref + inp["D"].view(H, P) * inp["u"].float()) * torch.nn.functional.silu(inp["z"].float().view(b, H, P))
    assert_fp32_close(h, h_ref, "c3 h")
    assert_bf16_close(y.float(), y_ref, "c3 y")


def test_ssu_errors():
    import selective_attention_b200 as sab

    g = load_golden("ssu_fp32_groups")
    i = g["inputs"]
    with pytest.raises(ValueError):
        sab.SSUFn.forward(i["u"], i["A"], i["B"], i["C"], i["delta_raw"], None, i["h"])
    with pytest.raises(ValueError):
        sab.SSUFn.forward(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]), None,
                          dev(i["h"][:, :2]))
