"""Pin the CPU oracle (oracle/ssd_ref.py) to the reference's own outputs.

The golden vectors come from the reference's Triton kernels run under the Triton
interpreter (tests/golden/make_golden.py). The oracle must reproduce them, stage by
stage, to fp32 rounding; it is also checked against the fp64 token recurrence and
against the prefill + decode consistency the reference's model test relies on
(tests/test_causal_lm.py:55-133 of the reference).
"""
import math

import pytest
import torch

from conftest import SSD_CASES, SSU_CASES, load_golden
from oracle import ssd_ref

TIGHT = dict(rtol=2e-5, atol=2e-6)


def f32(t):
    return None if t is None else t.float()


def run_oracle(g, dtype=torch.float32):
    i = g["inputs"]
    return ssd_ref.ssd_scan_forward(f32(i["u"]), i["A"], f32(i["B"]), f32(i["C"]), i["delta_raw"],
                                    i["delta_bias"], i["h_init"], g["length"], g["chunk_size"], g["use_sp"],
                                    g["limit"], True, dtype=dtype)


@pytest.mark.parametrize("case", SSD_CASES)
def test_oracle_matches_reference_ssd(case):
    g = load_golden(case)
    y, h = run_oracle(g)
    scale_y = g["y"].abs().max().item()
    torch.testing.assert_close(y, g["y"], rtol=2e-5, atol=2e-6 * max(1.0, scale_y))
    torch.testing.assert_close(h, g["h_last"], rtol=2e-5, atol=2e-6 * max(1.0, g["h_last"].abs().max().item()))


@pytest.mark.parametrize("case", ["ssd_c0_fp32", "ssd_ragged_fp32"])
def test_oracle_matches_reference_stages(case):
    g = load_golden(case)
    i = g["inputs"]
    cs = g["chunk_size"]
    cum, dt = ssd_ref.chunk_cumsum(i["A"], i["delta_raw"], i["delta_bias"], g["length"], cs, g["use_sp"], g["limit"])
    torch.testing.assert_close(dt, g["dt"], **TIGHT)
    torch.testing.assert_close(cum, g["cum"], rtol=2e-5, atol=2e-5)
    S = ssd_ref.chunk_state(i["u"], i["B"], g["dt"], g["cum"])
    torch.testing.assert_close(S, g["states"], rtol=2e-5, atol=2e-5)
    prev, h_last = ssd_ref.state_passing(g["states"], i["h_init"], g["cum"][..., -1])
    torch.testing.assert_close(prev, g["prev"], rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(h_last, g["h_last"], rtol=2e-5, atol=2e-5)
    CB = ssd_ref.bmm_chunk(i["B"], i["C"], cs)
    low = torch.tril(torch.ones(cs, cs, dtype=torch.bool))
    torch.testing.assert_close(CB[..., low], g["CB"][..., low], rtol=2e-5, atol=2e-6)
    y = ssd_ref.chunk_scan(i["u"], g["dt"], g["cum"], i["C"], g["prev"], g["CB"])
    torch.testing.assert_close(y, g["y_stage"], rtol=2e-5, atol=2e-5)


def test_oracle_matches_reference_varlen():
    g = load_golden("ssd_varlen_bf16")
    i = g["inputs"]
    y, h = ssd_ref.ssd_scan_varlen(f32(i["u"]), i["A"], f32(i["B"]), f32(i["C"]), i["delta_raw"], None,
                                   g["cu_seqlens"], g["chunk_size"])
    torch.testing.assert_close(y, g["y"], rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(h, g["h_last"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("case", SSU_CASES)
def test_oracle_matches_reference_ssu(case):
    g = load_golden(case)
    i = g["inputs"]
    limit = g.get("limit", (0.0, float("inf")))
    y, h = ssd_ref.ssu_forward(f32(i["u"]), i["A"], f32(i["B"]), f32(i["C"]), i["delta_raw"], i["delta_bias"],
                               i["h"], True, limit)
    torch.testing.assert_close(h, g["h_new"], rtol=2e-5, atol=2e-6)
    # the reference rounds y to u's dtype
    torch.testing.assert_close(y.to(g["y"].dtype).float(), g["y"].float(), rtol=1e-2 if g["y"].dtype != torch.float32 else 2e-5,
                               atol=1e-2 if g["y"].dtype != torch.float32 else 2e-6)


@pytest.mark.parametrize("case", ["ssd_c0_fp32", "ssd_ragged_fp32", "ssd_threshold_fp32"])
def test_oracle_matches_fp64_recurrence(case):
    g = load_golden(case)
    i = g["inputs"]
    y64, h64 = ssd_ref.ssd_recurrence(i["u"], i["A"], i["B"], i["C"], i["delta_raw"], i["delta_bias"],
                                      i["h_init"], g["length"], g["use_sp"], g["limit"])
    y, h = run_oracle(g, dtype=torch.float64)
    torch.testing.assert_close(y, y64, rtol=1e-9, atol=1e-11)
    torch.testing.assert_close(h, h64, rtol=1e-9, atol=1e-11)


def test_prefill_plus_decode_equals_full_scan():
    """SSD over L-k tokens followed by k SSU steps equals SSD over L tokens."""
    g = torch.Generator().manual_seed(11)
    b, L, H, P, N, G, cs, k = 2, 160, 2, 16, 8, 1, 32, 24
    u = torch.randn(b, L, H, P, generator=g)
    B = torch.randn(b, L, G, N, generator=g) / math.sqrt(N)
    C = torch.randn(b, L, G, N, generator=g) / math.sqrt(N)
    dr = torch.randn(b, L, H, generator=g) - 4
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    db = 0.1 * torch.randn(H, generator=g)
    y_full, h_full = ssd_ref.ssd_scan_forward(u, A, B, C, dr, db, None, None, cs, dtype=torch.float64)
    y_pre, h = ssd_ref.ssd_scan_forward(u[:, :L - k], A, B[:, :L - k], C[:, :L - k], dr[:, :L - k], db, None,
                                        None, cs, dtype=torch.float64)
    ys = []
    for t in range(L - k, L):
        yt, h = ssd_ref.ssu_forward(u[:, t], A, B[:, t], C[:, t], dr[:, t], db, h, dtype=torch.float64)
        ys.append(yt)
    y_dec = torch.stack(ys, 1)
    torch.testing.assert_close(y_pre, y_full[:, :L - k], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(y_dec, y_full[:, L - k:], rtol=1e-9, atol=1e-11)
    torch.testing.assert_close(h, h_full, rtol=1e-9, atol=1e-11)


def test_oracle_planted_mistake_is_caught():
    """A wrong decay sign in the oracle must break agreement with the golden vectors."""
    g = load_golden("ssd_c0_fp32")
    i = g["inputs"]
    y_bad, _ = ssd_ref.ssd_scan_forward(i["u"], -i["A"], i["B"], i["C"], i["delta_raw"], None, None,
                                        g["length"], g["chunk_size"])
    assert not torch.allclose(y_bad, g["y"], rtol=1e-3, atol=1e-4)
