"""SSD forward on the GPU against the reference's golden vectors and the CPU oracle.

Tolerances (north_star): fp32 within rel 1e-4 (assert_fp32_close), bf16 within
atol 2e-2 / rel 1e-2 (assert_bf16_close); both defined in conftest.py.
"""
import math

import pytest
import torch

from conftest import (SSD_CASES, assert_bf16_close, assert_close_for, assert_fp32_close, load_golden)
from oracle import ssd_ref

pytestmark = pytest.mark.gpu

INF = float("inf")


def dev(t):
    return None if t is None else t.cuda()


def run_case(g, impl, D=None, z=None):
    import selective_attention_b200 as sab

    i = g["inputs"]
    args = [dev(i[k]) for k in ("u", "A", "B", "C", "delta_raw", "delta_bias", "h_init")] + [dev(g["length"])]
    y, h = sab.SSDScanFn.apply(*args, g["chunk_size"], g["use_sp"], g["limit"], True, dev(D), dev(z), None, impl)
    sab.check_device_error()
    return y, h


TC_IMPLS = ["tc", "tc_staged"]  # chunk_state + state_passing fused / as separate launches


def skip_tc_for_fp32(g, impl):
    if impl in TC_IMPLS and g["inputs"]["u"].dtype == torch.float32:
        pytest.skip("the tensor-core kernels take 16-bit inputs")


@pytest.mark.parametrize("impl", ["auto", "simt"] + TC_IMPLS)
@pytest.mark.parametrize("case", SSD_CASES)
def test_ssd_matches_reference_golden(case, impl):
    g = load_golden(case)
    skip_tc_for_fp32(g, impl)
    y, h = run_case(g, impl)
    assert y.dtype == torch.float32 and h.dtype == torch.float32
    close = assert_close_for(g["inputs"]["u"].dtype)
    close(y, g["y"], f"{case}/{impl} y")
    close(h, g["h_last"], f"{case}/{impl} h_last")


@pytest.mark.parametrize("case", ["ssd_bf16_c1slice", "ssd_bf16_groups"])
def test_tensor_core_path_is_taken_for_bf16(case):
    from selective_attention_b200 import kernels

    g = load_golden(case)
    i = g["inputs"]
    p, keep, _ = kernels.ssd_scan_params(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]),
                                         chunk_size=g["chunk_size"])
    assert kernels.uses_tensor_cores(p)


@pytest.mark.parametrize("impl", ["auto", "simt"] + TC_IMPLS)
@pytest.mark.parametrize("case", ["ssd_bf16_c1slice", "ssd_bf16_groups", "ssd_c0_fp32"])
def test_ssd_fused_gate_epilogue(case, impl):
    """(y + D*u) * silu(z) fused in the scan epilogue, vs modules/ssm.py:145-150 on the golden y."""
    g = load_golden(case)
    skip_tc_for_fp32(g, impl)
    i = g["inputs"]
    D, z = i["D"], i["z"]
    y, h = run_case(g, impl, D=D, z=z)
    assert y.dtype == i["u"].dtype
    ref = ssd_ref.gate_epilogue(g["y"], i["u"], D, z)
    assert_close_for(i["u"].dtype)(y, ref, f"{case}/{impl} gated y")
    assert_close_for(i["u"].dtype)(h, g["h_last"], f"{case}/{impl} h_last")


@pytest.mark.parametrize("impl", ["auto", "simt"] + TC_IMPLS)
def test_ssd_varlen_matches_padded_reference(impl):
    import selective_attention_b200 as sab

    g = load_golden("ssd_varlen_bf16")
    i = g["inputs"]
    for cu in (g["cu_seqlens"], g["cu_seqlens"].long()):
        y, h = sab.SSDScanFn.apply(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]), None,
                                   None, None, g["chunk_size"], True, (0.0, INF), True, None, None, dev(cu), impl)
        sab.check_device_error()
        assert h.shape == (3, 2, 64, 128)
        assert_bf16_close(y, g["y"], "varlen y")
        assert_bf16_close(h, g["h_last"], "varlen h_last")


@pytest.mark.parametrize("case", ["ssd_c0_fp32", "ssd_ragged_fp32"])
def test_ssd_stages_match_reference(case):
    from selective_attention_b200 import kernels

    g = load_golden(case)
    i = g["inputs"]
    cs = g["chunk_size"]
    cum, dt = kernels.chunk_cumsum_forward(dev(i["A"]), dev(i["delta_raw"]), dev(i["delta_bias"]),
                                           dev(g["length"]), cs, g["use_sp"], g["limit"])
    assert_fp32_close(dt, g["dt"], "dt")
    torch.testing.assert_close(cum.cpu(), g["cum"], rtol=1e-4, atol=1e-4)
    S = kernels.chunk_state_forward(dev(i["u"]), dev(i["B"]), dev(g["dt"]), dev(g["cum"]))
    assert_fp32_close(S, g["states"], "states")
    b, nc, H, P, N = S.shape
    hs = S.view(b, nc, H, P * N)
    hi = None if i["h_init"] is None else dev(i["h_init"]).view(b, H, P * N)
    prev, h_last = kernels.state_passing_forward(hs, hi, dev(g["cum"][..., -1]))
    assert_fp32_close(prev.view(b, nc, H, P, N), g["prev"], "prev states")
    assert_fp32_close(h_last.view(b, H, P, N), g["h_last"], "h_last")
    CB = kernels.bmm_chunk_forward(dev(i["B"]), dev(i["C"]), cs, True)
    low = torch.tril(torch.ones(cs, cs, dtype=torch.bool))
    assert_fp32_close(CB.cpu()[..., low], g["CB"][..., low], "CB lower triangle")
    y = kernels.chunk_scan_forward(dev(i["u"]), dev(g["dt"]), dev(g["cum"]), dev(i["C"]), dev(g["prev"]),
                                   dev(g["CB"]))
    assert_fp32_close(y, g["y_stage"], "chunk_scan y")


def test_tc_chunk_state_stage_bf16():
    """Tensor-core chunk_state against the oracle on the bf16 golden inputs."""
    from selective_attention_b200 import kernels

    g = load_golden("ssd_bf16_groups")
    i = g["inputs"]
    cum, dt = kernels.chunk_cumsum_forward(dev(i["A"]), dev(i["delta_raw"]), dev(i["delta_bias"]),
                                           dev(g["length"]), 256)
    S_tc = kernels.chunk_state_forward(dev(i["u"]), dev(i["B"]), dt, cum, impl="tc")
    S_ref = ssd_ref.chunk_state(i["u"].float(), i["B"].float(), dt.cpu(), cum.cpu())
    assert_bf16_close(S_tc, S_ref, "tc chunk_state")


def _c_inputs(name, seed=0, **over):
    from selective_attention_b200 import workloads

    return workloads.make_ssd_inputs(workloads.CONFIGS[name], seed=seed, **over)


@pytest.mark.parametrize("impl", ["auto", "simt", "tc_staged"])
def test_c1_full_size_vs_oracle(impl):
    """Benchmark config c1 at full size (8 x 2048, H24 P64 N128, cs256, D + z)."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c1")
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                               None, None, None, 256, True, (0.0, INF), True, dev(inp["D"]), dev(inp["z"]), None,
                               impl)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_forward(inp["u"].float(), inp["A"], inp["B"].float(), inp["C"].float(),
                                            inp["delta_raw"], None, None, None, 256)
    y_ref = ssd_ref.gate_epilogue(y_ref, inp["u"], inp["D"], inp["z"])
    assert_bf16_close(y, y_ref, "c1 y")
    assert_bf16_close(h, h_ref, "c1 h_last")


@pytest.mark.parametrize("impl", TC_IMPLS)
def test_c4_shape_groups_partial_chunks_vs_oracle(impl):
    """c4 head/group shape (H16 over G8, 2 heads per group) with ragged rows and h_init."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c4", seed=3, batch=2, seqlen=1000, nheads=16, h_init=True, delta_bias=True)
    length = torch.tensor([1000, 613])
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                               dev(inp["delta_bias"]), dev(inp["h_init"]), dev(length), 256, True, (0.0, INF), True,
                               dev(inp["D"]), dev(inp["z"]), None, impl)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_forward(inp["u"].float(), inp["A"], inp["B"].float(), inp["C"].float(),
                                            inp["delta_raw"], inp["delta_bias"], inp["h_init"], length, 256)
    y_ref = ssd_ref.gate_epilogue(y_ref, inp["u"], inp["D"], inp["z"])
    assert_bf16_close(y, y_ref, "c4-shape y")
    assert_bf16_close(h, h_ref, "c4-shape h_last")


@pytest.mark.parametrize("impl", ["auto", "tc_staged"])
def test_c2_varlen_full_size_vs_oracle(impl):
    """Benchmark config c2: 32768 packed tokens, lengths U[128, 4096], H80, D + z."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c2")
    cu = inp["cu_seqlens"]
    assert int(cu[-1]) == 32768
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                               None, None, None, 256, True, (0.0, INF), True, dev(inp["D"]), dev(inp["z"]), dev(cu),
                               impl)
    sab.check_device_error()
    # oracle on the first three sequences and the last one (each sequence is independent)
    idx = [0, 1, 2, cu.numel() - 2]
    for s in idx:
        a, e = int(cu[s]), int(cu[s + 1])
        ys, hs = ssd_ref.ssd_scan_forward(inp["u"][:, a:e].float(), inp["A"], inp["B"][:, a:e].float(),
                                          inp["C"][:, a:e].float(), inp["delta_raw"][:, a:e], None, None, None, 256)
        ys = ssd_ref.gate_epilogue(ys, inp["u"][:, a:e], inp["D"], inp["z"][:, a:e])
        assert_bf16_close(y[:, a:e], ys, f"c2 seq {s} y")
        assert_bf16_close(h[s:s + 1], hs, f"c2 seq {s} h_last")


@pytest.mark.parametrize("impl", ["simt"] + TC_IMPLS)
def test_decay_edge_cases_vs_oracle(impl):
    """A head with A > 0 (the min(., 0) clamps of forward_kernel.py:178,438 are active),
    a head with a very fast decay (dt ~ 1, |A| up to 16: the factored decay would overflow
    on diagonal tiles, so the element-by-element form must be used), plus two ordinary heads."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c1", seed=7, batch=2, seqlen=520, nheads=4)
    A = inp["A"].clone()
    A[1] = 0.05
    A[2] = -16.0
    db = torch.zeros(4)
    db[2] = 4.0
    length = torch.tensor([520, 300])
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(A), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]), dev(db),
                               None, dev(length), 256, True, (0.0, INF), True, dev(inp["D"]), dev(inp["z"]), None,
                               impl)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_forward(inp["u"].float(), A, inp["B"].float(), inp["C"].float(),
                                            inp["delta_raw"], db, None, length, 256)
    y_ref = ssd_ref.gate_epilogue(y_ref, inp["u"], inp["D"], inp["z"])
    assert_bf16_close(y, y_ref, f"{impl} y")
    assert_bf16_close(h, h_ref, f"{impl} h_last")


def test_tc_and_simt_agree():
    """Both device paths on the same bf16 inputs (two chunks, ragged length)."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c1", seed=5, batch=3, seqlen=700)
    length = torch.tensor([700, 513, 1])
    outs = {}
    for impl in ("tc", "tc_staged", "simt"):
        outs[impl] = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]),
                                         dev(inp["delta_raw"]), None, None, dev(length), 256, True, (0.0, INF), True,
                                         dev(inp["D"]), dev(inp["z"]), None, impl)
    sab.check_device_error()
    for impl in TC_IMPLS:
        assert_bf16_close(outs[impl][0], outs["simt"][0].float(), f"{impl} vs simt y")
        assert_bf16_close(outs[impl][1], outs["simt"][1], f"{impl} vs simt h_last")


def test_prefill_then_decode_matches_full_scan():
    """SSD over L-k tokens then k SSU steps == SSD over L tokens (reference test_causal_lm.py:55-133, op level)."""
    import selective_attention_b200 as sab

    g = torch.Generator().manual_seed(12)
    b, L, H, P, N, G, cs, k = 2, 256, 4, 64, 128, 1, 64, 56
    u = torch.randn(b, L, H, P, generator=g)
    B = torch.randn(b, L, G, N, generator=g) / math.sqrt(N)
    C = torch.randn(b, L, G, N, generator=g) / math.sqrt(N)
    dr = torch.randn(b, L, H, generator=g) - 4
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    db = 0.1 * torch.randn(H, generator=g)
    u, B, C, dr, A, db = (t.cuda() for t in (u, B, C, dr, A, db))
    y_full, h_full = sab.SSDScanFn.apply(u, A, B, C, dr, db, None, None, cs)
    _, h = sab.SSDScanFn.apply(u[:, :L - k], A, B[:, :L - k], C[:, :L - k], dr[:, :L - k], db, None, None, cs)
    ys = []
    for t in range(L - k, L):
        yt, h = sab.SSUFn.forward(u[:, t], A, B[:, t], C[:, t], dr[:, t], db, h)
        ys.append(yt)
    sab.check_device_error()
    assert_fp32_close(torch.stack(ys, 1), y_full[:, L - k:], "decoded y")
    assert_fp32_close(h, h_full, "decoded state")


def test_errors_before_launch():
    import selective_attention_b200 as sab

    g = load_golden("ssd_c0_fp32")
    i = g["inputs"]
    with pytest.raises(ValueError):  # CPU tensors: no CPU path exists
        sab.SSDScanFn.apply(i["u"], i["A"], i["B"], i["C"], i["delta_raw"])
    with pytest.raises(ValueError):  # A has the wrong shape
        sab.SSDScanFn.apply(dev(i["u"]), dev(i["A"][:3]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]))
    with pytest.raises(ValueError):  # chunk_size above the supported 256
        sab.SSDScanFn.apply(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]), None, None,
                            None, 512)
    with pytest.raises(ValueError):  # tensor-core path requested for fp32
        sab.SSDScanFn.apply(dev(i["u"]), dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]), None, None,
                            None, 64, True, (0.0, INF), True, None, None, None, "tc")
    assert sab.device_error() == 0


def test_backward_through_fused_epilogue_raises():
    import selective_attention_b200 as sab

    g = load_golden("ssd_c0_fp32")
    i = g["inputs"]
    u = dev(i["u"]).requires_grad_(True)
    D = torch.ones(u.shape[2] * u.shape[3], device="cuda")
    y, _ = sab.SSDScanFn.apply(u, dev(i["A"]), dev(i["B"]), dev(i["C"]), dev(i["delta_raw"]), None, None, None, 64,
                               True, (0.0, INF), True, D)
    with pytest.raises(NotImplementedError):
        y.sum().backward()


@pytest.mark.parametrize("slices", [1, 3])
def test_host_stream_scan_matches_device_scan(slices):
    """HostStreamScan (host inputs, row slices through the copy-in / scan / copy-out
    pipeline, buffer sets reused) == ssd_scan_forward on the device."""
    import selective_attention_b200 as sab
    from selective_attention_b200 import kernels

    inp = _c_inputs("c1", seed=9, batch=5, seqlen=600, nheads=8, h_init=True, delta_bias=True)
    length = torch.tensor([600, 512, 333, 1, 600])
    host = {k: inp[k].pin_memory() for k in ("u", "B", "C", "delta_raw", "z", "h_init")}
    scan = sab.HostStreamScan(slices=slices, in_flight=2)
    for _ in range(2):  # second call reuses the device buffers
        y, h = scan(host["u"], inp["A"], host["B"], host["C"], host["delta_raw"], inp["delta_bias"], host["h_init"],
                    length, 256, True, (0.0, INF), inp["D"], host["z"])
        torch.cuda.synchronize()
        sab.check_device_error()
        assert not y.is_cuda and not h.is_cuda
        y_ref, h_ref = kernels.ssd_scan_forward(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]),
                                                dev(inp["delta_raw"]), dev(inp["delta_bias"]), dev(inp["h_init"]),
                                                dev(length), 256, True, (0.0, INF), True, dev(inp["D"]), dev(inp["z"]))
        assert_bf16_close(y.float(), y_ref.float().cpu(), f"stream scan y ({slices} slices)")
        assert_bf16_close(h, h_ref.cpu(), f"stream scan h_last ({slices} slices)")
    with pytest.raises(ValueError):
        scan(dev(inp["u"]), inp["A"], host["B"], host["C"], host["delta_raw"])


@pytest.mark.parametrize("impl", TC_IMPLS)
def test_packed_edge_lengths_odd_heads_per_group(impl):
    """Packed rows of lengths 1, 0, 63, 129, 256, 300, 17 with 3 heads per group (the
    fused kernel's last head pair holds one head), h_init per sequence, D and z, against
    the padded oracle (each sequence its own row with length = seqlen)."""
    import selective_attention_b200 as sab

    g = torch.Generator().manual_seed(31)
    lens = [1, 0, 63, 129, 256, 300, 17]
    T, H, P, N, G = sum(lens), 6, 64, 128, 2
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    u = torch.randn(1, T, H, P, generator=g).bfloat16()
    B = (torch.randn(1, T, G, N, generator=g) / math.sqrt(N)).bfloat16()
    C = (torch.randn(1, T, G, N, generator=g) / math.sqrt(N)).bfloat16()
    dr = torch.randn(1, T, H, generator=g) - 4.0
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    db = 0.1 * torch.randn(H, generator=g)
    h0 = 0.1 * torch.randn(len(lens), H, P, N, generator=g)
    D = torch.randn(H * P, generator=g)
    z = torch.randn(1, T, H, P, generator=g).bfloat16()
    y, h = sab.SSDScanFn.apply(dev(u), dev(A), dev(B), dev(C), dev(dr), dev(db), dev(h0), None, 256, True,
                               (0.0, INF), True, dev(D), dev(z), dev(cu), impl)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_varlen(u.float(), A, B.float(), C.float(), dr, db, cu, 256, h_init=h0)
    y_ref = ssd_ref.gate_epilogue(y_ref, u, D, z)
    assert_bf16_close(y, y_ref, f"packed edge y ({impl})")
    assert_bf16_close(h, h_ref, f"packed edge h_last ({impl})")


@pytest.mark.parametrize("impl", TC_IMPLS)
def test_padded_odd_heads_per_group_ragged(impl):
    """Padded rows with 3 heads per group, ragged lengths and h_init (fused kernel's
    single-head pair on the padded path)."""
    import selective_attention_b200 as sab

    inp = _c_inputs("c4", seed=13, batch=3, seqlen=700, nheads=6, h_init=True, delta_bias=True)
    length = torch.tensor([700, 129, 0])
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"][:, :, :2]), dev(inp["C"][:, :, :2]),
                               dev(inp["delta_raw"]), dev(inp["delta_bias"]), dev(inp["h_init"]), dev(length), 256,
                               True, (0.0, INF), True, dev(inp["D"]), dev(inp["z"]), None, impl)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_forward(inp["u"].float(), inp["A"], inp["B"][:, :, :2].float(),
                                            inp["C"][:, :, :2].float(), inp["delta_raw"], inp["delta_bias"],
                                            inp["h_init"], length, 256)
    y_ref = ssd_ref.gate_epilogue(y_ref, inp["u"], inp["D"], inp["z"])
    assert_bf16_close(y, y_ref, f"odd heads y ({impl})")
    assert_bf16_close(h, h_ref, f"odd heads h_last ({impl})")


@pytest.mark.parametrize("impl", TC_IMPLS)
def test_repeated_runs_are_bit_identical(impl):
    """Every kernel of the chain is deterministic (no atomics, fixed MMA order), so
    repeated runs on the same inputs must agree bit for bit. A missing wait between the
    warp roles shows up here as rare differing runs long before it breaks a tolerance
    (c2: packed ragged rows, 10 head blocks, many item boundaries per CTA)."""
    from selective_attention_b200 import kernels, workloads

    inp = workloads.make_ssd_inputs(workloads.CONFIGS["c2"], seed=0, device=torch.device("cuda"), gen_device="cuda")
    args = (inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None, None, 256, True, (0.0, INF), True,
            inp["D"], inp["z"], inp["cu_seqlens"])
    y0, h0 = kernels.ssd_scan_forward(*args, impl=impl)
    differ = 0
    for _ in range(40):
        y, h = kernels.ssd_scan_forward(*args, impl=impl)
        differ += int(not (torch.equal(y, y0) and torch.equal(h, h0)))
    torch.cuda.synchronize()
    assert differ == 0, f"{differ} of 40 runs differ from the first"


def _oracle_slice(inp, row, group, hpg, chunk=256):
    """Oracle y (with the D / z epilogue) and h_last of one batch row x one head group:
    the scan is independent per (row, group), so a slice of the full problem is a
    complete problem of its own."""
    hs = slice(group * hpg, (group + 1) * hpg)
    P = inp["u"].shape[-1]
    u = inp["u"][row:row + 1, :, hs].cpu()
    B = inp["B"][row:row + 1, :, group:group + 1].cpu().float()
    C = inp["C"][row:row + 1, :, group:group + 1].cpu().float()
    dr = inp["delta_raw"][row:row + 1, :, hs].cpu()
    A = inp["A"][hs].cpu()
    D = inp["D"][group * hpg * P:(group + 1) * hpg * P].cpu()
    z = inp["z"][row:row + 1, :, group * hpg * P:(group + 1) * hpg * P].cpu()
    y, h = ssd_ref.ssd_scan_forward(u.float(), A, B, C, dr, None, None, None, chunk)
    return ssd_ref.gate_epilogue(y, u, D, z), h


def test_c4_full_size_first_and_last_row_group_vs_oracle():
    """Benchmark config c4 at its real size on one GPU: 8 x 65536 tokens, H128 over G8
    (16 heads a group), P64 N128, cs256, D + z, bf16: 256 chunks per state chain and
    u / z / y of 4.3e9 elements, so byte offsets run far past 2^32. The first and the last
    (row, group) slices, which hold the smallest and the largest offsets, are checked
    against the oracle (forward.py:223-276 over the whole chain)."""
    import selective_attention_b200 as sab
    from selective_attention_b200 import kernels, workloads

    cfg = workloads.CONFIGS["c4"]
    inp = workloads.make_ssd_inputs(cfg, seed=0, device=torch.device("cuda"), gen_device="cuda")
    p, keep, _ = kernels.ssd_scan_params(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None, None,
                                         256, True, (0.0, INF), inp["D"], inp["z"])
    assert kernels.scan_path(p) == "tc_fused"
    y, h = kernels.ssd_scan_forward(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None, None, 256,
                                    True, (0.0, INF), True, inp["D"], inp["z"])
    torch.cuda.synchronize()
    sab.check_device_error()
    assert y.numel() * y.element_size() > (1 << 32)  # byte offsets beyond 32 bits
    hpg = cfg.nheads // cfg.ngroups
    for row, group in ((0, 0), (cfg.batch - 1, cfg.ngroups - 1)):
        y_ref, h_ref = _oracle_slice(inp, row, group, hpg)
        hs = slice(group * hpg, (group + 1) * hpg)
        assert_bf16_close(y[row:row + 1, :, hs], y_ref, f"c4 row {row} group {group} y")
        assert_bf16_close(h[row:row + 1, hs], h_ref, f"c4 row {row} group {group} h_last")


def test_c1_default_dispatch_repeated_runs_are_bit_identical():
    """c1 on the default dispatch: the fused chain with 8 rows x 12 head pairs = 96 state
    chains, one wave on 148 SMs, so chunk_scan is launched as a programmatic dependent of
    the state pass and its producer waits on the grid before reading dt, cum and the
    16-bit states. 40 repeated runs must match the first bit for bit."""
    from selective_attention_b200 import kernels, workloads

    inp = workloads.make_ssd_inputs(workloads.CONFIGS["c1"], seed=0, device=torch.device("cuda"), gen_device="cuda")
    args = (inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None, None, 256, True, (0.0, INF), True,
            inp["D"], inp["z"], None)
    p, keep, _ = kernels.ssd_scan_params(*args[:11], inp["D"], inp["z"])
    assert kernels.scan_path(p) == "tc_fused"
    y0, h0 = kernels.ssd_scan_forward(*args)
    differ = 0
    for _ in range(40):
        y, h = kernels.ssd_scan_forward(*args)
        differ += int(not (torch.equal(y, y0) and torch.equal(h, h0)))
    torch.cuda.synchronize()
    assert differ == 0, f"{differ} of 40 runs differ from the first"
