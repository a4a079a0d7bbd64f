"""fp32 SSD forward on tensor cores with split-bf16 products (``csrc/ssd_split.cu``).

fp32 inputs at headdim 64, dstate 128, chunk 256 take this chain under ``impl="auto"``;
``impl="simt"`` keeps the CUDA-core kernels. Both are held to the fp32 tolerance of the
north star (rel 1e-4 of each element plus 1e-5 of the tensor's largest magnitude,
``assert_fp32_close``) against the CPU oracle, whose stages restate
ssd_scan/forward_kernel.py.
"""
import pytest
import torch

from conftest import assert_fp32_close
from oracle import ssd_ref

pytestmark = pytest.mark.gpu

INF = float("inf")


def dev(t):
    return None if t is None else t.cuda()


def _inputs(seed=0, **over):
    from selective_attention_b200 import workloads

    return workloads.make_ssd_inputs(workloads.CONFIGS["c1"], seed=seed, dtype="f32", **over)


def _run(inp, impl, length=None, cu=None, h_init=None, delta_bias=None, A=None):
    import selective_attention_b200 as sab

    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"] if A is None else A), dev(inp["B"]), dev(inp["C"]),
                               dev(inp["delta_raw"]), dev(delta_bias), dev(h_init), dev(length), 256, True,
                               (0.0, INF), True, dev(inp["D"]), dev(inp["z"]), dev(cu), impl)
    sab.check_device_error()
    return y, h


def _oracle(inp, length=None, h_init=None, delta_bias=None, A=None, sl=slice(None)):
    y, h = ssd_ref.ssd_scan_forward(inp["u"][:, sl], inp["A"] if A is None else A, inp["B"][:, sl], inp["C"][:, sl],
                                    inp["delta_raw"][:, sl], delta_bias, h_init, length, 256)
    z = None if inp["z"] is None else inp["z"][:, sl]
    return ssd_ref.gate_epilogue(y, inp["u"][:, sl], inp["D"], z), h


def test_split_path_taken_for_fp32():
    from selective_attention_b200 import kernels

    inp = _inputs(batch=1, seqlen=512, nheads=2)
    p, _keep, _ = kernels.ssd_scan_params(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]),
                                          dev(inp["delta_raw"]), None, None, None, 256, True, (0.0, INF),
                                          dev(inp["D"]), dev(inp["z"]), None, "auto")
    assert kernels.scan_path(p) == "tc_split"
    assert kernels.uses_tensor_cores(p)
    p2, _keep2, _ = kernels.ssd_scan_params(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]),
                                            dev(inp["delta_raw"]), None, None, None, 256, True, (0.0, INF),
                                            dev(inp["D"]), dev(inp["z"]), None, "simt")
    assert kernels.scan_path(p2) == "simt"


def test_split_c1_heads_vs_oracle():
    """c1's head shape (H24 P64 N128, D + z) on two 2048-token rows."""
    inp = _inputs(seed=11, batch=2)
    y, h = _run(inp, "auto")
    y_ref, h_ref = _oracle(inp)
    assert_fp32_close(y, y_ref, "split y")
    assert_fp32_close(h, h_ref, "split h_last")


def test_split_ragged_init_bias_and_decay_edges_vs_oracle():
    """Ragged rows (a one-token row, a row ending inside the first half of a chunk), h_init,
    delta_bias, a head with A > 0 (the clamps of forward_kernel.py:178,438) and a fast-decay head."""
    inp = _inputs(seed=3, batch=3, seqlen=700, nheads=4, h_init=True, delta_bias=True)
    A = inp["A"].clone()
    A[1] = 0.05
    A[2] = -16.0
    db = inp["delta_bias"].clone()
    db[2] = 4.0
    length = torch.tensor([700, 300, 1])
    y, h = _run(inp, "auto", length=length, h_init=inp["h_init"], delta_bias=db, A=A)
    y_ref, h_ref = _oracle(inp, length=length, h_init=inp["h_init"], delta_bias=db, A=A)
    # rows past a row's length hold no output the reference defines beyond the zero-dt scan
    assert_fp32_close(y, y_ref, "split ragged y")
    assert_fp32_close(h, h_ref, "split ragged h_last")


def test_split_packed_varlen_vs_oracle():
    """Packed sequences (cu_seqlens) with lengths that end mid-chunk and one shorter than a half."""
    inp = _inputs(seed=5, batch=1, seqlen=1500, nheads=3)
    lens = [700, 100, 456, 244]
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int32), 0)
    y, h = _run(inp, "auto", cu=cu)
    for s in range(len(lens)):
        a, e = int(cu[s]), int(cu[s + 1])
        ys, hs = _oracle(inp, sl=slice(a, e))
        assert_fp32_close(y[:, a:e], ys, f"split seq {s} y")
        assert_fp32_close(h[s:s + 1], hs, f"split seq {s} h_last")


def test_split_groups_vs_oracle():
    """Several groups with an odd number of heads each (H6 over G2: B / C rows and the operand
    tiles are per (chunk, group)), h_init and a ragged row."""
    inp = _inputs(seed=13, batch=2, seqlen=600, nheads=6, ngroups=2, h_init=True)
    length = torch.tensor([600, 389])
    y, h = _run(inp, "auto", length=length, h_init=inp["h_init"])
    y_ref, h_ref = _oracle(inp, length=length, h_init=inp["h_init"])
    assert_fp32_close(y, y_ref, "split groups y")
    assert_fp32_close(h, h_ref, "split groups h_last")


def test_split_without_gate_returns_fp32_scan_output():
    """No D / z: y is the plain scan output (the reference contract, fp32)."""
    import selective_attention_b200 as sab

    inp = _inputs(seed=17, batch=1, seqlen=512, nheads=4, D=False, z=False)
    y, h = sab.SSDScanFn.apply(dev(inp["u"]), dev(inp["A"]), dev(inp["B"]), dev(inp["C"]), dev(inp["delta_raw"]),
                               None, None, None, 256)
    sab.check_device_error()
    y_ref, h_ref = ssd_ref.ssd_scan_forward(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None,
                                            None, 256)
    assert y.dtype == torch.float32
    assert_fp32_close(y, y_ref, "split y (no gate)")
    assert_fp32_close(h, h_ref, "split h_last (no gate)")


def test_split_and_simt_agree_and_repeat_bit_identically():
    inp = _inputs(seed=9, batch=2, seqlen=1024, nheads=8)
    y1, h1 = _run(inp, "auto")
    y2, h2 = _run(inp, "auto")
    ys, hs = _run(inp, "simt")
    assert torch.equal(y1, y2) and torch.equal(h1, h2)
    assert_fp32_close(y1, ys.double(), "split vs simt y")
    assert_fp32_close(h1, hs.double(), "split vs simt h_last")
