"""The allocation-free SSD forward, ``ssd_scan_fwd_noalloc``, called through the C ABI.

Some callers cannot allocate device memory when they run the scan (a host whose
device memory is reserved by another runtime's pool, a hot path that must not wait on
an allocation). For them the library keeps a fixed scratch array and this entry point
takes no workspace. Its output must match ``ssd_scan_fwd`` (the entry point with a
caller workspace) within the bf16 tolerance the other tests use (atol 2e-2 / rel 1e-2;
fp32: rel 1e-4), on two calls in a row, since every call reuses the same scratch.

This file is collected last so that a run stopping at the first failure has run every
other test; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from conftest import assert_bf16_close, assert_fp32_close

pytestmark = pytest.mark.gpu

INF = float("inf")


# (dtype, batch, seqlen, heads, chain the default dispatch takes). 2 x 8 (row, head)
# chains run the staged tensor-core chain (bf16) or the split-bf16 tensor-core chain (fp32,
# fp32 states and CB in the scratch array); 8 x 16 = 128 chains reach the fused chain, whose
# state pass and chunk_scan overlap through a dependent launch and read dt, cum and the
# 16-bit chunk states from the scratch array.
CASES = [
    (torch.bfloat16, 2, 700, 8, "tc_staged"),
    (torch.float32, 2, 700, 8, "tc_split"),
    (torch.bfloat16, 8, 700, 16, "tc_fused"),
]


def _inputs(dtype, seed, batch, seqlen, nheads):
    from selective_attention_b200 import workloads

    cfg = workloads.CONFIGS["c1"]
    name = {torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    inp = workloads.make_ssd_inputs(cfg, seed=seed, batch=batch, seqlen=seqlen, nheads=nheads, dtype=name,
                                    delta_bias=True, h_init=True)
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


def _params(inp, y, h_last):
    from selective_attention_b200 import kernels

    p, keep, _ = kernels.ssd_scan_params(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"],
                                         inp["delta_bias"], inp["h_init"], None, 256, True, (0.0, INF),
                                         inp["D"], inp["z"])
    p.y, p.h_last = y.data_ptr(), h_last.data_ptr()
    return p, keep


@pytest.mark.parametrize("dtype,batch,seqlen,nheads,path", CASES, ids=[c[4] for c in CASES])
def test_noalloc_matches_workspace_entry_point_twice(dtype, batch, seqlen, nheads, path):
    import selective_attention_b200 as sab
    from selective_attention_b200 import _lib, kernels

    inp = _inputs(dtype, 21, batch, seqlen, nheads)
    y_ref, h_ref = kernels.ssd_scan_forward(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"],
                                            inp["delta_bias"], inp["h_init"], None, 256, True, (0.0, INF), True,
                                            inp["D"], inp["z"])
    close = assert_bf16_close if dtype == torch.bfloat16 else assert_fp32_close
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        y = torch.full_like(y_ref, float("nan"))
        h_last = torch.full_like(h_ref, float("nan"))
        p, keep = _params(inp, y, h_last)
        assert p.workspace is None  # nothing is passed in
        assert kernels.scan_path(p) == path
        assert L.ssd_scan_fwd_workspace_size(ctypes.byref(p)) <= (32 << 20)
        st = L.ssd_scan_fwd_noalloc(ctypes.byref(p), stream)
        assert st == _lib.SSD_OK, L.ssd_b200_status_string(st).decode()
        torch.cuda.synchronize()
        sab.check_device_error()
        close(y.float(), y_ref.float(), f"noalloc call {call} y")
        close(h_last, h_ref, f"noalloc call {call} h_last")


def test_noalloc_rejects_problems_beyond_its_scratch():
    from selective_attention_b200 import _lib, kernels

    L = _lib.lib()
    p = kernels._params(batch=16, seqlen=2048, nheads=24, headdim=64, dstate=128, ngroups=1, chunk_size=256,
                        x_dtype=1, dt_dtype=0, y_dtype=1)
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(p)) > (32 << 20)
    st = L.ssd_scan_fwd_noalloc(ctypes.byref(p), None)
    assert st == _lib.SSD_ERR_SCRATCH_LIMIT
    assert b"scratch" in L.ssd_b200_status_string(st)
