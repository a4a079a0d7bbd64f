"""The C ABI library: it loads without a GPU, exports every symbol include/ssd_b200.h
declares, its ctypes mirror of ``ssd_params`` matches the C layout, and host-side
argument checks answer without launching anything."""
import ctypes
import os
import re
import shutil
import subprocess
import tempfile

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ssd_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s+\*?([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from selective_attention_b200 import _lib

    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 12, names
    for n in names:
        assert hasattr(L, n), f"{n} missing from {_lib.LIB_PATH}"
    assert set(names) == set(_lib.EXPORTS), "ctypes signature table out of sync with the header"
    assert L.ssd_b200_version().decode().startswith("ssd_b200")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("cname,pyname", [("ssd_params", "SSDParams"), ("ssd_bwd_params", "SSDBwdParams")])
def test_params_struct_layout_matches_c(cname, pyname):
    from selective_attention_b200 import _lib

    cls = getattr(_lib, pyname)
    fields = [f[0] for f in cls._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
            f'printf("%zu\\n", sizeof({cname}));']
    prog += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    prog += ["return 0;}"]
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "p.c")
        exe = os.path.join(d, "p")
        open(c, "w").write("\n".join(prog))
        subprocess.run(["gcc", "-std=c99", c, "-o", exe], check=True)
        out = [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(cls)
    for f, off in zip(fields, out[1:]):
        assert getattr(cls, f).offset == off, f


def test_header_constants_match_the_binding():
    from selective_attention_b200 import _lib

    src = open(HEADER).read()
    consts = dict(re.findall(r"^\s*(SSD_[A-Z_]+)\s*=\s*(\d+)", src, flags=re.M))
    assert int(consts["SSD_IMPL_AUTO"]) == _lib.IMPL_AUTO
    assert int(consts["SSD_IMPL_TC"]) == _lib.IMPL_TC
    assert int(consts["SSD_IMPL_SIMT"]) == _lib.IMPL_SIMT
    assert int(consts["SSD_IMPL_TC_STAGED"]) == _lib.IMPL_TC_STAGED
    assert int(consts["SSD_ERR_SCRATCH_LIMIT"]) == _lib.SSD_ERR_SCRATCH_LIMIT
    m = re.search(r"#define\s+SSD_FUSED_MIN_CHAINS\s+(\d+)", src)
    assert m and int(m.group(1)) == _lib.FUSED_MIN_CHAINS


def _params(**kw):
    from selective_attention_b200 import kernels

    base = dict(batch=8, seqlen=2048, nheads=24, headdim=64, dstate=128, ngroups=1, chunk_size=256,
                x_dtype=1, dt_dtype=0, y_dtype=1)
    base.update(kw)
    return kernels._params(**base)


def test_workspace_and_dispatch_queries_are_host_only():
    from selective_attention_b200 import _lib

    L = _lib.lib()
    p = _params()
    assert L.ssd_scan_uses_tensor_cores(ctypes.byref(p)) == 1
    ws = L.ssd_scan_fwd_workspace_size(ctypes.byref(p))
    nk, H = 8 * 8, 24
    # 192 (row, head) chains: chunk_state and state_passing fused, no fp32 chunk states
    expect = 2 * nk * H * 256 * 4 + nk * H * 64 * 128 * 2
    assert ws == expect
    staged = _params(impl=_lib.IMPL_TC_STAGED)
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(staged)) == expect + nk * H * 64 * 128 * 4
    few = _params(batch=4)  # 96 chains < SSD_FUSED_MIN_CHAINS: staged under AUTO, fused under TC
    nk4 = 4 * 8
    base4 = 2 * nk4 * H * 256 * 4 + nk4 * H * 64 * 128 * 2
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(few)) == base4 + nk4 * H * 64 * 128 * 4
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(_params(batch=4, impl=_lib.IMPL_TC))) == base4
    p32 = _params(x_dtype=0)
    assert L.ssd_scan_uses_tensor_cores(ctypes.byref(p32)) == 0
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(_params(nheads=24, ngroups=5))) == 0  # H % G != 0
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(_params(chunk_size=512))) == 0
    simt = _params(impl=2)
    assert L.ssd_scan_uses_tensor_cores(ctypes.byref(simt)) == 0
    # fp32 in and out: the split-bf16 tensor-core chain under AUTO (fp32 states, and per
    # (chunk, group) fourteen 32 KB operand tiles: four of B rows for chunk_state, six of
    # masked CB and four of C rows for chunk_scan),
    # the CUDA-core chain under SIMT (fp32 states and the fp32 CB)
    f32 = _params(x_dtype=0, y_dtype=0)
    assert L.ssd_scan_uses_tensor_cores(ctypes.byref(f32)) == 1
    assert L.ssd_scan_path(ctypes.byref(f32)) == 3
    assert L.ssd_scan_path(ctypes.byref(_params(x_dtype=0, y_dtype=0, impl=2))) == 0
    base32 = 2 * nk * H * 256 * 4 + nk * H * 64 * 128 * 4
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(f32)) == base32 + nk * 14 * 32768
    assert L.ssd_scan_fwd_workspace_size(ctypes.byref(_params(x_dtype=0, y_dtype=0, impl=2))) == \
        base32 + nk * 256 * 256 * 4


def test_entry_points_reject_bad_arguments_without_launching():
    from selective_attention_b200 import _lib

    L = _lib.lib()
    p = _params()  # all pointers NULL
    assert L.ssd_scan_fwd(ctypes.byref(p), None) == _lib.SSD_ERR_INVALID_ARGUMENT
    assert L.ssd_chunk_state_fwd(ctypes.byref(p), None) == _lib.SSD_ERR_INVALID_ARGUMENT
    bad = _params(x_dtype=7)
    assert L.ssd_scan_fwd(ctypes.byref(bad), None) == _lib.SSD_ERR_UNSUPPORTED_DTYPE
    assert L.ssu_fwd(*([None] * 10), 1, 1, 1, 1, 1, 0, 0, 0, 0, 1, 0.0, 1.0, None) == _lib.SSD_ERR_INVALID_ARGUMENT
    g = _lib.SSDBwdParams()
    assert L.ssd_scan_bwd(ctypes.byref(p), ctypes.byref(g), None) == _lib.SSD_ERR_INVALID_ARGUMENT
    assert L.ssd_scan_bwd_workspace_size(ctypes.byref(_params(headdim=128))) == 0  # outside the backward's shapes
    assert L.ssd_scan_bwd_workspace_size(ctypes.byref(_params())) > 0
    # fp32 u / B / C at headdim 64, dstate 128, chunk 256 add the split path's backward
    # buffers: B and C operand tiles (four 32 KB tiles per chunk and group each), accY
    # (chunk, head, 256, 64) and G = y_grad u^T (chunk, head, 256, 256), all fp32
    nk, H = 8 * 8, 24
    extra = 2 * nk * 4 * 32768 + nk * H * 256 * 64 * 4 + nk * H * 256 * 256 * 4
    assert L.ssd_scan_bwd_workspace_size(ctypes.byref(_params(x_dtype=0, y_dtype=0))) == \
        L.ssd_scan_bwd_workspace_size(ctypes.byref(_params())) + extra
    assert L.sattn_decode_step(*([None] * 7), 0, 16, None, 1, 1, 64, 0.125, 0, None) == _lib.SSD_ERR_INVALID_ARGUMENT
    assert L.sattn_prefill_fwd(*([None] * 5), 1, 1, 16, 64, 0.125, 0, 0, None) == _lib.SSD_ERR_INVALID_ARGUMENT
    for s in range(7):
        assert L.ssd_b200_status_string(s)


def test_ops_validate_like_the_reference_before_any_device_work():
    import selective_attention_b200 as sab

    u = torch.randn(2, 64, 4, 8)
    A = torch.randn(4)
    B = torch.randn(2, 64, 1, 16)
    dr = torch.randn(2, 64, 4)
    with pytest.raises(ValueError):
        sab.SSDScanFn.apply(u[0], A, B, B, dr)  # ndim
    with pytest.raises(ValueError):
        sab.SSDScanFn.apply(u, A[:3], B, B, dr)  # shape
    with pytest.raises(ValueError):
        sab.SSDScanFn.apply(u, A, B, B, dr)  # CPU tensors: no CPU path
    with pytest.raises(ValueError):
        sab.SSUFn.forward(u[:, 0], A, B[:, 0], B[:, 0], dr[:, 0], None, torch.zeros(2, 4, 8, 15))
