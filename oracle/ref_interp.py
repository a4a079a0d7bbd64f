"""Run the reference's own Triton kernels on CPU under the Triton interpreter.

TEST INFRASTRUCTURE ONLY: used by ``tests/golden/make_golden*.py`` to produce the
committed golden vectors. It needs the reference's Python sources: the directory named
by ``SA_REFERENCE_SRC`` (the checkout's ``src/``), else the copy that
``baseline/install_reference.sh`` installs into ``baseline/_ref`` of this repository.
Nothing in the product, the GPU tests or ``bench.py`` imports it.

Recipe:
- ``TRITON_INTERPRET=1`` must be set before ``triton`` is first imported;
- each autotuned forward kernel is pinned to one config (its last), so the
  autotuner does not try to benchmark (which needs a GPU driver);
- ``length`` is always passed explicitly, since the reference's default allocates
  on ``"cuda"`` (``ops/ssd_scan.py:67-68``).
"""
from __future__ import annotations

import os
import sys

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEFAULT_SRC = os.environ.get("SA_REFERENCE_SRC") or os.path.join(_REPO, "baseline", "_ref")

_loaded = None


def load():
    """Import the reference package in interpreter mode; returns a namespace dict."""
    global _loaded
    if _loaded is not None:
        return _loaded
    if "triton" in sys.modules and os.environ.get("TRITON_INTERPRET") != "1":
        raise RuntimeError("triton was imported before TRITON_INTERPRET=1 could be set")
    os.environ["TRITON_INTERPRET"] = "1"
    if not os.path.isdir(DEFAULT_SRC):
        raise FileNotFoundError(f"reference sources not found at {DEFAULT_SRC}: set SA_REFERENCE_SRC to the "
                                "reference checkout's src/ or run baseline/install_reference.sh")
    if DEFAULT_SRC not in sys.path:
        sys.path.insert(0, DEFAULT_SRC)
    import selective_attention.triton_kernels.ssd_scan.forward_kernel as fk  # noqa: E402
    for name in ("chunk_cumsum_forward_kernel", "chunk_state_forward_kernel",
                 "state_passing_forward_kernel", "bmm_chunk_forward_kernel",
                 "chunk_scan_forward_kernel"):
        k = getattr(fk, name)
        k.configs = [k.configs[-1]]
    from selective_attention.ops import SSDScanFn, SSUFn
    from selective_attention.triton_kernels.ssd_scan import forward as fwd
    _loaded = {
        "SSDScanFn": SSDScanFn,
        "SSUFn": SSUFn,
        "chunk_cumsum_forward": fwd.chunk_cumsum_forward,
        "chunk_state_forward": fwd.chunk_state_forward,
        "state_passing_forward": fwd.state_passing_forward,
        "bmm_chunk_forward": fwd.bmm_chunk_forward,
        "chunk_scan_forward": fwd.chunk_scan_forward,
    }
    return _loaded


_loaded_bwd = None


def load_backward():
    """Also pin the reference's backward kernels; returns ``ssd_scan_backward``.

    Three host wrappers of the backward size their head splits from
    ``torch.cuda.get_device_properties(device).multi_processor_count``
    (``triton_kernels/ssd_scan/backward.py:197,251,301``), which has no CPU answer:
    while this loader is in use it reports a 148-SM device for CPU tensors. The
    split count only changes the order of the reference's fp32 sums.
    """
    global _loaded_bwd
    if _loaded_bwd is not None:
        return _loaded_bwd
    ns = load()
    import types

    import torch
    import selective_attention.triton_kernels.ssd_scan.backward_kernel as bk
    for name in ("chunk_scan_backward_h_kernel", "state_passing_backward_kernel",
                 "chunk_scan_chunk_state_backward_u_kernel", "chunk_state_backward_B_kernel",
                 "chunk_scan_backward_C_grad_kernel", "chunk_scan_backward_CB_kernel",
                 "bmm_chunk_backward_kernel", "chunk_scan_backward_decay_cumsum_kernel",
                 "chunk_cumsum_backward_kernel"):
        k = getattr(bk, name)
        k.configs = [k.configs[-1]]
    real = torch.cuda.get_device_properties

    def props(device=None):
        if device is None or torch.device(device).type == "cpu":
            return types.SimpleNamespace(multi_processor_count=148)
        return real(device)

    torch.cuda.get_device_properties = props
    from selective_attention.triton_kernels.ssd_scan import backward as bwd
    _loaded_bwd = dict(ns, ssd_scan_backward=bwd.ssd_scan_backward)
    return _loaded_bwd
