"""ctypes binding of ``libssd_b200.so`` (the C ABI in ``include/ssd_b200.h``).

The library is required: there is no CPU or eager fallback. ``lib()`` raises
``RuntimeError`` when the shared object has not been built, and the op wrappers
raise ``ValueError`` for tensors that are not on a CUDA device.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libssd_b200.so")

SSD_OK = 0
SSD_ERR_INVALID_ARGUMENT = 1
SSD_ERR_UNSUPPORTED_DTYPE = 2
SSD_ERR_WORKSPACE_TOO_SMALL = 3
SSD_ERR_SCRATCH_LIMIT = 7

IMPL_AUTO, IMPL_TC, IMPL_SIMT, IMPL_TC_STAGED = 0, 1, 2, 3
IMPLS = {"auto": IMPL_AUTO, "tc": IMPL_TC, "simt": IMPL_SIMT, "tc_staged": IMPL_TC_STAGED}
FUSED_MIN_CHAINS = 128  # SSD_FUSED_MIN_CHAINS

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

# Every symbol include/ssd_b200.h declares, with its ctypes signature.
EXPORTS = {
    "ssd_b200_version": (ctypes.c_char_p, []),
    "ssd_b200_status_string": (ctypes.c_char_p, [c_int]),
    "ssd_b200_device_error": (c_int, [c_void_p]),
    "ssd_scan_uses_tensor_cores": (c_int, [c_void_p]),
    "ssd_scan_path": (c_int, [c_void_p]),
    "ssd_scan_fwd_workspace_size": (c_size_t, [c_void_p]),
    "ssd_scan_fwd": (c_int, [c_void_p, c_void_p]),
    "ssd_scan_fwd_noalloc": (c_int, [c_void_p, c_void_p]),
    "ssd_scan_bwd_workspace_size": (c_size_t, [c_void_p]),
    "ssd_scan_bwd": (c_int, [c_void_p, c_void_p, c_void_p]),
    "ssd_chunk_cumsum_fwd": (c_int, [c_void_p, c_void_p]),
    "ssd_chunk_state_fwd": (c_int, [c_void_p, c_void_p]),
    "ssd_state_passing_fwd": (c_int, [c_void_p, c_void_p]),
    "ssd_bmm_chunk_fwd": (c_int, [c_void_p, c_void_p]),
    "ssd_chunk_scan_fwd": (c_int, [c_void_p, c_void_p]),
    "ssu_fwd": (c_int, [c_void_p] * 10 + [c_int64] * 5 + [c_int32] * 5 + [c_float, c_float, c_void_p]),
    "ssm_conv_prefill": (c_int, [c_void_p, c_int64] + [c_void_p] * 7 + [c_int64] * 5 + [c_int32, c_void_p]),
    "ssm_conv_decode": (c_int, [c_void_p, c_int64] + [c_void_p] * 6 + [c_int64] * 4 + [c_int32, c_void_p]),
    "sattn_decode_step": (c_int, [c_void_p] * 7 + [c_int64, c_int64, c_void_p] + [c_int64] * 3
                          + [c_float, c_int32, c_void_p]),
    "sattn_prefill_fwd": (c_int, [c_void_p] * 5 + [c_int64] * 4 + [c_float, c_int32, c_int32, c_void_p]),
    "sattn_train_workspace_size": (c_size_t, [c_void_p]),
    "sattn_train_fwd": (c_int, [c_void_p, c_void_p]),
    "sattn_train_bwd": (c_int, [c_void_p] * 7),
}


class SSDParams(ctypes.Structure):
    """Mirror of ``ssd_params`` in include/ssd_b200.h (same field order and types)."""

    _fields_ = [
        ("batch", c_int64), ("seqlen", c_int64), ("nheads", c_int64), ("headdim", c_int64),
        ("dstate", c_int64), ("ngroups", c_int64), ("chunk_size", c_int64), ("nseq", c_int64),
        ("x_dtype", c_int32), ("dt_dtype", c_int32), ("y_dtype", c_int32), ("cu_dtype", c_int32),
        ("use_delta_softplus", c_int32), ("delta_min", c_float), ("delta_max", c_float), ("impl", c_int32),
        ("u", c_void_p), ("A", c_void_p), ("B", c_void_p), ("C", c_void_p), ("delta_raw", c_void_p),
        ("delta_bias", c_void_p), ("h_init", c_void_p), ("length", c_void_p), ("D", c_void_p), ("z", c_void_p),
        ("cu_seqlens", c_void_p), ("y", c_void_p), ("h_last", c_void_p), ("dt", c_void_p), ("cum", c_void_p),
        ("states", c_void_p), ("CB", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("events", c_void_p * 6),
    ]


class SSDBwdParams(ctypes.Structure):
    """Mirror of ``ssd_bwd_params`` in include/ssd_b200.h."""

    _fields_ = [
        ("y_grad", c_void_p), ("y_grad_dtype", c_int32), ("h_last_grad", c_void_p), ("u_grad", c_void_p),
        ("A_grad", c_void_p), ("B_grad", c_void_p), ("C_grad", c_void_p), ("delta_raw_grad", c_void_p),
        ("delta_bias_grad", c_void_p), ("h_init_grad", c_void_p),
    ]


class SattnTrainParams(ctypes.Structure):
    """Mirror of ``sattn_train_params`` in include/ssd_b200.h."""

    _fields_ = [
        ("batch", c_int64), ("nheads", c_int64), ("seqlen", c_int64), ("head_dim", c_int64),
        ("dtype", c_int32), ("is_causal", c_int32), ("impl", c_int32), ("scale", c_float),
        ("log_gate_penalty", c_float),
        ("q_rot", c_void_p), ("k_rot", c_void_p), ("v", c_void_p), ("select_gate", c_void_p), ("lengths", c_void_p),
        ("out", c_void_p), ("lse", c_void_p), ("log_gate", c_void_p), ("stats", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


_LIB = None


def lib() -> ctypes.CDLL:
    """Load the CUDA library once; raise if it is missing (no fallback path exists)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m selective_attention_b200._build` "
                "(the B200 SSD ops have no fallback implementation)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in EXPORTS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype, what: str) -> int:
    try:
        return DTYPE_CODES[dt]
    except KeyError:
        raise ValueError(f"[{what}] unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, what: str) -> None:
    if status == SSD_OK:
        return
    msg = f"{what}: {lib().ssd_b200_status_string(status).decode()} (status {status})"
    if status in (SSD_ERR_INVALID_ARGUMENT, SSD_ERR_UNSUPPORTED_DTYPE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error(device=None) -> int:
    """Synchronize the current stream and return (and clear) the kernels' error flag."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(lib().ssd_b200_device_error(c_void_p(stream_handle(dev))))


def check_device_error(device=None) -> None:
    """Raise ``RuntimeError`` if a kernel gave up on a bounded wait since the last check."""
    code = device_error(device)
    if code:
        raise RuntimeError(f"ssd_b200 kernel reported device error 0x{code:x} (a bounded wait timed out)")
