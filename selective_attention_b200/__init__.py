"""B200-native SSD chunked scan (forward and backward), selective state update, the SSM
layer's conv front ends and the selective-attention inference kernels.

Public surface (mirrors the reference's ``selective_attention.ops`` and
``selective_attention.triton_kernels``):

- ``SSDScanFn`` / ``SSUFn``: drop-in ops with the reference's signatures.
- ``SelectiveAttnTrainFn``: the training-mode selective attention (score statistics, std-scaled
  gates, gated softmax) with its backward.
- ``kernels``: stage-level host functions (``chunk_cumsum_forward`` ... ``ssd_scan_forward``,
  ``ssd_scan_backward``, ``ssu_forward``, ``ssm_conv_prefill`` / ``ssm_conv_decode``,
  ``sattn_decode_step`` / ``selective_attn_step`` / ``sattn_prefill``) over the C ABI of
  ``libssd_b200.so`` (``include/ssd_b200.h``).
- ``HostStreamScan``: the SSD forward on inputs in pinned host memory, with the copies
  of row slices overlapped with the scan (no reference counterpart).
- ``shim.install()``: make an installed reference package use these kernels.
- ``check_device_error()``: surface a kernel's bounded-wait timeout as ``RuntimeError``.
"""
from ._lib import check_device_error, device_error
from .ops import SSDScanFn, SSUFn, SelectiveAttnTrainFn, selective_attn_train
from .streaming import HostStreamScan
from .kernels import (
    bmm_chunk_forward,
    chunk_cumsum_forward,
    chunk_scan_forward,
    chunk_state_forward,
    sattn_decode_step,
    sattn_prefill,
    sattn_train_backward,
    sattn_train_forward,
    selective_attn_step,
    ssd_scan_backward,
    ssd_scan_forward,
    ssm_conv_decode,
    ssm_conv_prefill,
    ssu_forward,
    state_passing_forward,
)

__all__ = [
    "SSDScanFn", "SSUFn", "HostStreamScan", "ssd_scan_forward", "ssu_forward", "chunk_cumsum_forward",
    "chunk_state_forward", "state_passing_forward", "bmm_chunk_forward", "chunk_scan_forward",
    "ssd_scan_backward", "ssm_conv_prefill", "ssm_conv_decode", "sattn_decode_step", "selective_attn_step",
    "sattn_prefill", "sattn_train_forward", "sattn_train_backward", "SelectiveAttnTrainFn", "selective_attn_train",
    "check_device_error", "device_error",
]
