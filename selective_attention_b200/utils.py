"""Tensor validation with the reference's conventions (``utils/tensor_utils.py:5-45``).

``check_ndim`` / ``check_shape`` raise ``ValueError`` before any launch, as the
reference does (``tensor_utils.py:18-38``). Messages here always carry the tensor
name; the reference's inverted conditional drops it (``:13,31,36``), so callers
must not depend on message text.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def check_ndim(tensor: Optional[torch.Tensor], ndim: int, name: Optional[str] = None, optional: bool = False):
    prefix = f"[{name}] " if name else ""
    if tensor is None:
        if not optional:
            raise ValueError(f"{prefix}Expected tensor with ndim {ndim}, but got None")
        return
    if tensor.ndim != ndim:
        raise ValueError(f"{prefix}Dim mismatch: expected ndim={ndim}, got ndim={tensor.ndim}, "
                         f"shape={tuple(tensor.shape)}")


def check_shape(tensor: Optional[torch.Tensor], shape: Tuple[int, ...], name: Optional[str] = None,
                optional: bool = False):
    prefix = f"[{name}] " if name else ""
    if tensor is None:
        if not optional:
            raise ValueError(f"{prefix}Expected tensor with shape {shape}, but got None")
    elif tuple(tensor.shape) != tuple(shape):
        raise ValueError(f"{prefix}Shape mismatch: expected {tuple(shape)}, got {tuple(tensor.shape)}")


def to_contiguous(tensor: Optional[torch.Tensor]):
    if tensor is None or tensor.is_contiguous():
        return tensor
    return tensor.contiguous()


def check_cuda(tensors, names) -> torch.device:
    """All given tensors must live on one CUDA device (there is no CPU path)."""
    dev = None
    for t, n in zip(tensors, names):
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"[{n}] expected a CUDA tensor, got device {t.device}; "
                             "the B200 SSD ops run only on the GPU")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"[{n}] is on {t.device}, other inputs are on {dev}")
    return dev
