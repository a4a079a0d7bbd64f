"""``SSUFn``: drop-in for the reference's ``ops/ssu.py:8-63``.

An ``nn.Module`` whose ``forward`` is a ``@staticmethod`` run under
``torch.inference_mode()`` (``:9-10``), with the reference's positional signature
``(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus, delta_limit)``, its
``ValueError`` checks (``:35-51``) and contiguity handling (``:53-59``). ``h`` is
updated in place and returned; ``y`` has ``u``'s dtype (``ssu/forward.py:34``).
As in the reference, a non-contiguous ``h`` is copied first, so the caller's
tensor is then not the one updated: rebind it to the returned ``h``.

Extension (optional trailing positional): ``D`` (``(H*P,)``) and ``z``
(``(b, H*P)`` or ``(b, H, P)``) apply the decode epilogue of ``modules/ssm.py:199-202``,
``y = (y + D*u) * silu(z)``, inside the kernel.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn

from .. import kernels
from ..utils import check_ndim, check_shape, to_contiguous

INF = float("inf")


class SSUFn(nn.Module):
    @staticmethod
    @torch.inference_mode()
    def forward(
        u: torch.Tensor,
        A: torch.Tensor,
        B: torch.Tensor,
        C: torch.Tensor,
        delta_raw: torch.Tensor,
        delta_bias: torch.Tensor | None,
        h: torch.Tensor,
        use_delta_softplus: bool = True,
        delta_limit: Tuple = (0.0, INF),
        D: torch.Tensor | None = None,
        z: torch.Tensor | None = None,
    ):
        check_ndim(u, 3, name="u")
        check_ndim(A, 1, name="A")
        check_ndim(B, 3, name="B")
        check_ndim(C, 3, name="C")
        check_ndim(delta_raw, 2, name="delta_raw")
        check_ndim(delta_bias, 1, name="delta_bias", optional=True)
        check_ndim(h, 4, name="h")
        check_ndim(D, 1, name="D", optional=True)

        batch_size, num_heads, head_dim = u.shape
        num_groups, state_dim = B.shape[1], B.shape[2]

        check_shape(A, (num_heads,), name="A")
        check_shape(B, (batch_size, num_groups, state_dim), name="B")
        check_shape(C, (batch_size, num_groups, state_dim), name="C")
        check_shape(delta_raw, (batch_size, num_heads), name="delta_raw")
        check_shape(delta_bias, (num_heads,), name="delta_bias", optional=True)
        check_shape(h, (batch_size, num_heads, head_dim, state_dim), name="h")
        check_shape(D, (num_heads * head_dim,), name="D", optional=True)
        if z is not None:
            if z.ndim == 3:
                check_shape(z, (batch_size, num_heads, head_dim), name="z")
            else:
                check_ndim(z, 2, name="z")
                check_shape(z, (batch_size, num_heads * head_dim), name="z")
        if num_heads % num_groups != 0:
            raise ValueError(f"[B] num_heads={num_heads} is not a multiple of num_groups={num_groups}")

        u = to_contiguous(u)
        A = to_contiguous(A)
        B = to_contiguous(B)
        C = to_contiguous(C)
        delta_raw = to_contiguous(delta_raw)
        delta_bias = to_contiguous(delta_bias)
        h = to_contiguous(h)

        y, h = kernels.ssu_forward(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus, delta_limit,
                                   D=D, z=z)
        return y, h
