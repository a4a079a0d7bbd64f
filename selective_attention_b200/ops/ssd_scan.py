"""``SSDScanFn``: drop-in for the reference's ``ops/ssd_scan.py:7-96``.

Same positional signature (``u, A, B, C, delta_raw, delta_bias, h_init, length,
chunk_size, use_delta_softplus, delta_limit, is_causal``), same ``ValueError``
checks in the same order (``:38-56``), same contiguity handling (``:58-65``), same
outputs: ``y (b, L, H, P)`` fp32 and ``h_last (b, H, P, N)`` fp32
(``triton_kernels/ssd_scan/forward.py:120,200``).

Extensions, appended as optional trailing positional arguments so existing
callers are unchanged:
- ``D`` (``(H*P,)``) and ``z`` (``(b, L, H*P)`` or ``(b, L, H, P)``): fused epilogue
  ``y = (y + D*u) * silu(z)`` of ``modules/ssm.py:145-150``; ``y`` then has ``u``'s dtype.
- ``cu_seqlens`` (``(nseq+1,)`` int32/int64): packed variable-length rows; ``u`` etc.
  have batch 1 and ``h_last`` / ``h_init`` are ``(nseq, H, P, N)``.
- ``impl``: ``"auto"`` (tensor cores when supported), ``"tc"`` or ``"simt"``.

Backward: ``SSDScanFn.backward`` is the reference's (``ops/ssd_scan.py:83-96``):
the forward intermediates are recomputed and ``kernels.ssd_scan_backward`` returns
the gradients of ``u, A, B, C, delta_raw, delta_bias, h_init`` (``None`` for the
rest), also for packed ``cu_seqlens`` rows. The fused ``D`` / ``z`` epilogue has no
backward here (the reference applies ``D`` and ``z`` outside the op): a backward
through a call that used them raises ``NotImplementedError``.
"""
from __future__ import annotations

from typing import Tuple

import torch

from .. import kernels
from ..utils import check_ndim, check_shape, to_contiguous

INF = float("inf")


class SSDScanFn(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx,
        u: torch.Tensor,
        A: torch.Tensor,
        B: torch.Tensor,
        C: torch.Tensor,
        delta_raw: torch.Tensor,
        delta_bias: torch.Tensor | None = None,
        h_init: torch.Tensor | None = None,
        length: torch.Tensor | None = None,
        chunk_size: int = 256,
        use_delta_softplus: bool = True,
        delta_limit: Tuple[float, float] = (0.0, INF),
        is_causal: bool = True,
        D: torch.Tensor | None = None,
        z: torch.Tensor | None = None,
        cu_seqlens: torch.Tensor | None = None,
        impl: str = "auto",
    ):
        check_ndim(u, 4, name="u")
        check_ndim(A, 1, name="A")
        check_ndim(B, 4, name="B")
        check_ndim(C, 4, name="C")
        check_ndim(delta_raw, 3, name="delta_raw")
        check_ndim(delta_bias, 1, name="delta_bias", optional=True)
        check_ndim(h_init, 4, name="h_init", optional=True)
        check_ndim(length, 1, name="length", optional=True)
        check_ndim(D, 1, name="D", optional=True)
        check_ndim(cu_seqlens, 1, name="cu_seqlens", optional=True)

        batch_size, seq_len, num_heads, head_dim = u.shape
        num_groups, state_dim = B.shape[2], B.shape[3]
        nrows = batch_size if cu_seqlens is None else cu_seqlens.shape[0] - 1

        check_shape(A, (num_heads,), name="A")
        check_shape(B, (batch_size, seq_len, num_groups, state_dim), name="B")
        check_shape(C, (batch_size, seq_len, num_groups, state_dim), name="C")
        check_shape(delta_raw, (batch_size, seq_len, num_heads), name="delta_raw")
        check_shape(delta_bias, (num_heads,), name="delta_bias", optional=True)
        check_shape(h_init, (nrows, num_heads, head_dim, state_dim), name="h_init", optional=True)
        check_shape(length, (batch_size,), name="length", optional=True)
        check_shape(D, (num_heads * head_dim,), name="D", optional=True)
        if z is not None:
            if z.ndim == 4:
                check_shape(z, (batch_size, seq_len, num_heads, head_dim), name="z")
            else:
                check_ndim(z, 3, name="z")
                check_shape(z, (batch_size, seq_len, num_heads * head_dim), name="z")
        if cu_seqlens is not None:
            if batch_size != 1:
                raise ValueError("[cu_seqlens] packed mode expects batch size 1")
            if length is not None:
                raise ValueError("[length] cannot be combined with cu_seqlens")
        if num_heads % num_groups != 0:
            raise ValueError(f"[B] num_heads={num_heads} is not a multiple of num_groups={num_groups}")

        u = to_contiguous(u)
        A = to_contiguous(A)
        B = to_contiguous(B)
        C = to_contiguous(C)
        delta_raw = to_contiguous(delta_raw)
        delta_bias = to_contiguous(delta_bias)
        h_init = to_contiguous(h_init)
        length = to_contiguous(length)

        y, h_last = kernels.ssd_scan_forward(
            u, A, B, C, delta_raw, delta_bias, h_init, length, chunk_size, use_delta_softplus,
            delta_limit, is_causal, D=D, z=z, cu_seqlens=cu_seqlens, impl=impl)
        ctx.save_for_backward(u, A, B, C, delta_raw, delta_bias, h_init, length, cu_seqlens)
        ctx.chunk_size = chunk_size
        ctx.use_delta_softplus = use_delta_softplus
        ctx.delta_limit = delta_limit
        ctx.is_causal = is_causal
        ctx.fused_epilogue = D is not None or z is not None
        return y, h_last

    @staticmethod
    def backward(ctx, y_grad, h_last_grad):
        if ctx.fused_epilogue:
            raise NotImplementedError(
                "SSDScanFn.backward: the fused D / z epilogue has no backward; apply D and z outside the op "
                "(as modules/ssm.py:144-150 does) to train through it")
        u, A, B, C, delta_raw, delta_bias, h_init, length, cu_seqlens = ctx.saved_tensors
        grads = kernels.ssd_scan_backward(
            u, A, B, C, delta_raw, delta_bias, h_init, y_grad, h_last_grad, length, ctx.chunk_size,
            ctx.use_delta_softplus, ctx.delta_limit, ctx.is_causal, cu_seqlens=cu_seqlens)
        return (*grads, None, None, None, None, None, None, None, None, None)
