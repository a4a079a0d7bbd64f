"""Training-mode selective attention as an autograd op.

The reference computes this part of ``SelectiveMHA.forward`` (``modules/selective_attention.py``
``:232-280`` with ``self.training``) as torch matmuls, a masked score-statistics pass and a
softmax, and differentiates it with autograd. ``SelectiveAttnTrainFn`` runs the same maths
through ``kernels.sattn_train_forward`` / ``sattn_train_backward`` (C-ABI ``sattn_train_fwd`` /
``sattn_train_bwd``), including the gradient that flows through the per-head score std into
the queries and keys.
"""
from __future__ import annotations

import torch

from .. import kernels


class SelectiveAttnTrainFn(torch.autograd.Function):
    """``(q_rot, k_rot, v, select_gate, lengths, log_gate_penalty, is_causal, scale, impl) -> (out, std)``.

    ``out`` ``(b, H, L, D)`` is ``attn_weight @ v`` (``:278``); ``std`` ``(H,)`` is the layer's
    ``head_attention_score_std`` (``:251``), returned detached for the ``score_std_ema`` update
    (``:252-256``, under ``no_grad`` in the reference). Gradients: q_rot, k_rot, v, select_gate.
    """

    @staticmethod
    def forward(ctx, q_rot, k_rot, v, select_gate, lengths=None, log_gate_penalty=1.0, is_causal=True, scale=None,
                impl="auto"):
        out, lse, lg, stats = kernels.sattn_train_forward(q_rot, k_rot, v, select_gate, log_gate_penalty, lengths,
                                                          is_causal, scale, impl)
        ctx.save_for_backward(q_rot, k_rot, v, select_gate, out, lse, lg, stats,
                              lengths if lengths is not None else torch.empty(0))
        ctx.has_lengths = lengths is not None
        ctx.penalty, ctx.is_causal, ctx.scale, ctx.impl = log_gate_penalty, is_causal, scale, impl
        std = stats[:, 1].clone()
        ctx.mark_non_differentiable(std)
        return out, std

    @staticmethod
    def backward(ctx, dout, dstd_unused):
        q_rot, k_rot, v, select_gate, out, lse, lg, stats, lengths = ctx.saved_tensors
        if dout is None:
            return (None,) * 9
        dq, dk, dv, dg = kernels.sattn_train_backward(
            q_rot, k_rot, v, select_gate, out, lse, lg, stats.clone(), dout, ctx.penalty,
            lengths if ctx.has_lengths else None, ctx.is_causal, ctx.scale, ctx.impl)
        return (dq.to(q_rot.dtype), dk.to(k_rot.dtype), dv.to(v.dtype), dg.to(select_gate.dtype),
                None, None, None, None, None)


def selective_attn_train(q_rot, k_rot, v, select_gate, lengths=None, log_gate_penalty=1.0, is_causal=True,
                         scale=None, impl="auto"):
    """``SelectiveAttnTrainFn.apply`` with keyword defaults; returns ``(out, std)``. ``impl``:
    ``"auto"`` (tcgen05 for 16-bit inputs with head_dim 64), ``"tc"`` or ``"simt"``."""
    return SelectiveAttnTrainFn.apply(q_rot, k_rot, v, select_gate, lengths, log_gate_penalty, is_causal, scale,
                                      impl)
