"""CPU restatement of the SSM layer's prefill front end (TEST INFRASTRUCTURE ONLY).

Parity checker for ``ssm_conv_prefill``. Imported only by ``tests/`` and ``bench.py``'s
CPU legs; the product path never imports it.

Restates nmquan1503/selective-attention ``src/selective_attention/modules/ssm.py:112-134``
(transpose, optional conv-context capture, SiLU, depthwise ``nn.Conv1d`` with padding
K - 1 truncated to the sequence, transpose back, split into x, B, C) and
``inference/ssm_cache.py:10-36`` (``SSMCache.build_conv_ctx``).

Parity pin: checked against golden vectors made by the reference's own ``SSM.conv``
layer and ``SSMCache.build_conv_ctx`` (``tests/golden/make_golden_front.py``).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def build_conv_ctx(x: torch.Tensor, lengths: Optional[torch.Tensor], cache_size: int) -> torch.Tensor:
    """x (b, dim, L) -> (b, dim, cache_size): the last cache_size inputs before each row's
    length, zeros where the row is shorter (inference/ssm_cache.py:10-36)."""
    b, dim, L = x.shape
    n = torch.full((b,), L, dtype=torch.int64) if lengths is None else lengths.to(torch.int64).cpu()
    out = torch.zeros(b, dim, cache_size, dtype=x.dtype)
    for r in range(b):
        for k in range(cache_size):
            t = int(n[r]) - cache_size + k
            if 0 <= t < int(n[r]) and t < L:
                out[r, :, k] = x[r, :, t]
    return out


def prefill_front(hBC: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], inner: int, gn: int,
                  lengths: Optional[torch.Tensor] = None, act_dtype: Optional[torch.dtype] = None):
    """hBC (b, L, inner + 2 gn) -> x (b, L, inner), B, C (b, L, gn), conv_ctx (b, conv_dim, K),
    computed in fp32. ``act_dtype``: round the SiLU output to this dtype first, as
    ``F.silu`` on a tensor of that dtype does (modules/ssm.py:125)."""
    b, L, conv_dim = hBC.shape
    w = weight.reshape(conv_dim, -1).float()
    K = w.shape[1]
    x_t = hBC.transpose(1, 2)                                    # ssm.py:119
    ctx = build_conv_ctx(x_t, lengths, K)                        # ssm.py:121-123
    s = F.silu(x_t.float())                                      # ssm.py:125
    if act_dtype is not None:
        s = s.to(act_dtype).float()
    out = F.conv1d(s, w[:, None, :], None if bias is None else bias.float(), padding=K - 1,
                   groups=conv_dim)                              # ssm.py:126 (nn.Conv1d, groups=conv_dim)
    out = out[:, :, :L].transpose(1, 2)                          # ssm.py:126-127
    x, B, C = torch.split(out, [inner, gn, gn], dim=-1)          # ssm.py:129-134
    return x, B, C, ctx


def update_conv_ctx(ctx: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """SSMCache.update (inference/ssm_cache.py:38-43): shift left by one, append x."""
    out = torch.roll(ctx, shifts=-1, dims=-1)
    out[:, :, -1] = x
    return out


def decode_front(hBC: torch.Tensor, ctx: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], inner: int,
                 gn: int):
    """One decode step's front end (modules/ssm.py:173-186) with torch ops on tensors of
    hBC's dtype, as the reference runs them: the cache update, silu of the whole window,
    the product with the conv weight, the sum over the window and the bias add, then the
    split. Returns x (b, inner), B, C (b, gn) and the updated cache."""
    dt = hBC.dtype
    new_ctx = update_conv_ctx(ctx, hBC)                               # ssm.py:173-174
    s = F.silu(new_ctx)                                               # :175
    w = weight.reshape(weight.shape[0], -1).to(dt)
    out = (s * w).sum(dim=-1)                                         # :176
    if bias is not None:
        out = out + bias.to(dt)
    x, B, C = torch.split(out, [inner, gn, gn], dim=-1)              # :177-184
    return x, B, C, new_ctx
