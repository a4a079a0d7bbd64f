"""CPU restatement of selective attention: decode step, inference prefill and the
training-mode forward (TEST INFRASTRUCTURE ONLY).

Parity checker for the CUDA kernels (``csrc/sattn.cu``, ``csrc/sattn_train.cu``). Imported
only by ``tests/`` and ``bench.py``'s CPU legs; the product never imports it.

Follows nmquan1503/selective-attention (paths relative to ``src/selective_attention/``):
- ``inference/selective_attn_cache.py:27-42`` ``SelectiveAttnCache.update_kv``: the new
  key, value and log-gate are written at ``write_idx``, which then advances;
- ``modules/selective_attention.py:390-404`` (``SelectiveMHA.step``): scores of the
  query against the first ``write_idx`` cached keys, times ``scale``; the pos-mode gated
  softmax (``:121-123``) adds every cached key's log-gate except the newest one's
  (the token itself); the output is the weighted sum of the cached values.

Parity pin: golden vectors made with the reference's own cache class, ``_reset_cache``
and ``_gated_softmax`` (``tests/golden/make_golden_sattn.py``).
"""
from __future__ import annotations

import torch


def update_kv(k_cache, v_cache, lg_cache, write_idx, k_rot, v, log_gate):
    """``selective_attn_cache.py:39-42``: in-place write at ``write_idx``; returns the new index."""
    k_cache[:, :, write_idx, :] = k_rot
    v_cache[:, :, write_idx, :] = v
    lg_cache[:, :, write_idx] = log_gate
    return write_idx + 1


def gated_softmax_pos(attn, log_gate):
    """``modules/selective_attention.py:121-123``: gate every key but the last, then softmax."""
    attn = attn.clone()
    attn[..., :-1] += log_gate[..., :-1]
    return torch.softmax(attn, dim=-1)


def decode_attention(q_rot, k_cache, v_cache, lg_cache, n_keys, scale, dtype=torch.float32):
    """``modules/selective_attention.py:398-405`` over the first ``n_keys`` cache slots.

    ``q_rot`` ``(b, H, D)``; caches ``(b, H, cap, D)`` / ``(b, H, cap)``. Returns ``(b, H, D)``.
    """
    k = k_cache[:, :, :n_keys, :].to(dtype)
    v = v_cache[:, :, :n_keys, :].to(dtype)
    lg = lg_cache[:, :, :n_keys].to(dtype)
    attn = (q_rot.to(dtype).unsqueeze(2) @ k.transpose(-2, -1)).squeeze(2) * scale
    w = gated_softmax_pos(attn, lg)
    return (w.unsqueeze(2) @ v).squeeze(2)


def decode_step(q_rot, k_rot, v, log_gate, k_cache, v_cache, lg_cache, write_idx, scale, dtype=torch.float32):
    """One decode step's cache update plus attention, as ``SelectiveMHA.step`` runs them
    (``:390``, ``:399-404``). Updates the caches in place; returns ``(out, new write_idx)``."""
    n = update_kv(k_cache, v_cache, lg_cache, write_idx, k_rot, v, log_gate)
    return decode_attention(q_rot, k_cache, v_cache, lg_cache, n, scale, dtype), n


def prefill_attention(q_rot, k_rot, v, log_gate, scale, dtype=torch.float32):
    """Inference prefill without compression, ``modules/selective_attention.py:27-144``:
    ``_build_attn_matrix`` (``q k^T * scale``, causal ``-inf`` above the diagonal, ``:55-64``),
    the seq-mode ``_gated_softmax`` (log-gate of each key added off the diagonal, ``:134-137``)
    and ``attn_weight @ v`` (``:280``). Keys with log-gate ``-inf`` drop out, which is also
    what the compressed path (``:66-88``, ``:270-278``) computes. Shapes ``(b, H, L, D)``."""
    L = q_rot.shape[2]
    attn = (q_rot.to(dtype) @ k_rot.to(dtype).transpose(-2, -1)) * scale
    attn = attn.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), diagonal=1), float("-inf"))
    diag = torch.arange(L)
    d = attn[:, :, diag, diag].clone()
    attn = attn + log_gate.to(dtype).unsqueeze(2)
    attn[:, :, diag, diag] = d
    return torch.softmax(attn, dim=-1) @ v.to(dtype)


def train_attention(q_rot, k_rot, v, select_gate, log_gate_penalty, lengths=None, is_causal=True, scale=None,
                    dtype=torch.float32):
    """``SelectiveMHA.forward`` with ``self.training`` from the score matrix to ``attn_weight @ v``
    (``modules/selective_attention.py:232-280``), differentiable with torch autograd (the
    reference's backward is autograd over these same lines). Shapes: ``q_rot, k_rot, v``
    ``(b, H, L, D)``, ``select_gate`` ``(b, H, L)``, ``lengths`` ``(b,)`` or ``None``.
    Returns ``(out, std)``.
    """
    b, H, L, D = q_rot.shape
    scale = D ** -0.5 if scale is None else scale
    q, k, vv = (t.to(dtype) for t in (q_rot, k_rot, v))
    attn = (q @ k.transpose(-2, -1)) * scale                                        # :89-90
    if is_causal:                                                                    # :92-98
        attn = attn.masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), diagonal=1), float("-inf"))
    valid = attn != float("-inf")                                                    # :235
    pad = None
    if lengths is not None:
        pad = torch.arange(L).unsqueeze(0) >= lengths.to(torch.long).unsqueeze(1)    # :208
        valid = valid & ~pad[:, None, :, None] & ~pad[:, None, None, :]              # :236-237
    count = valid.sum(dim=(0, 2, 3)).to(dtype)                                       # :238
    vs = attn.masked_fill(~valid, 0.0)
    mean = vs.sum(dim=(0, 2, 3)) / count.clamp(min=1)                                # :242-246
    var = vs.square().sum(dim=(0, 2, 3)) / count.clamp(min=1) - mean.square()       # :247-250
    std = var.clamp(min=0).sqrt()                                                    # :251
    lg = torch.log(select_gate.to(dtype)) * (std[None, :, None] * log_gate_penalty)  # :259-263
    if pad is not None:
        lg = lg.masked_fill(pad.unsqueeze(1), float("-inf"))                         # :265-269
    diag = torch.arange(L)                                                           # :134-142 (training)
    d = attn[:, :, diag, diag]
    attn = attn + lg.unsqueeze(2)
    attn[:, :, diag, diag] = d
    return torch.softmax(attn, dim=-1) @ vv, std                                     # :144, :278
