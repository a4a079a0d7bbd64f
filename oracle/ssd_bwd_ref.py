"""CPU restatement of the reference SSD backward (TEST INFRASTRUCTURE ONLY).

Parity checker for the CUDA backward. Imported only by ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs; the product path never
imports it.

Follows ``triton_kernels/ssd_scan/backward.py:467-555`` (``ssd_scan_backward``)
stage by stage, each function citing the kernel it restates in
``triton_kernels/ssd_scan/backward_kernel.py`` (paths relative to
``src/selective_attention/`` of nmquan1503/selective-attention). The reference's
own choices are kept, including the ones that are not the exact derivative of
its forward:
- every stage masks token rows at ``length`` (``chunk_size_limit``), so ``y_grad``
  past ``length`` is ignored although the forward writes ``y`` there;
- the ``min(., 0)`` clamps of the decays get no derivative;
- clamped ``dt`` gets zero gradient, softplus gets ``sigmoid`` below 20.

Parity pin: golden vectors from the reference's own backward kernels run under
the Triton interpreter (``tests/golden/make_golden_bwd.py``), and torch autograd
through the forward restatement where the two agree (full-length rows).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .ssd_ref import INF, bmm_chunk, chunk_cumsum, chunk_state, state_passing


def _pad_rows(t: torch.Tensor, nc: int, cs: int, dtype) -> torch.Tensor:
    """``(b, L, ...)`` -> ``(b, nc, cs, ...)`` zero-padded to whole chunks."""
    b, L = t.shape[:2]
    out = torch.zeros((b, nc * cs) + tuple(t.shape[2:]), dtype=dtype)
    out[:, :L] = t.to(dtype)
    return out.view((b, nc, cs) + tuple(t.shape[2:]))


def _valid(length: torch.Tensor, L: int, nc: int, cs: int) -> torch.Tensor:
    """``(b, nc, cs)`` mask of the rows every backward kernel keeps (``t < length``)."""
    t = torch.arange(nc * cs)
    return (t[None, :] < torch.clamp(length.to(torch.long), max=L)[:, None]).view(-1, nc, cs)


def chunk_scan_backward_h(C, cum, y_grad, length, dtype=torch.float32):
    """``backward_kernel.py:23-93``: the intra-chunk state gradient.

    ``h_grad[b,c,h,p,n] = sum_{l<lim} y_grad[l,p] * exp(cum_l) * C[l,n]``. Returns
    ``(b, nc, H, P, N)``.
    """
    b, L, H, P = y_grad.shape
    G, N = C.shape[2], C.shape[3]
    nc, cs = cum.shape[2], cum.shape[3]
    hpg = H // G
    v = _valid(length, L, nc, cs)
    yg = _pad_rows(y_grad, nc, cs, dtype) * v[..., None, None]
    Ch = _pad_rows(C, nc, cs, dtype).repeat_interleave(hpg, dim=3)
    e = torch.exp(cum.to(dtype)).permute(0, 2, 3, 1)  # (b,nc,cs,H)
    return torch.einsum("bclhp,bclhn->bchpn", yg * e[..., None], Ch)


def state_passing_backward(prev, decay_last, h_grad, h_last_grad, has_h_init, dtype=torch.float32):
    """``backward_kernel.py:96-161``: reverse recurrence over chunks.

    With ``g`` the gradient of the state leaving chunk ``c`` (``h_last_grad`` for the
    last chunk): ``decay_last_grad[c] = sum(prev[c] * g) * exp(decay_last[c])``;
    ``h_grad[c] <- g``; ``g = exp(decay_last[c]) * g + h_grad_intra[c]``. ``g`` after
    chunk 0 is ``h_init_grad``; without ``h_init`` ``decay_last_grad[:, :, 0] = 0``.
    Returns ``(h_grad, decay_last_grad (b,H,nc), h_init_grad or None)``.
    """
    b, nc, H = prev.shape[:3]
    g = torch.zeros_like(prev[:, 0], dtype=dtype) if h_last_grad is None else h_last_grad.to(dtype).clone()
    out = torch.empty_like(prev, dtype=dtype)
    dlast = torch.zeros(b, H, nc, dtype=dtype)
    for c in range(nc - 1, -1, -1):
        scale = torch.exp(decay_last[:, :, c].to(dtype))
        dlast[:, :, c] = (prev[:, c].to(dtype) * g).sum((-2, -1)) * scale
        out[:, c] = g
        g = scale[..., None, None] * g + h_grad[:, c].to(dtype)
    if not has_h_init:
        dlast[:, :, 0] = 0.0
    return out, dlast, (g if has_h_init else None)


def chunk_grads(u, B, C, dt, cum, CB, prev, h_grad, y_grad, length, dtype=torch.float32):
    """The per-chunk kernels of ``backward.py:531-545`` in one place.

    - ``u_grad``, ``delta_grad`` (``backward_kernel.py:186-314``):
      ``acc[l,p] = exp(min(cum_last - cum_l, 0)) * sum_n B[l,n] h_grad[p,n]
      + sum_{l<=s<lim} CB[s,l] exp(min(cum_s - cum_l, 0)) y_grad[s,p]``;
      ``u_grad = acc * dt_l``; ``delta_grad[l] = sum_p acc[l,p] u[l,p]``.
    - ``B_grad`` and the B-side decay gradient (``:317-441``):
      ``contrib[l,n] = exp(min(cum_last - cum_l, 0)) dt_l sum_p u[l,p] h_grad[p,n]``,
      summed over the group's heads; ``sum_n contrib * B`` lands one row later and is
      cumulated (``backward.py:215-216``).
    - ``C_grad`` and the C-side decay gradient (``:444-555``):
      ``exp(cum_l) sum_p y_grad[l,p] prev[p,n]``.
    - ``CB_grad`` (``:558-683``): ``sum_h sum_p y_grad[l,p] u[s,p] dt_s
      exp(min(cum_l - cum_s, 0))`` for ``s <= l < lim``; then ``bmm_chunk_backward``
      (``:686-780``) adds ``CB_grad^T C`` to ``B_grad`` and ``CB_grad B`` to ``C_grad``.
    - the intra-chunk decay gradient (``:783-895``): with
      ``w[l,s] = (y_grad[l] . u[s]) dt_s CB[l,s] exp(min(cum_l - cum_s, 0))`` for
      ``s < l``, ``decay[j] = sum_{l>=j} sum_{s<j} w[l,s]``.

    Returns ``u_grad (b,L,H,P)``, ``delta_grad (b,H,nc,cs)``, ``B_grad``, ``C_grad``
    (``(b,L,G,N)``), ``decay_from_B``, ``decay_from_C``, ``decay_intra`` (each
    ``(b,H,nc,cs)``), ``CB_grad (b,nc,G,cs,cs)``.
    """
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    nc, cs = cum.shape[2], cum.shape[3]
    hpg = H // G
    v = _valid(length, L, nc, cs)  # (b,nc,cs)
    vf = v.to(dtype)
    up = _pad_rows(u, nc, cs, dtype) * vf[..., None, None]       # (b,nc,cs,H,P)
    yg = _pad_rows(y_grad, nc, cs, dtype) * vf[..., None, None]
    Bp = _pad_rows(B, nc, cs, dtype) * vf[..., None, None]       # (b,nc,cs,G,N)
    Cp = _pad_rows(C, nc, cs, dtype) * vf[..., None, None]
    Bh = Bp.repeat_interleave(hpg, dim=3)
    Ch = Cp.repeat_interleave(hpg, dim=3)
    cumr = torch.where(v[:, None], cum.to(dtype), torch.zeros((), dtype=dtype)).permute(0, 2, 1, 3)  # (b,nc,H,cs)
    dtr = torch.where(v[:, None], dt.to(dtype), torch.zeros((), dtype=dtype)).permute(0, 2, 1, 3)
    clast = cum.to(dtype).permute(0, 2, 1, 3)[..., -1:]  # unmasked element cs-1
    scale = torch.exp(torch.clamp(clast - cumr, max=0.0))  # (b,nc,H,cs)
    hg = h_grad.to(dtype)
    pv = prev.to(dtype)
    CBh = CB.to(dtype).repeat_interleave(hpg, dim=2)  # (b,nc,H,cs,cs)
    vv = v[:, :, None, :, None] & v[:, :, None, None, :]  # (b,nc,1,l,s)
    seg = torch.exp(torch.clamp(cumr[..., :, None] - cumr[..., None, :], max=0.0))  # [l,s]

    # u_grad / delta_grad
    accS = torch.einsum("bclhn,bchpn->bchlp", Bh, hg) * scale[..., None]
    upper = torch.triu(torch.ones(cs, cs, dtype=torch.bool))  # s >= l  as [l,s]
    My = torch.where(upper & vv, CBh.transpose(-1, -2) * seg.transpose(-1, -2), torch.zeros((), dtype=dtype))
    accY = torch.einsum("bchls,bcshp->bchlp", My, yg)
    acc = accS + accY                                             # (b,nc,H,cs,P)
    ug = acc * dtr[..., None]
    u_grad = (ug.permute(0, 1, 3, 2, 4) * vf[..., None, None]).reshape(b, nc * cs, H, P)[:, :L]
    delta_grad = (acc * up.permute(0, 1, 3, 2, 4)).sum(-1)       # (b,nc,H,cs)

    # B side
    contribB = torch.einsum("bclhp,bchpn->bchln", up, hg) * (scale * dtr)[..., None]
    B_grad = contribB.view(b, nc, G, hpg, cs, N).sum(3).permute(0, 1, 3, 2, 4)  # (b,nc,cs,G,N)
    gB = (contribB * Bh.permute(0, 1, 3, 2, 4)).sum(-1)          # (b,nc,H,cs)
    lim = v.sum(-1)                                               # (b,nc)
    li = torch.arange(cs)
    keep = li[None, None, :] < (lim[..., None] - 1)               # l < lim - 1
    shifted = torch.zeros_like(gB)
    shifted[..., 1:] = torch.where(keep[:, :, None, :-1], gB[..., :-1], torch.zeros((), dtype=dtype))
    decay_from_B = torch.cumsum(shifted, dim=-1)

    # C side
    contribC = torch.einsum("bclhp,bchpn->bchln", yg, pv) * torch.exp(cumr)[..., None] * vf[:, :, None, :, None]
    C_grad = contribC.view(b, nc, G, hpg, cs, N).sum(3).permute(0, 1, 3, 2, 4)
    decay_from_C = (contribC * Ch.permute(0, 1, 3, 2, 4)).sum(-1)

    # CB_grad and bmm backward
    lower = torch.tril(torch.ones(cs, cs, dtype=torch.bool))     # s <= l as [l,s]
    Gm = torch.einsum("bclhp,bcshp->bchls", yg, up)
    CBg_h = torch.where(lower & vv, Gm * dtr[..., None, :] * seg, torch.zeros((), dtype=dtype))
    CB_grad = CBg_h.view(b, nc, G, hpg, cs, cs).sum(3)           # (b,nc,G,cs,cs)
    B_grad = B_grad + torch.einsum("bcgls,bclgn->bcsgn", CB_grad, Cp)
    C_grad = C_grad + torch.einsum("bcgls,bcsgn->bclgn", CB_grad, Bp)

    # intra-chunk decay gradient
    strict = torch.tril(torch.ones(cs, cs, dtype=torch.bool), diagonal=-1)
    w = torch.where(strict & vv, CBg_h * CBh, torch.zeros((), dtype=dtype))
    R = torch.cumsum(w, dim=-1)                                   # R[l, j-1] = sum_{s<j} w[l,s]
    ge = (li[:, None] >= li[None, :])                              # [l, j]: l >= j
    decay_intra = torch.zeros_like(delta_grad)
    decay_intra[..., 1:] = (R[..., :, :-1] * ge[:, 1:]).sum(-2)

    B_grad = B_grad.reshape(b, nc * cs, G, N)[:, :L]
    C_grad = C_grad.reshape(b, nc * cs, G, N)[:, :L]
    perm = lambda t: t.permute(0, 2, 1, 3)  # (b,nc,H,cs) -> (b,H,nc,cs)  # noqa: E731
    return (u_grad, perm(delta_grad), B_grad, C_grad, perm(decay_from_B), perm(decay_from_C),
            perm(decay_intra), CB_grad)


def chunk_cumsum_backward(A, delta_raw, delta_bias, delta_grad, decay_grad_total, length, chunk_size,
                          use_softplus=True, delta_limit=(0.0, INF), dtype=torch.float32):
    """``backward_kernel.py:898-1039``.

    ``g = decay_total * A + delta_grad``, zero where ``dt`` was clamped, times
    ``sigmoid(pre)`` where softplus applied (``pre <= 20``); ``A_grad = sum
    decay_total * dt``; ``delta_bias_grad = sum g``. Rows past ``length`` are zero.
    Returns ``(A_grad, delta_raw_grad (b,L,H), delta_bias_grad or None)``.
    """
    b, L, H = delta_raw.shape
    nc, cs = delta_grad.shape[2], delta_grad.shape[3]
    v = _valid(length, L, nc, cs).reshape(b, nc * cs)[:, :L]
    to_rows = lambda t: t.to(dtype).permute(0, 2, 3, 1).reshape(b, nc * cs, H)[:, :L]  # noqa: E731
    dg = to_rows(delta_grad)
    tot = to_rows(decay_grad_total)
    pre = delta_raw.to(dtype)
    if delta_bias is not None:
        pre = pre + delta_bias.to(dtype)[None, None, :]
    d = torch.where(pre <= 20.0, torch.log(torch.exp(pre) + 1.0), pre) if use_softplus else pre
    clamped = (d < delta_limit[0]) | (d > delta_limit[1])
    d = torch.clamp(torch.clamp(d, min=delta_limit[0]), max=delta_limit[1])
    g = tot * A.to(dtype)[None, None, :] + dg
    g = torch.where(clamped, torch.zeros((), dtype=dtype), g)
    if use_softplus:
        g = torch.where(pre <= 20.0, g * torch.sigmoid(pre), g)
    zero = torch.zeros((), dtype=dtype)
    g = torch.where(v[..., None], g, zero)
    A_grad = torch.where(v[..., None], tot * d, zero).sum((0, 1))
    bias_grad = g.sum((0, 1)) if delta_bias is not None else None
    return A_grad, g, bias_grad


def ssd_scan_backward(u, A, B, C, delta_raw, delta_bias, h_init, y_grad, h_last_grad, length=None,
                      chunk_size=256, use_delta_softplus=True, delta_limit: Tuple[float, float] = (0.0, INF),
                      dtype=torch.float32):
    """``backward.py:467-555``: recompute the forward intermediates, then the stages.

    Returns ``(u_grad, A_grad, B_grad, C_grad, delta_raw_grad, delta_bias_grad,
    h_init_grad)`` in ``dtype`` (``delta_bias_grad`` / ``h_init_grad`` None when the
    input was None).
    """
    b, L, H, P = u.shape
    if length is None:
        length = torch.full((b,), L, dtype=torch.long)
    cum, dt = chunk_cumsum(A, delta_raw, delta_bias, length, chunk_size, use_delta_softplus,
                           delta_limit, dtype=dtype)
    S = chunk_state(u, B, dt, cum, dtype=dtype)
    prev, _ = state_passing(S, h_init, cum[..., -1], dtype=dtype)
    CB = bmm_chunk(B, C, chunk_size, dtype=dtype)
    hgi = chunk_scan_backward_h(C, cum, y_grad, length, dtype=dtype)
    hg, dlast, h_init_grad = state_passing_backward(prev, cum[..., -1], hgi, h_last_grad, h_init is not None,
                                                    dtype=dtype)
    (u_grad, delta_grad, B_grad, C_grad, dB, dC, dI, _) = chunk_grads(
        u, B, C, dt, cum, CB, prev, hg, y_grad, length, dtype=dtype)
    dC = dC.clone()
    dC[..., -1] += dlast
    dC_rev = dC.flip([-1]).cumsum(-1).flip([-1])
    total = dI + dB + dC_rev
    A_grad, draw, dbias = chunk_cumsum_backward(A, delta_raw, delta_bias, delta_grad, total, length,
                                                chunk_size, use_delta_softplus, delta_limit, dtype=dtype)
    return u_grad, A_grad, B_grad, C_grad, draw, dbias, h_init_grad


def ssd_scan_backward_varlen(u, A, B, C, delta_raw, delta_bias, cu_seqlens, y_grad, h_last_grad=None,
                             chunk_size=256, use_delta_softplus=True, delta_limit=(0.0, INF),
                             dtype=torch.float32, h_init=None):
    """Packed rows as the padded reference computes them: unpack, run, gather back."""
    from .ssd_ref import padded_to_varlen, varlen_to_padded
    up, lens = varlen_to_padded(u, cu_seqlens)
    Bp, _ = varlen_to_padded(B, cu_seqlens)
    Cp, _ = varlen_to_padded(C, cu_seqlens)
    dp, _ = varlen_to_padded(delta_raw, cu_seqlens)
    yp, _ = varlen_to_padded(y_grad, cu_seqlens)
    ug, Ag, Bg, Cg, dg, bg, hg = ssd_scan_backward(up, A, Bp, Cp, dp, delta_bias, h_init, yp, h_last_grad,
                                                   lens, chunk_size, use_delta_softplus, delta_limit, dtype)
    return (padded_to_varlen(ug, cu_seqlens), Ag, padded_to_varlen(Bg, cu_seqlens),
            padded_to_varlen(Cg, cu_seqlens), padded_to_varlen(dg, cu_seqlens), bg, hg)
