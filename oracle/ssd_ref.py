"""CPU restatement of the reference SSD forward and SSU decode (TEST INFRASTRUCTURE ONLY).

This module is the parity checker for the CUDA path. It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py``. The product path (``selective_attention_b200``)
never imports it and fails loudly when its CUDA library is missing.

Each function follows one stage of the reference's Triton implementation
(nmquan1503/selective-attention, paths relative to ``src/selective_attention/``)
and cites the lines it restates. The maths is written with torch CPU tensor ops
in a chosen compute dtype (fp32 to match the reference's own arithmetic, fp64 for
an exact-ish yardstick).

Parity pin: the restatement is checked against golden vectors produced by the
reference's own kernels run under the Triton interpreter
(``tests/golden/make_golden.py``) and against the fp64 sequential recurrence
``ssd_recurrence`` below.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

INF = float("inf")


def _dt_transform(d: torch.Tensor, use_softplus: bool, delta_limit: Tuple[float, float]) -> torch.Tensor:
    """softplus-with-threshold then clamp.

    ``triton_kernels/softplus.py:8`` (``log(exp(x)+1)``), applied only where
    ``x <= 20`` (``ssd_scan/forward_kernel.py:76-77``, ``ssu/forward_kernel.py:128-129``),
    then ``min(max(d, lo), hi)`` (``forward_kernel.py:79``).
    """
    if use_softplus:
        d = torch.where(d <= 20.0, torch.log(torch.exp(d) + 1.0), d)
    return torch.clamp(torch.clamp(d, min=delta_limit[0]), max=delta_limit[1])


def chunk_cumsum(A, delta_raw, delta_bias, length, chunk_size, use_softplus=True,
                 delta_limit=(0.0, INF), dtype=torch.float32):
    """``ssd_scan/forward.py:14-56`` + kernel ``forward_kernel.py:19-87``.

    Returns ``(decay_cumsum, delta)``, both ``(b, H, nc, cs)``. ``delta`` is zero
    for tokens at or past ``length[b]`` (``:62-65,80``) and for the padded tail of
    the last chunk; ``decay_cumsum = cumsum(delta * A)`` within each chunk (``:83-84``).
    """
    b, L, H = delta_raw.shape
    cs = chunk_size
    nc = math.ceil(L / cs)
    d = delta_raw.to(dtype)
    if delta_bias is not None:
        d = d + delta_bias.to(dtype)[None, None, :]
    d = _dt_transform(d, use_softplus, delta_limit)
    t = torch.arange(nc * cs)
    valid = t[None, :] < torch.clamp(length.to(torch.long), max=L)[:, None]  # (b, nc*cs)
    dpad = torch.zeros(b, nc * cs, H, dtype=dtype)
    dpad[:, :L] = d
    dpad = torch.where(valid[:, :, None], dpad, torch.zeros((), dtype=dtype))
    delta = dpad.view(b, nc, cs, H).permute(0, 3, 1, 2).contiguous()  # (b,H,nc,cs)
    decay = delta * A.to(dtype)[None, :, None, None]
    cum = torch.cumsum(decay, dim=-1)
    return cum, delta


def chunk_state(u, B, delta, decay_cumsum, dtype=torch.float32):
    """``ssd_scan/forward.py:62-96`` + kernel ``forward_kernel.py:107-185``.

    ``S[b,c,h,p,n] = sum_{l<lim} u[l,p] * B[l,g(h),n] * exp(min(cum_last - cum_l, 0)) * dt_l``
    with ``cum_last`` the chunk's element ``cs-1`` (``:155``) and ``lim`` bounded by
    ``seq_len`` (``:135``). Returns ``(b, nc, H, P, N)``.
    """
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    _, _, nc, cs = delta.shape
    hpg = H // G
    up = torch.zeros(b, nc * cs, H, P, dtype=dtype)
    up[:, :L] = u.to(dtype)
    Bp = torch.zeros(b, nc * cs, G, N, dtype=dtype)
    Bp[:, :L] = B.to(dtype)
    up = up.view(b, nc, cs, H, P)
    Bh = Bp.view(b, nc, cs, G, N).repeat_interleave(hpg, dim=3)  # (b,nc,cs,H,N)
    cum_last = decay_cumsum[..., -1:]
    w = torch.exp(torch.clamp(cum_last - decay_cumsum, max=0.0)) * delta  # (b,H,nc,cs)
    w = w.permute(0, 2, 3, 1)  # (b,nc,cs,H)
    return torch.einsum("bclhp,bclhn->bchpn", up, Bh * w[..., None])


def state_passing(states, h_init, decay_last, dtype=torch.float32):
    """``ssd_scan/forward.py:102-133`` + kernel ``forward_kernel.py:202-250``.

    ``prev = h_init or 0``; for each chunk ``c``: ``out[c] = prev``;
    ``prev = exp(decay_last[c]) * prev + S[c]`` (``:244-249``); ``h_last = prev`` (``:250``).
    ``states``: ``(b, nc, H, ...)``; ``decay_last``: ``(b, H, nc)``. Returns
    ``(prev_states, h_last)``.
    """
    b, nc, H = states.shape[:3]
    rest = states.shape[3:]
    prev = torch.zeros((b, H) + rest, dtype=dtype) if h_init is None else h_init.to(dtype).clone()
    out = torch.empty_like(states, dtype=dtype)
    extra = (None,) * len(rest)
    for c in range(nc):
        out[:, c] = prev
        scale = torch.exp(decay_last[:, :, c].to(dtype))[(...,) + extra]
        prev = scale * prev + states[:, c].to(dtype)
    return out, prev


def bmm_chunk(B, C, chunk_size, dtype=torch.float32):
    """``ssd_scan/forward.py:139-169`` + kernel ``forward_kernel.py:270-328``.

    ``CB[b,c,g,l,s] = sum_n C[l,n] * B[s,n]`` with rows/columns past ``seq_len``
    masked to zero (``:320,324``). Returns the full ``(b, nc, G, cs, cs)`` block; the
    reference leaves whole tiles above the diagonal unwritten when causal
    (``:298-300``), so only the lower triangle is comparable.
    """
    b, L, G, N = B.shape
    cs = chunk_size
    nc = math.ceil(L / cs)
    Bp = torch.zeros(b, nc * cs, G, N, dtype=dtype)
    Bp[:, :L] = B.to(dtype)
    Cp = torch.zeros(b, nc * cs, G, N, dtype=dtype)
    Cp[:, :L] = C.to(dtype)
    Bp = Bp.view(b, nc, cs, G, N)
    Cp = Cp.view(b, nc, cs, G, N)
    return torch.einsum("bclgn,bcsgn->bcgls", Cp, Bp)


def chunk_scan(u, delta, decay_cumsum, C, prev_states, CB, dtype=torch.float32):
    """``ssd_scan/forward.py:175-217`` + kernel ``forward_kernel.py:350-455``.

    ``y[l,p] = exp(cum_l) * sum_n C[l,n] * prev[p,n]`` (``:411-419``, unclamped exp)
    ``+ sum_{s<=l} CB[l,s] * exp(min(cum_l - cum_s, 0)) * dt_s * u[s,p]`` (``:428-453``,
    causal hardcoded at ``forward.py:213``). Rows past ``seq_len`` are not produced
    (``:455``). Returns fp ``(b, L, H, P)``.
    """
    b, L, H, P = u.shape
    G, N = C.shape[2], C.shape[3]
    _, _, nc, cs = delta.shape
    hpg = H // G
    up = torch.zeros(b, nc * cs, H, P, dtype=dtype)
    up[:, :L] = u.to(dtype)
    Cp = torch.zeros(b, nc * cs, G, N, dtype=dtype)
    Cp[:, :L] = C.to(dtype)
    up = up.view(b, nc, cs, H, P)
    Ch = Cp.view(b, nc, cs, G, N).repeat_interleave(hpg, dim=3)  # (b,nc,cs,H,N)
    cum = decay_cumsum.to(dtype).permute(0, 2, 1, 3)  # (b,nc,H,cs)
    dt = delta.to(dtype).permute(0, 2, 1, 3)
    # inter-chunk term
    y_off = torch.einsum("bclhn,bchpn->bclhp", Ch, prev_states.to(dtype))
    y_off = y_off * torch.exp(cum).permute(0, 1, 3, 2)[..., None]
    # intra-chunk term
    CBh = CB.to(dtype).repeat_interleave(hpg, dim=2)  # (b,nc,H,cs,cs)
    seg = torch.clamp(cum[..., :, None] - cum[..., None, :], max=0.0)
    causal = torch.tril(torch.ones(cs, cs, dtype=torch.bool))
    M = torch.where(causal, CBh * torch.exp(seg) * dt[..., None, :], torch.zeros((), dtype=dtype))
    y_in = torch.einsum("bchls,bcshp->bclhp", M, up)
    y = (y_off + y_in).reshape(b, nc * cs, H, P)[:, :L]
    return y


def ssd_scan_forward(u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None,
                     chunk_size=256, use_delta_softplus=True, delta_limit=(0.0, INF),
                     is_causal=True, dtype=torch.float32):
    """``ssd_scan/forward.py:223-276``: chain of the five stages.

    ``decay_last = decay_cumsum[..., -1]`` (``:262``). ``is_causal`` does not change
    ``y`` (chunk_scan hardcodes causal, ``forward.py:213``). Returns ``(y, h_last)``
    in ``dtype``: ``y (b, L, H, P)``, ``h_last (b, H, P, N)``.
    """
    b, L, H, P = u.shape
    if length is None:
        length = torch.full((b,), L, dtype=torch.long)
    cum, dt = chunk_cumsum(A, delta_raw, delta_bias, length, chunk_size,
                           use_delta_softplus, delta_limit, dtype=dtype)
    S = chunk_state(u, B, dt, cum, dtype=dtype)
    prev, h_last = state_passing(S, h_init, cum[..., -1], dtype=dtype)
    CB = bmm_chunk(B, C, chunk_size, dtype=dtype)
    y = chunk_scan(u, dt, cum, C, prev, CB, dtype=dtype)
    return y, h_last


def gate_epilogue(y, x, D=None, z=None):
    """D-skip and z-gate as the reference SSM layer applies them after the scan.

    ``modules/ssm.py:144-150``: ``y = (y + D * x) * silu(z)`` with ``D`` per channel
    (``(H*P,)``, ``ssm.py:69``); computed in fp32.
    """
    b, L, H, P = y.shape
    out = y.to(torch.float32)
    if D is not None:
        out = out + D.to(torch.float32).view(H, P) * x.to(torch.float32)
    if z is not None:
        zz = z.to(torch.float32).reshape(b, L, H, P)
        out = out * (zz * torch.sigmoid(zz))
    return out


def ssu_forward(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus=True,
                delta_limit=(0.0, INF), dtype=torch.float32):
    """``ssu/forward.py:7-63`` + kernel ``ssu/forward_kernel.py:6-78``.

    ``h' = h * exp(A*dt) + (B[n]*dt) * u[p]`` (``:135``); ``y[p] = sum_n h'[p,n] C[n]``
    (``:137``). Returns ``(y, h_new)`` in ``dtype`` without touching ``h``; the
    reference stores ``h'`` in place and returns ``y`` in ``u``'s dtype.
    """
    b, H, P = u.shape
    G, N = B.shape[1], B.shape[2]
    hpg = H // G
    d = delta_raw.to(dtype)
    if delta_bias is not None:
        d = d + delta_bias.to(dtype)[None, :]
    d = _dt_transform(d, use_delta_softplus, delta_limit)  # (b,H)
    Bh = B.to(dtype).repeat_interleave(hpg, dim=1)  # (b,H,N)
    Ch = C.to(dtype).repeat_interleave(hpg, dim=1)
    decay = torch.exp(A.to(dtype)[None, :] * d)  # (b,H)
    h_new = h.to(dtype) * decay[..., None, None] + (Bh * d[..., None])[:, :, None, :] * u.to(dtype)[..., None]
    y = (h_new * Ch[:, :, None, :]).sum(-1)
    return y, h_new


def ssd_recurrence(u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None,
                   use_delta_softplus=True, delta_limit=(0.0, INF), dtype=torch.float64):
    """Token-sequential recurrence the chunked scan is an algebraic rewrite of.

    ``h_t = exp(A dt_t) h_{t-1} + dt_t x_t B_t^T``, ``y_t = h_t C_t``, with
    ``dt_t = 0`` past ``length`` (state frozen, ``forward_kernel.py:80``). Exact for
    ``A <= 0`` and ``dt >= 0`` (the ``min(.,0)`` clamps at ``:178,438`` are inert then).
    Pure-Python loop over tokens: small shapes only.
    """
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    if length is None:
        length = torch.full((b,), L, dtype=torch.long)
    d = delta_raw.to(dtype)
    if delta_bias is not None:
        d = d + delta_bias.to(dtype)
    d = _dt_transform(d, use_delta_softplus, delta_limit)
    t = torch.arange(L)
    d = torch.where(t[None, :, None] < length[:, None, None], d, torch.zeros((), dtype=dtype))
    h = torch.zeros(b, H, P, N, dtype=dtype) if h_init is None else h_init.to(dtype).clone()
    Bh = B.to(dtype).repeat_interleave(hpg, dim=2)
    Ch = C.to(dtype).repeat_interleave(hpg, dim=2)
    x = u.to(dtype)
    Ad = A.to(dtype)
    y = torch.empty(b, L, H, P, dtype=dtype)
    for i in range(L):
        dti = d[:, i]  # (b,H)
        h = h * torch.exp(Ad[None, :] * dti)[..., None, None] + (dti[..., None, None] * x[:, i][..., None]) * Bh[:, i][:, :, None, :]
        y[:, i] = (h * Ch[:, i][:, :, None, :]).sum(-1)
    return y, h


def varlen_to_padded(x_packed: torch.Tensor, cu_seqlens: torch.Tensor):
    """Unpack ``(1, T, ...)`` packed rows into a right-padded ``(nseq, maxlen, ...)`` batch.

    The reference has no packed mode; its equivalent is a padded batch plus
    ``length`` (``ops/ssd_scan.py:18,67-68``), which is how packed inputs are checked.
    """
    cu = cu_seqlens.tolist()
    lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    maxlen = max(lens)
    out = torch.zeros((len(lens), maxlen) + tuple(x_packed.shape[2:]), dtype=x_packed.dtype)
    for i, n in enumerate(lens):
        out[i, :n] = x_packed[0, cu[i]:cu[i] + n]
    return out, torch.tensor(lens, dtype=torch.long)


def padded_to_varlen(y_pad: torch.Tensor, cu_seqlens: torch.Tensor):
    """Inverse of :func:`varlen_to_padded` for outputs: gather the valid rows back."""
    cu = cu_seqlens.tolist()
    parts = [y_pad[i, :cu[i + 1] - cu[i]] for i in range(len(cu) - 1)]
    return torch.cat(parts, dim=0)[None]


def ssd_scan_varlen(u, A, B, C, delta_raw, delta_bias, cu_seqlens, chunk_size=256,
                    use_delta_softplus=True, delta_limit=(0.0, INF), dtype=torch.float32,
                    h_init=None):
    """Packed-sequence SSD as the padded reference computes it.

    Each sequence of the packed batch is run as its own right-padded row with
    ``length = seqlen`` and zero (or given per-sequence) initial state; outputs are
    gathered back to packed order. Returns ``(y (1,T,H,P), h_last (nseq,H,P,N))``.
    """
    up, lens = varlen_to_padded(u, cu_seqlens)
    Bp, _ = varlen_to_padded(B, cu_seqlens)
    Cp, _ = varlen_to_padded(C, cu_seqlens)
    dp, _ = varlen_to_padded(delta_raw, cu_seqlens)
    y, h_last = ssd_scan_forward(up, A, Bp, Cp, dp, delta_bias, h_init, lens, chunk_size,
                                 use_delta_softplus, delta_limit, True, dtype=dtype)
    return padded_to_varlen(y, cu_seqlens), h_last
