"""Host functions over the C ABI, mirroring ``triton_kernels`` of the reference.

Names, argument order and return layouts follow
``triton_kernels/ssd_scan/forward.py`` (``chunk_cumsum_forward`` :14,
``chunk_state_forward`` :62, ``state_passing_forward`` :102, ``bmm_chunk_forward`` :139,
``chunk_scan_forward`` :175, ``ssd_scan_forward`` :223) and ``triton_kernels/ssu/forward.py``
(``ssu_forward`` :7). Every launch goes on the current torch stream of the inputs'
device; nothing synchronizes.

Internal layout note: the CUDA kernels keep ``delta`` / ``decay_cumsum`` chunk-major,
``(b, nc, H, cs)``; the functions here return them as ``(b, H, nc, cs)`` views, the
reference's layout, and accept either.
"""
from __future__ import annotations

import math
from ctypes import byref, c_void_p
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from .utils import check_cuda, to_contiguous

INF = float("inf")


def _params(**kw) -> _lib.SSDParams:
    p = _lib.SSDParams()
    p.delta_min, p.delta_max = 0.0, INF
    p.use_delta_softplus = 1
    p.cu_dtype = 64
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def _chunk_major(t: torch.Tensor) -> torch.Tensor:
    """(b, H, nc, cs) reference layout -> contiguous (b, nc, H, cs) kernel layout."""
    return t.permute(0, 2, 1, 3).contiguous()


def _aligned16(t: torch.Tensor) -> torch.Tensor:
    """The tensor-core path moves tiles with TMA / bulk copies, which need 16-byte
    aligned base addresses; an offset view is copied into a fresh allocation."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _stream(dev) -> c_void_p:
    return c_void_p(_lib.stream_handle(dev))


def chunk_cumsum_forward(A, delta_raw, delta_bias, length, chunk_size, use_delta_softplus=True,
                         delta_limit: Tuple[float, float] = (0.0, INF)):
    """Returns ``(decay_cumsum, delta)``, each ``(b, H, nc, cs)`` fp32 (views)."""
    b, L, H = delta_raw.shape
    dev = check_cuda([A, delta_raw, delta_bias, length], ["A", "delta_raw", "delta_bias", "length"])
    nc = math.ceil(L / chunk_size)
    A = to_contiguous(A.float())
    delta_raw = to_contiguous(delta_raw)
    delta_bias = None if delta_bias is None else to_contiguous(delta_bias.float())
    length = None if length is None else to_contiguous(length.to(torch.int64))
    dt = torch.empty(b, nc, H, chunk_size, device=dev, dtype=torch.float32)
    cum = torch.empty_like(dt)
    p = _params(batch=b, seqlen=L, nheads=H, headdim=1, dstate=4, ngroups=1, chunk_size=chunk_size,
                dt_dtype=_lib.dtype_code(delta_raw.dtype, "delta_raw"),
                use_delta_softplus=int(bool(use_delta_softplus)),
                delta_min=float(delta_limit[0]), delta_max=float(delta_limit[1]),
                A=_lib.ptr(A), delta_raw=_lib.ptr(delta_raw), delta_bias=_lib.ptr(delta_bias),
                length=_lib.ptr(length), dt=_lib.ptr(dt), cum=_lib.ptr(cum))
    _lib.check(_lib.lib().ssd_chunk_cumsum_fwd(byref(p), _stream(dev)), "chunk_cumsum_forward")
    return cum.permute(0, 2, 1, 3), dt.permute(0, 2, 1, 3)


def chunk_state_forward(u, B, delta, decay_cumsum, impl: str = "auto"):
    """Per-chunk states ``(b, nc, H, P, N)`` fp32."""
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    nc, cs = delta.shape[2], delta.shape[3]
    dev = check_cuda([u, B, delta, decay_cumsum], ["u", "B", "delta", "decay_cumsum"])
    u, B = to_contiguous(u), to_contiguous(B)
    if B.dtype != u.dtype:
        raise ValueError(f"[B] dtype {B.dtype} differs from u's {u.dtype}")
    dt, cum = _chunk_major(delta.float()), _chunk_major(decay_cumsum.float())
    states = torch.empty(b, nc, H, P, N, device=dev, dtype=torch.float32)
    p = _params(batch=b, seqlen=L, nheads=H, headdim=P, dstate=N, ngroups=G, chunk_size=cs,
                x_dtype=_lib.dtype_code(u.dtype, "u"), impl=_lib.IMPLS[impl],
                u=_lib.ptr(u), B=_lib.ptr(B), dt=_lib.ptr(dt), cum=_lib.ptr(cum), states=_lib.ptr(states))
    _lib.check(_lib.lib().ssd_chunk_state_fwd(byref(p), _stream(dev)), "chunk_state_forward")
    return states


def state_passing_forward(h, h_init, decay_last):
    """``h``: ``(b, nc, H, P*N)`` per-chunk states, overwritten in place with the
    states entering each chunk; returns ``(h, h_last)`` like the reference."""
    b, nc, H, PN = h.shape
    dev = check_cuda([h, h_init, decay_last], ["h", "h_init", "decay_last"])
    if h.dtype != torch.float32 or not h.is_contiguous():
        raise ValueError("[h] expected a contiguous float32 tensor (updated in place)")
    h_init = None if h_init is None else to_contiguous(h_init.float())
    # decay_last (b, H, nc) is presented to the kernel as a cumsum with chunk_size 1.
    last = decay_last.float().permute(0, 2, 1).contiguous()  # (b, nc, H)
    h_last = torch.empty(b, H, PN, device=dev, dtype=torch.float32)
    p = _params(batch=b, seqlen=nc, nheads=H, headdim=1, dstate=PN, ngroups=1, chunk_size=1,
                states=_lib.ptr(h), cum=_lib.ptr(last), h_init=_lib.ptr(h_init), h_last=_lib.ptr(h_last))
    _lib.check(_lib.lib().ssd_state_passing_fwd(byref(p), _stream(dev)), "state_passing_forward")
    return h, h_last


def bmm_chunk_forward(B, C, chunk_size, is_causal=False):
    """``CB = C B^T`` per chunk and group, ``(b, nc, G, cs, cs)`` fp32; rows/columns
    past ``seq_len`` are zero. (Written for every tile regardless of ``is_causal``.)"""
    b, L, G, N = B.shape
    dev = check_cuda([B, C], ["B", "C"])
    B, C = to_contiguous(B), to_contiguous(C)
    nc = math.ceil(L / chunk_size)
    CB = torch.empty(b, nc, G, chunk_size, chunk_size, device=dev, dtype=torch.float32)
    p = _params(batch=b, seqlen=L, nheads=G, headdim=1, dstate=N, ngroups=G, chunk_size=chunk_size,
                x_dtype=_lib.dtype_code(B.dtype, "B"), B=_lib.ptr(B), C=_lib.ptr(C), CB=_lib.ptr(CB))
    # headdim*dstate must be a multiple of 4 for the geometry check; bmm ignores headdim.
    p.headdim = 4
    _lib.check(_lib.lib().ssd_bmm_chunk_fwd(byref(p), _stream(dev)), "bmm_chunk_forward")
    return CB


def chunk_scan_forward(u, delta, decay_cumsum, C, h, CB, D=None, z=None, out_dtype=torch.float32):
    """``y (b, L, H, P)``; ``h`` holds the states entering each chunk (fp32)."""
    b, L, H, P = u.shape
    G, N = C.shape[2], C.shape[3]
    nc, cs = delta.shape[2], delta.shape[3]
    dev = check_cuda([u, delta, decay_cumsum, C, h, CB, D, z], ["u", "delta", "decay_cumsum", "C", "h", "CB", "D", "z"])
    u, C = to_contiguous(u), to_contiguous(C)
    h, CB = to_contiguous(h.float()), to_contiguous(CB.float())
    dt, cum = _chunk_major(delta.float()), _chunk_major(decay_cumsum.float())
    D = None if D is None else to_contiguous(D.float())
    z = None if z is None else to_contiguous(z.to(u.dtype))
    y = torch.empty(b, L, H, P, device=dev, dtype=out_dtype)
    p = _params(batch=b, seqlen=L, nheads=H, headdim=P, dstate=N, ngroups=G, chunk_size=cs,
                x_dtype=_lib.dtype_code(u.dtype, "u"), dt_dtype=0, y_dtype=_lib.dtype_code(out_dtype, "y"),
                u=_lib.ptr(u), C=_lib.ptr(C), dt=_lib.ptr(dt), cum=_lib.ptr(cum), states=_lib.ptr(h),
                CB=_lib.ptr(CB), D=_lib.ptr(D), z=_lib.ptr(z), y=_lib.ptr(y))
    _lib.check(_lib.lib().ssd_chunk_scan_fwd(byref(p), _stream(dev)), "chunk_scan_forward")
    return y


def ssd_scan_params(u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None, chunk_size=256,
                    use_delta_softplus=True, delta_limit=(0.0, INF), D=None, z=None, cu_seqlens=None,
                    impl: str = "auto", y_dtype: Optional[torch.dtype] = None):
    """Build the ``ssd_params`` block for ``ssd_scan_fwd`` (no outputs or workspace yet).

    Returns ``(params, keep)``; ``keep`` holds the converted tensors the pointers refer to.
    """
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    A = to_contiguous(A.float())
    delta_bias = None if delta_bias is None else to_contiguous(delta_bias.float())
    h_init = None if h_init is None else to_contiguous(h_init.float())
    length = None if length is None else to_contiguous(length.to(torch.int64))
    D = None if D is None else _aligned16(to_contiguous(D.float()))
    if z is not None:
        if z.dtype != u.dtype:
            raise ValueError(f"[z] dtype {z.dtype} differs from u's {u.dtype}")
        z = _aligned16(to_contiguous(z))
    u, B, C = _aligned16(u), _aligned16(B), _aligned16(C)
    if y_dtype is None:
        y_dtype = u.dtype if (D is not None or z is not None) else torch.float32
    nseq = 0
    cu_dtype = 64
    if cu_seqlens is not None:
        if cu_seqlens.dtype not in (torch.int32, torch.int64):
            raise ValueError("[cu_seqlens] expected int32 or int64")
        cu_seqlens = to_contiguous(cu_seqlens)
        nseq = cu_seqlens.numel() - 1
        cu_dtype = 64 if cu_seqlens.dtype == torch.int64 else 32
    p = _params(batch=b, seqlen=L, nheads=H, headdim=P, dstate=N, ngroups=G, chunk_size=int(chunk_size),
                nseq=nseq, x_dtype=_lib.dtype_code(u.dtype, "u"),
                dt_dtype=_lib.dtype_code(delta_raw.dtype, "delta_raw"), y_dtype=_lib.dtype_code(y_dtype, "y"),
                cu_dtype=cu_dtype, use_delta_softplus=int(bool(use_delta_softplus)),
                delta_min=float(delta_limit[0]), delta_max=float(delta_limit[1]), impl=_lib.IMPLS[impl],
                u=_lib.ptr(u), A=_lib.ptr(A), B=_lib.ptr(B), C=_lib.ptr(C), delta_raw=_lib.ptr(delta_raw),
                delta_bias=_lib.ptr(delta_bias), h_init=_lib.ptr(h_init), length=_lib.ptr(length),
                D=_lib.ptr(D), z=_lib.ptr(z), cu_seqlens=_lib.ptr(cu_seqlens))
    keep = (u, A, B, C, delta_raw, delta_bias, h_init, length, D, z, cu_seqlens)
    return p, keep, y_dtype


def workspace_size(params) -> int:
    return int(_lib.lib().ssd_scan_fwd_workspace_size(byref(params)))


def uses_tensor_cores(params) -> bool:
    return bool(_lib.lib().ssd_scan_uses_tensor_cores(byref(params)))


SCAN_PATHS = {0: "simt", 1: "tc_staged", 2: "tc_fused", 3: "tc_split"}


def scan_path(params) -> str:
    """Kernel chain of ``ssd_scan_fwd`` for these parameters: "simt", "tc_staged",
    "tc_fused" (chunk_state and state_passing in one kernel) or "tc_split" (fp32 inputs:
    chunk_state, bmm_chunk and chunk_scan on tensor cores with split-bf16 products)."""
    code = _lib.lib().ssd_scan_path(byref(params))
    if code < 0:
        raise ValueError("invalid SSD geometry")
    return SCAN_PATHS[code]


def ssd_scan_forward(u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None, chunk_size=256,
                     use_delta_softplus=True, delta_limit=(0.0, INF), is_causal=True, D=None, z=None,
                     cu_seqlens=None, impl: str = "auto", out: Optional[Sequence[torch.Tensor]] = None,
                     workspace: Optional[torch.Tensor] = None, events=None):
    """Fused SSD forward. Returns ``(y, h_last)``.

    ``y`` is fp32 (the reference contract, ``forward.py:200``) unless ``D`` or ``z``
    is given, in which case the epilogue ``(y + D*u) * silu(z)`` is applied and
    ``y`` has ``u``'s dtype. ``is_causal`` does not change the result (the reference
    hardcodes causal chunk_scan, ``forward.py:213``). With ``cu_seqlens`` (packed
    mode, b = 1) ``h_last`` is ``(nseq, H, P, N)``.
    """
    b, L, H, P = u.shape
    N = B.shape[3]
    dev = check_cuda([u, A, B, C, delta_raw, delta_bias, h_init, length, D, z, cu_seqlens],
                     ["u", "A", "B", "C", "delta_raw", "delta_bias", "h_init", "length", "D", "z", "cu_seqlens"])
    u, B, C, delta_raw = to_contiguous(u), to_contiguous(B), to_contiguous(C), to_contiguous(delta_raw)
    for t, n in ((B, "B"), (C, "C")):
        if t.dtype != u.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from u's {u.dtype}")
    p, keep, y_dtype = ssd_scan_params(u, A, B, C, delta_raw, delta_bias, h_init, length, chunk_size,
                                       use_delta_softplus, delta_limit, D, z, cu_seqlens, impl)
    nrows = b if cu_seqlens is None else cu_seqlens.numel() - 1
    if out is None:
        y = torch.empty(b, L, H, P, device=dev, dtype=y_dtype)
        h_last = torch.empty(nrows, H, P, N, device=dev, dtype=torch.float32)
    else:
        y, h_last = out
    need = workspace_size(p)
    if need == 0:
        raise ValueError("invalid SSD geometry (sizes, heads/groups, chunk_size <= 256)")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=dev, dtype=torch.uint8)
    p.y, p.h_last = _lib.ptr(y), _lib.ptr(h_last)
    p.workspace, p.workspace_bytes = _lib.ptr(workspace), workspace.numel()
    if events is not None:
        for i, e in enumerate(events):
            p.events[i] = None if e is None else e
    _lib.check(_lib.lib().ssd_scan_fwd(byref(p), _stream(dev)), "ssd_scan_forward")
    del keep
    return y, h_last


def ssd_scan_backward(u, A, B, C, delta_raw, delta_bias, h_init, y_grad, h_last_grad, length=None,
                      chunk_size=256, use_delta_softplus=True, delta_limit=(0.0, INF), is_causal=True,
                      cu_seqlens=None, workspace: Optional[torch.Tensor] = None, events=None):
    """SSD backward, the reference's ``ssd_scan/backward.py:467 ssd_scan_backward``.

    Same arguments and outputs: ``(u_grad, A_grad, B_grad, C_grad, delta_raw_grad,
    delta_bias_grad, h_init_grad)`` with ``u_grad`` in ``u``'s dtype, ``delta_raw_grad``
    in ``delta_raw``'s, the rest fp32 (``backward.py:90,144,200,254,439-441``);
    ``delta_bias_grad`` / ``h_init_grad`` are None when ``delta_bias`` / ``h_init`` are.
    ``h_last_grad`` may be None (zero). ``is_causal`` changes nothing (the forward is
    always causal). ``cu_seqlens`` selects packed rows as in :func:`ssd_scan_forward`.
    """
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    dev = check_cuda([u, A, B, C, delta_raw, delta_bias, h_init, length, y_grad, h_last_grad, cu_seqlens],
                     ["u", "A", "B", "C", "delta_raw", "delta_bias", "h_init", "length", "y_grad",
                      "h_last_grad", "cu_seqlens"])
    u, B, C, delta_raw = to_contiguous(u), to_contiguous(B), to_contiguous(C), to_contiguous(delta_raw)
    for t, n in ((B, "B"), (C, "C")):
        if t.dtype != u.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from u's {u.dtype}")
    if tuple(y_grad.shape) != (b, L, H, P):
        raise ValueError(f"[y_grad] expected shape {(b, L, H, P)}, got {tuple(y_grad.shape)}")
    y_grad = _aligned16(to_contiguous(y_grad))
    nrows = b if cu_seqlens is None else cu_seqlens.numel() - 1
    if h_last_grad is not None:
        if tuple(h_last_grad.shape) != (nrows, H, P, N):
            raise ValueError(f"[h_last_grad] expected shape {(nrows, H, P, N)}, got {tuple(h_last_grad.shape)}")
        h_last_grad = _aligned16(to_contiguous(h_last_grad.float()))
    p, keep, _ = ssd_scan_params(u, A, B, C, delta_raw, delta_bias, h_init, length, chunk_size,
                                 use_delta_softplus, delta_limit, None, None, cu_seqlens, "simt",
                                 y_dtype=torch.float32)
    need = int(_lib.lib().ssd_scan_bwd_workspace_size(byref(p)))
    if need == 0:
        raise ValueError("unsupported SSD backward geometry (headdim <= 64 and dstate <= 128, multiples of 8; "
                         "chunk_size a multiple of 32 up to 256; heads a multiple of groups)")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=dev, dtype=torch.uint8)
    p.workspace, p.workspace_bytes = _lib.ptr(workspace), workspace.numel()
    if events is not None:
        for i, e in enumerate(events):
            p.events[i] = None if e is None else e
    u_grad = torch.empty_like(u)
    A_grad = torch.empty(H, device=dev, dtype=torch.float32)
    B_grad = torch.empty(b, L, G, N, device=dev, dtype=torch.float32)
    C_grad = torch.empty(b, L, G, N, device=dev, dtype=torch.float32)
    delta_raw_grad = torch.empty_like(delta_raw)
    delta_bias_grad = None if delta_bias is None else torch.empty(H, device=dev, dtype=torch.float32)
    h_init_grad = None if h_init is None else torch.empty(nrows, H, P, N, device=dev, dtype=torch.float32)
    g = _lib.SSDBwdParams(y_grad=_lib.ptr(y_grad), y_grad_dtype=_lib.dtype_code(y_grad.dtype, "y_grad"),
                          h_last_grad=_lib.ptr(h_last_grad), u_grad=_lib.ptr(u_grad), A_grad=_lib.ptr(A_grad),
                          B_grad=_lib.ptr(B_grad), C_grad=_lib.ptr(C_grad), delta_raw_grad=_lib.ptr(delta_raw_grad),
                          delta_bias_grad=_lib.ptr(delta_bias_grad), h_init_grad=_lib.ptr(h_init_grad))
    _lib.check(_lib.lib().ssd_scan_bwd(byref(p), byref(g), _stream(dev)), "ssd_scan_backward")
    del keep
    return u_grad, A_grad, B_grad, C_grad, delta_raw_grad, delta_bias_grad, h_init_grad


def ssu_forward(u, A, B, C, delta_raw, delta_bias, h, use_delta_softplus=True, delta_limit=(0.0, INF),
                D=None, z=None, y=None):
    """One-token state update; ``h`` is updated in place. Returns ``(y, h)`` with ``y``
    in ``u``'s dtype (``ssu/forward.py:34``)."""
    b, H, P = u.shape
    G, N = B.shape[1], B.shape[2]
    dev = check_cuda([u, A, B, C, delta_raw, delta_bias, h, D, z],
                     ["u", "A", "B", "C", "delta_raw", "delta_bias", "h", "D", "z"])
    u, B, C, delta_raw = to_contiguous(u), to_contiguous(B), to_contiguous(C), to_contiguous(delta_raw)
    for t, n in ((B, "B"), (C, "C")):
        if t.dtype != u.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from u's {u.dtype}")
    A = to_contiguous(A.float())
    delta_bias = None if delta_bias is None else to_contiguous(delta_bias.float())
    D = None if D is None else to_contiguous(D.float())
    if z is not None:
        if z.dtype != u.dtype:
            raise ValueError(f"[z] dtype {z.dtype} differs from u's {u.dtype}")
        z = to_contiguous(z)
    if h.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"[h] unsupported state dtype {h.dtype}; expected float32 or bfloat16")
    if y is None:
        y = torch.empty_like(u)
    st = _lib.lib().ssu_fwd(
        _lib.ptr(u), _lib.ptr(A), _lib.ptr(B), _lib.ptr(C), _lib.ptr(delta_raw), _lib.ptr(delta_bias),
        _lib.ptr(h), _lib.ptr(y), _lib.ptr(D), _lib.ptr(z), b, H, P, N, G,
        _lib.dtype_code(u.dtype, "u"), _lib.dtype_code(delta_raw.dtype, "delta_raw"),
        _lib.dtype_code(h.dtype, "h"), _lib.dtype_code(y.dtype, "y"), int(bool(use_delta_softplus)),
        float(delta_limit[0]), float(delta_limit[1]), _stream(dev))
    _lib.check(st, "ssu_forward")
    return y, h


def ssm_conv_prefill(hBC, conv_weight, conv_bias, inner_dim, gn, lengths=None, build_ctx=False, out=None):
    """SSM prefill front end (``modules/ssm.py:112-134``): ``silu`` then the depthwise causal
    conv over the sequence, split into ``x`` (b, L, inner_dim), ``B`` and ``C`` (b, L, gn),
    in ``hBC``'s dtype; with ``build_ctx`` also the decode cache ``conv_ctx`` (b, conv_dim, K)
    of ``SSMCache.build_conv_ctx`` (``inference/ssm_cache.py:10-36``), the last K inputs
    before each row's length (zeros where missing).

    ``hBC`` is (b, L, conv_dim) with contiguous channels and any token stride, e.g. the
    first ``conv_dim`` columns of the input projection's output. ``conv_weight`` is the
    depthwise ``nn.Conv1d`` weight (conv_dim, 1, K) or (conv_dim, K); ``conv_bias``
    (conv_dim,) or None. Returns ``(x, B, C, conv_ctx or None)``."""
    if hBC.dim() != 3:
        raise ValueError(f"[hBC] expected (batch, seq_len, conv_dim), got {tuple(hBC.shape)}")
    b, L, conv_dim = hBC.shape
    if conv_dim != inner_dim + 2 * gn:
        raise ValueError(f"[hBC] conv_dim {conv_dim} != inner_dim + 2 * gn = {inner_dim + 2 * gn}")
    w = conv_weight.reshape(conv_weight.shape[0], -1)
    if w.shape[0] != conv_dim or not 1 <= w.shape[1] <= 8:
        raise ValueError(f"[conv_weight] expected (conv_dim, 1, K) with K <= 8, got {tuple(conv_weight.shape)}")
    K = w.shape[1]
    dev = check_cuda([hBC, conv_weight, conv_bias, lengths], ["hBC", "conv_weight", "conv_bias", "lengths"])
    if hBC.stride(2) != 1:
        hBC = hBC.contiguous()
    if hBC.stride(0) != L * hBC.stride(1):
        hBC = hBC.contiguous()  # rows of one batch entry must follow each other at the token stride
    w = to_contiguous(w.float())
    bias = None if conv_bias is None else to_contiguous(conv_bias.float())
    if lengths is not None:
        lengths = to_contiguous(lengths.to(torch.int64))
    if out is None:
        x = torch.empty(b, L, inner_dim, dtype=hBC.dtype, device=hBC.device)
        Bo = torch.empty(b, L, gn, dtype=hBC.dtype, device=hBC.device)
        Co = torch.empty(b, L, gn, dtype=hBC.dtype, device=hBC.device)
    else:
        x, Bo, Co = out
    ctx = torch.empty(b, conv_dim, K, dtype=hBC.dtype, device=hBC.device) if build_ctx else None
    st = _lib.lib().ssm_conv_prefill(
        _lib.ptr(hBC), hBC.stride(1), _lib.ptr(w), _lib.ptr(bias), _lib.ptr(x), _lib.ptr(Bo), _lib.ptr(Co),
        _lib.ptr(ctx), _lib.ptr(lengths), b, L, inner_dim, gn, K, _lib.dtype_code(hBC.dtype, "hBC"), _stream(dev))
    _lib.check(st, "ssm_conv_prefill")
    return x, Bo, Co, ctx


def ssm_conv_decode(hBC, conv_ctx, conv_weight, conv_bias, inner_dim, gn, out=None):
    """SSM decode-step front end (``modules/ssm.py:173-186``): ``SSMCache.update``
    (``inference/ssm_cache.py:38-43``, the cache window shifted left by one with ``hBC``
    appended, in place in ``conv_ctx``), then ``(silu(conv_ctx) * weight).sum(-1) + bias``
    with the reference's roundings to ``hBC``'s dtype, split into ``x`` (b, inner_dim),
    ``B`` and ``C`` (b, gn). ``hBC`` (b, conv_dim) may be a slice of the projection output
    (contiguous channels, any row stride); ``conv_ctx`` (b, conv_dim, K) contiguous, in
    ``hBC``'s dtype. Returns ``(x, B, C)``."""
    if hBC.dim() != 2:
        raise ValueError(f"[hBC] expected (batch, conv_dim), got {tuple(hBC.shape)}")
    b, conv_dim = hBC.shape
    if conv_dim != inner_dim + 2 * gn:
        raise ValueError(f"[hBC] conv_dim {conv_dim} != inner_dim + 2 * gn = {inner_dim + 2 * gn}")
    w = conv_weight.reshape(conv_weight.shape[0], -1)
    K = w.shape[1]
    if w.shape[0] != conv_dim or not 1 <= K <= 8:
        raise ValueError(f"[conv_weight] expected (conv_dim, 1, K) with K <= 8, got {tuple(conv_weight.shape)}")
    if conv_ctx.shape != (b, conv_dim, K) or conv_ctx.dtype != hBC.dtype or not conv_ctx.is_contiguous():
        raise ValueError(f"[conv_ctx] expected a contiguous {(b, conv_dim, K)} tensor of {hBC.dtype}")
    dev = check_cuda([hBC, conv_ctx, conv_weight, conv_bias], ["hBC", "conv_ctx", "conv_weight", "conv_bias"])
    if hBC.stride(1) != 1:
        hBC = hBC.contiguous()
    w = to_contiguous(w.float())
    bias = None if conv_bias is None else to_contiguous(conv_bias.float())
    if out is None:
        x = torch.empty(b, inner_dim, dtype=hBC.dtype, device=hBC.device)
        Bo = torch.empty(b, gn, dtype=hBC.dtype, device=hBC.device)
        Co = torch.empty(b, gn, dtype=hBC.dtype, device=hBC.device)
    else:
        x, Bo, Co = out
    st = _lib.lib().ssm_conv_decode(
        _lib.ptr(hBC), hBC.stride(0), _lib.ptr(conv_ctx), _lib.ptr(w), _lib.ptr(bias), _lib.ptr(x), _lib.ptr(Bo),
        _lib.ptr(Co), b, inner_dim, gn, K, _lib.dtype_code(hBC.dtype, "hBC"), _stream(dev))
    _lib.check(st, "ssm_conv_decode")
    return x, Bo, Co


def sattn_decode_step(q_rot, k_rot, v, log_gate, k_cache, v_cache, log_gate_cache, write_idx, scale=None,
                      out=None):
    """Selective-attention decode step on a KV cache (C-ABI ``sattn_decode_step``).

    Writes ``k_rot``, ``v`` and ``log_gate`` at slot ``write_idx`` of the caches, in place
    (``inference/selective_attn_cache.py:39-41``), then returns the pos-mode gated softmax
    attention of ``q_rot`` over the first ``write_idx + 1`` slots
    (``modules/selective_attention.py:399-404``), ``(b, H, D)`` in ``q_rot``'s dtype. The caller
    advances its write index. ``scale`` defaults to ``D ** -0.5`` (``:163``). Caches must be
    contiguous ``(b, H, cap, D)`` / ``(b, H, cap)`` with ``log_gate_cache`` fp32.
    """
    b, H, D = q_rot.shape
    dev = check_cuda([q_rot, k_rot, v, log_gate, k_cache, v_cache, log_gate_cache],
                     ["q_rot", "k_rot", "v", "log_gate", "k_cache", "v_cache", "log_gate_cache"])
    cap = k_cache.shape[2]
    if k_cache.dim() != 4 or tuple(k_cache.shape) != (b, H, cap, D) or tuple(v_cache.shape) != (b, H, cap, D):
        raise ValueError(f"[k_cache] expected (b, H, cap, D) = ({b}, {H}, cap, {D}) caches")
    if tuple(log_gate_cache.shape) != (b, H, cap) or log_gate_cache.dtype != torch.float32:
        raise ValueError("[log_gate_cache] expected a (b, H, cap) float32 cache")
    for t, n in ((k_rot, "k_rot"), (v, "v")):
        if tuple(t.shape) != (b, H, D):
            raise ValueError(f"[{n}] expected shape {(b, H, D)}, got {tuple(t.shape)}")
    for t, n in ((k_rot, "k_rot"), (v, "v"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        if t.dtype != q_rot.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from q_rot's {q_rot.dtype}")
    for t, n in ((k_cache, "k_cache"), (v_cache, "v_cache"), (log_gate_cache, "log_gate_cache")):
        if not t.is_contiguous():
            raise ValueError(f"[{n}] must be contiguous (it is updated in place)")
    if not 0 <= int(write_idx) < cap:
        raise ValueError(f"[write_idx] {write_idx} outside the cache's {cap} slots")
    q_rot = _aligned16(to_contiguous(q_rot))
    k_rot, v = to_contiguous(k_rot), to_contiguous(v)
    log_gate = to_contiguous(log_gate.float()).reshape(b, H)
    if out is None:
        out = torch.empty(b, H, D, device=dev, dtype=q_rot.dtype)
    scale = float(D ** -0.5 if scale is None else scale)
    st = _lib.lib().sattn_decode_step(_lib.ptr(q_rot), _lib.ptr(k_rot), _lib.ptr(v), _lib.ptr(log_gate),
                                      _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(log_gate_cache),
                                      int(write_idx), cap, _lib.ptr(out), b, H, D, scale,
                                      _lib.dtype_code(q_rot.dtype, "q_rot"), _stream(dev))
    _lib.check(st, "sattn_decode_step")
    return out


def selective_attn_step(cache, q_rot, k_rot, v, log_select_gate, scale=None):
    """``SelectiveMHA.step``'s cache update and attention (``modules/selective_attention.py:390-404``)
    on a ``SelectiveAttnCache``-like object (``k_rot``, ``v``, ``log_gate`` tensors and
    ``write_idx``): one kernel, ``cache.write_idx`` advanced. Returns ``out`` as
    ``(b, H * D)``, the tensor the layer gates and projects."""
    out = sattn_decode_step(q_rot, k_rot, v, log_select_gate, cache.k_rot, cache.v, cache.log_gate,
                            cache.write_idx, scale)
    cache.write_idx += 1
    return out.view(out.shape[0], -1)


def sattn_prefill(q_rot, k_rot, v, log_gate, scale=None, out=None, impl: str = "auto"):
    """Selective-attention prefill (inference) over whole sequences (C-ABI ``sattn_prefill_fwd``).

    ``q_rot, k_rot, v`` ``(b, H, L, D)``; ``log_gate`` ``(b, H, L)`` (the layer's
    ``log_select_gate`` after its padding mask). Returns ``(b, H, L, D)`` in ``q_rot``'s dtype:
    causal softmax attention where each earlier key adds its log-gate and the token's own
    score is ungated (``modules/selective_attention.py:27-144``, ``:270-280``); zero gates
    (log-gate ``-inf``) drop their key, which is what the reference's compressed path computes.
    ``scale`` defaults to ``D ** -0.5``. ``impl``: ``"auto"`` (tensor cores for 16-bit inputs
    with ``D`` 64 or 128), ``"tc"`` or ``"simt"``.
    """
    b, H, L, D = q_rot.shape
    dev = check_cuda([q_rot, k_rot, v, log_gate], ["q_rot", "k_rot", "v", "log_gate"])
    for t, n in ((k_rot, "k_rot"), (v, "v")):
        if tuple(t.shape) != (b, H, L, D):
            raise ValueError(f"[{n}] expected shape {(b, H, L, D)}, got {tuple(t.shape)}")
        if t.dtype != q_rot.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from q_rot's {q_rot.dtype}")
    if tuple(log_gate.shape) != (b, H, L):
        raise ValueError(f"[log_gate] expected shape {(b, H, L)}, got {tuple(log_gate.shape)}")
    q_rot, k_rot, v = (_aligned16(to_contiguous(t)) for t in (q_rot, k_rot, v))
    log_gate = to_contiguous(log_gate.float())
    if out is None:
        out = torch.empty(b, H, L, D, device=dev, dtype=q_rot.dtype)
    scale = float(D ** -0.5 if scale is None else scale)
    st = _lib.lib().sattn_prefill_fwd(_lib.ptr(q_rot), _lib.ptr(k_rot), _lib.ptr(v), _lib.ptr(log_gate),
                                      _lib.ptr(out), b, H, L, D, scale, _lib.dtype_code(q_rot.dtype, "q_rot"),
                                      _lib.IMPLS[impl], _stream(dev))
    _lib.check(st, "sattn_prefill")
    return out


def _train_params(q_rot, k_rot, v, select_gate, lengths, log_gate_penalty, is_causal, scale, impl):
    b, H, L, D = q_rot.shape
    dev = check_cuda([q_rot, k_rot, v, select_gate, lengths], ["q_rot", "k_rot", "v", "select_gate", "lengths"])
    for t, n in ((k_rot, "k_rot"), (v, "v")):
        if tuple(t.shape) != (b, H, L, D):
            raise ValueError(f"[{n}] expected shape {(b, H, L, D)}, got {tuple(t.shape)}")
        if t.dtype != q_rot.dtype:
            raise ValueError(f"[{n}] dtype {t.dtype} differs from q_rot's {q_rot.dtype}")
    if tuple(select_gate.shape) != (b, H, L):
        raise ValueError(f"[select_gate] expected shape {(b, H, L)}, got {tuple(select_gate.shape)}")
    if lengths is not None and tuple(lengths.shape) != (b,):
        raise ValueError(f"[lengths] expected shape {(b,)}, got {tuple(lengths.shape)}")
    q_rot, k_rot, v = (_aligned16(to_contiguous(t)) for t in (q_rot, k_rot, v))
    select_gate = to_contiguous(select_gate.to(q_rot.dtype))
    lengths = None if lengths is None else to_contiguous(lengths.to(torch.int64))
    p = _lib.SattnTrainParams()
    p.batch, p.nheads, p.seqlen, p.head_dim = b, H, L, D
    p.dtype = _lib.dtype_code(q_rot.dtype, "q_rot")
    p.is_causal = 1 if is_causal else 0
    p.impl = _lib.IMPLS[impl]
    p.scale = float(D ** -0.5 if scale is None else scale)
    p.log_gate_penalty = float(log_gate_penalty)
    p.q_rot, p.k_rot, p.v = _lib.ptr(q_rot), _lib.ptr(k_rot), _lib.ptr(v)
    p.select_gate, p.lengths = _lib.ptr(select_gate), _lib.ptr(lengths)
    keep = (q_rot, k_rot, v, select_gate, lengths)
    return p, dev, keep


def sattn_train_forward(q_rot, k_rot, v, select_gate, log_gate_penalty, lengths=None, is_causal=True, scale=None,
                        impl: str = "auto"):
    """Selective attention in training mode (C-ABI ``sattn_train_fwd``): the part of
    ``SelectiveMHA.forward`` with ``self.training`` from the score matrix to ``attn_weight @ v``
    (``modules/selective_attention.py:232-280``).

    ``q_rot, k_rot, v`` ``(b, H, L, D)``; ``select_gate`` ``(b, H, L)`` (the sigmoid gate,
    transposed as ``:204``); ``lengths`` ``(b,)`` or ``None``. Per head, the mean and std of the
    valid scores (``:234-251``) scale the log-gates (``:259-268``; ``-inf`` past the length), and
    the seq-mode gated softmax (``:125-144``) weights ``v``. Returns ``(out, lse, log_gate, stats)``:
    ``out`` ``(b, H, L, D)`` in ``q_rot``'s dtype; fp32 ``lse`` and ``log_gate`` ``(b, H, L)``;
    ``stats`` ``(H, 4)`` fp32 = mean, std, count of valid scores, and a slot the backward fills.
    ``impl``: ``"auto"`` (tensor cores for 16-bit inputs with ``D`` 64), ``"tc"`` or ``"simt"``.
    """
    p, dev, keep = _train_params(q_rot, k_rot, v, select_gate, lengths, log_gate_penalty, is_causal, scale, impl)
    b, H, L, D = q_rot.shape
    out = torch.empty(b, H, L, D, device=dev, dtype=q_rot.dtype)
    lse = torch.empty(b, H, L, device=dev, dtype=torch.float32)
    lg = torch.empty(b, H, L, device=dev, dtype=torch.float32)
    stats = torch.empty(H, 4, device=dev, dtype=torch.float32)
    L_ = _lib.lib()
    ws = torch.empty(L_.sattn_train_workspace_size(byref(p)), device=dev, dtype=torch.uint8)
    p.out, p.lse, p.log_gate, p.stats = _lib.ptr(out), _lib.ptr(lse), _lib.ptr(lg), _lib.ptr(stats)
    p.workspace, p.workspace_bytes = _lib.ptr(ws), ws.numel()
    _lib.check(L_.sattn_train_fwd(byref(p), _stream(dev)), "sattn_train_fwd")
    del keep
    return out, lse, lg, stats


def sattn_train_backward(q_rot, k_rot, v, select_gate, out, lse, log_gate, stats, dout, log_gate_penalty,
                         lengths=None, is_causal=True, scale=None, impl: str = "auto"):
    """Backward of ``sattn_train_forward`` (C-ABI ``sattn_train_bwd``), the gradients torch's
    autograd gives for ``modules/selective_attention.py:232-280`` including the path through
    the score std. ``out, lse, log_gate, stats`` are the forward's outputs (``stats`` gets its
    backward coefficient written). Returns ``(dq, dk, dv, dselect_gate)`` in ``q_rot``'s dtype.
    ``impl`` as for the forward (both calls must take the same path: the statistics tiles differ).
    """
    p, dev, keep = _train_params(q_rot, k_rot, v, select_gate, lengths, log_gate_penalty, is_causal, scale, impl)
    dout = _aligned16(to_contiguous(dout.to(q_rot.dtype)))
    if tuple(dout.shape) != tuple(q_rot.shape):
        raise ValueError(f"[dout] expected shape {tuple(q_rot.shape)}, got {tuple(dout.shape)}")
    dq, dk, dv = (torch.empty_like(t, memory_format=torch.contiguous_format) for t in (q_rot, q_rot, q_rot))
    dgate = torch.empty(select_gate.shape, device=dev, dtype=q_rot.dtype)
    L_ = _lib.lib()
    ws = torch.empty(L_.sattn_train_workspace_size(byref(p)), device=dev, dtype=torch.uint8)
    p.out, p.lse, p.log_gate, p.stats = _lib.ptr(out), _lib.ptr(lse), _lib.ptr(log_gate), _lib.ptr(stats)
    p.workspace, p.workspace_bytes = _lib.ptr(ws), ws.numel()
    st = L_.sattn_train_bwd(byref(p), _lib.ptr(dout), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv),
                            _lib.ptr(dgate), _stream(dev))
    _lib.check(st, "sattn_train_bwd")
    del keep
    return dq, dk, dv, dgate
