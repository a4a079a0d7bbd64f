"""Generate the selective-attention decode-step golden vectors from the reference.

Uses nmquan1503/selective-attention's own code on CPU: ``SelectiveAttnCache``
(``inference/selective_attn_cache.py``: ``build_kv`` after a prefill, ``update_kv`` per
step), ``_reset_cache`` (``modules/selective_attention.py:11-25``, the buffer growth and
compression ``SelectiveMHA.step`` runs every ``cache_update_interval`` steps) and
``_gated_softmax`` in pos mode (``:121-123``), with the attention lines of
``SelectiveMHA.step`` (``:399-404``) around them. Saves the cache after the reset, every
step's inputs (``q_rot, k_rot, v, log_gate``) and outputs, and the final cache as
``sattn_decode_<case>.pt``.

Prefill cases (``sattn_prefill_<case>.pt``) run the inference attention of
``SelectiveMHA.forward`` (``:252-280``) through the reference's ``_build_attn_matrix``,
``compress`` and the seq-mode ``_gated_softmax``: with some gates at zero the reference takes
its compressed path, with a fully kept (batch row, head) its dense one. Saved: ``q_rot,
k_rot, v``, the log-gates as the layer hands them on (``-inf`` for dropped and padding keys)
and the output. Needs the reference checkout; run from the repository root:
``python tests/golden/make_golden_sattn.py``.
"""
from __future__ import annotations

import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_interp  # noqa: E402  (puts the reference on sys.path, interpreter mode)

ref_interp.load()

import torch  # noqa: E402
from selective_attention.inference import SelectiveAttnCache  # noqa: E402
from selective_attention.modules import selective_attention as sa  # noqa: E402
from selective_attention.utils.tensor_utils import compress  # noqa: E402


def log_gates(g, *shape, p_zero=0.0):
    """log(sigmoid(x + 2)) * 2 (the layer's gate bias is 2.0 and its penalty scales the log),
    with a fraction of gates at exactly zero (log-gate -inf, a key the layer drops)."""
    lg = torch.log(torch.sigmoid(torch.randn(*shape, generator=g) + 2.0)) * 2.0
    if p_zero:
        lg = torch.where(torch.rand(*shape, generator=g) < p_zero, torch.full_like(lg, -math.inf), lg)
    return lg


def run(seed, b, H, D, prefill, interval, steps, p_zero):
    g = torch.Generator().manual_seed(seed)
    scale = D ** -0.5
    cache = SelectiveAttnCache()
    if prefill:
        cache.build_kv(torch.randn(b, H, prefill, D, generator=g), torch.randn(b, H, prefill, D, generator=g),
                       log_gates(g, b, H, prefill, p_zero=p_zero))
        sa._reset_cache(cache, interval)
    else:  # SelectiveMHA.step's first allocation (:364-366); zero-filled here for determinism
        cache.k_rot = torch.zeros(b, H, interval, D)
        cache.v = torch.zeros(b, H, interval, D)
        cache.log_gate = torch.zeros(b, H, interval)
    rec = {"scale": scale, "k0": cache.k_rot.clone(), "v0": cache.v.clone(), "lg0": cache.log_gate.clone(),
           "w0": cache.write_idx, "q": [], "k": [], "v": [], "lg": [], "out": []}
    for _ in range(steps):
        q = torch.randn(b, H, D, generator=g)
        k = torch.randn(b, H, D, generator=g)
        v = torch.randn(b, H, D, generator=g)
        lg = log_gates(g, b, H, p_zero=p_zero)
        cache.update_kv(k, v, lg)
        # SelectiveMHA.step, modules/selective_attention.py:399-404
        ck = cache.k_rot[:, :, :cache.write_idx, :]
        cv = cache.v[:, :, :cache.write_idx, :]
        clg = cache.log_gate[:, :, :cache.write_idx]
        attn = (q.unsqueeze(2) @ ck.transpose(-2, -1)).squeeze(2)
        attn.mul_(scale)
        w = sa._gated_softmax(attn, clg, mode="pos", is_infer=True)
        out = (w.unsqueeze(2) @ cv).squeeze(2)
        for key, t in (("q", q), ("k", k), ("v", v), ("lg", lg), ("out", out)):
            rec[key].append(t)
    for key in ("q", "k", "v", "lg", "out"):
        rec[key] = torch.stack(rec[key])
    rec.update(k_end=cache.k_rot.clone(), v_end=cache.v.clone(), lg_end=cache.log_gate.clone(),
               w_end=cache.write_idx)
    return rec


CASES = {
    # prefilled cache with dropped keys: _reset_cache compresses rows to their kept keys
    "dropped_fp32": dict(seed=21, b=3, H=4, D=64, prefill=37, interval=16, steps=6, p_zero=0.15),
    # fresh cache: the first step attends to the token alone
    "fresh_d128_fp32": dict(seed=22, b=2, H=2, D=128, prefill=0, interval=8, steps=4, p_zero=0.0),
    # a longer prefill (many key groups per warp), every key kept
    "long_fp32": dict(seed=23, b=1, H=2, D=64, prefill=700, interval=4, steps=2, p_zero=0.0),
}


def run_prefill(seed, b, H, L, D, p_zero, lengths=None):
    g = torch.Generator().manual_seed(seed)
    scale = D ** -0.5
    q = torch.randn(b, H, L, D, generator=g)
    k = torch.randn(b, H, L, D, generator=g)
    v = torch.randn(b, H, L, D, generator=g)
    gate = torch.sigmoid(torch.randn(b, H, L, generator=g) + 2.0)
    if p_zero:
        gate = torch.where(torch.rand(b, H, L, generator=g) < p_zero, torch.zeros_like(gate), gate)
    valid = gate > 0.0                                                   # :206
    lg = torch.log(gate) * 2.0                                           # :255-257 (std_ema * penalty = 2)
    if lengths is not None:
        pad = torch.arange(L)[None, :] >= torch.tensor(lengths)[:, None]
        valid &= ~pad[:, None, :]                                        # :210-211
        lg = lg.masked_fill(pad[:, None, :], float("-inf"))              # :263-265
    # SelectiveMHA.forward in inference, :252-280
    attn, _, comp = sa._build_attn_matrix(q, k, scale, valid, True, True)
    lg_soft = compress(lg.unsqueeze(-1), valid, pad_value=float("-inf")).squeeze(-1) if comp else lg
    w = sa._gated_softmax(attn, lg_soft, mode="seq", is_infer=True, is_compressed=comp)
    if comp:
        out = torch.matmul(w[..., :-1], compress(v, valid)) + w[..., -1:] * v
    else:
        out = w @ v
    return {"scale": scale, "q": q, "k": k, "v": v, "log_gate": lg, "out": out, "compressed": comp}


PREFILL_CASES = {
    # some gates zero everywhere: the reference's compressed path
    "dropped_fp32": dict(seed=31, b=2, H=3, L=150, D=64, p_zero=0.2),
    # padding only, row 0 fully kept: the dense path with -inf at the padding keys
    "padded_d32_fp32": dict(seed=32, b=2, H=2, L=130, D=32, p_zero=0.0, lengths=[130, 97]),
    # head_dim 128, every key kept
    "kept_d128_fp32": dict(seed=33, b=1, H=2, L=200, D=128, p_zero=0.0),
}


def main(only=None):
    for name, cfg in CASES.items():
        if only and name not in only:
            continue
        torch.save(run(**cfg), os.path.join(HERE, f"sattn_decode_{name}.pt"))
        print(name, "ok", flush=True)
    for name, cfg in PREFILL_CASES.items():
        if only and name not in only:
            continue
        rec = run_prefill(**cfg)
        torch.save(rec, os.path.join(HERE, f"sattn_prefill_{name}.pt"))
        print(name, "compressed" if rec["compressed"] else "dense", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
