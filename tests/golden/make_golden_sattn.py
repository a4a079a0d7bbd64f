"""Generate the selective-attention decode-step golden vectors from the reference.

Uses nmquan1503/selective-attention's own code on CPU: ``SelectiveAttnCache``
(``inference/selective_attn_cache.py``: ``build_kv`` after a prefill, ``update_kv`` per
step), ``_reset_cache`` (``modules/selective_attention.py:11-25``, the buffer growth and
compression ``SelectiveMHA.step`` runs every ``cache_update_interval`` steps) and
``_gated_softmax`` in pos mode (``:126-128``), with the attention lines of
``SelectiveMHA.step`` (``:399-405``) around them. Saves the cache after the reset, every
step's inputs (``q_rot, k_rot, v, log_gate``) and outputs, and the final cache as
``sattn_decode_<case>.pt``. Needs the reference checkout; run from the repository root:
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
    else:  # SelectiveMHA.step's first allocation (:363-366); zero-filled here for determinism
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
        # SelectiveMHA.step, modules/selective_attention.py:399-405
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


def main(only=None):
    for name, cfg in CASES.items():
        if only and name not in only:
            continue
        torch.save(run(**cfg), os.path.join(HERE, f"sattn_decode_{name}.pt"))
        print(name, "ok", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
