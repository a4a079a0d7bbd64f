"""Generate the SSD backward golden vectors from the reference implementation.

Runs nmquan1503/selective-attention's own backward (``SSDScanFn.backward`` ->
``triton_kernels/ssd_scan/backward.py:467 ssd_scan_backward``, nine Triton kernels)
on CPU under the Triton interpreter (``oracle/ref_interp.load_backward``) through
its public autograd boundary, on seeded inputs, and saves inputs and gradients as
``ssd_bwd_<case>.pt``. Needs the reference checkout; run from the repository root:
``python tests/golden/make_golden_bwd.py``.

bf16 cases: the reference cannot take bf16 operands, so inputs are drawn in fp32,
rounded to bf16, stored as bf16 and fed to the reference upcast to fp32.
"""
from __future__ import annotations

import math
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_interp  # noqa: E402  (sets TRITON_INTERPRET before triton loads)

REF = ref_interp.load_backward()

import torch  # noqa: E402

INF = float("inf")


def gen(seed, b, L, H, P, N, G, *, dtype=torch.float32, h_init=False, delta_bias=False, dr_shift=-4.0,
        dr_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    u = rn(b, L, H, P)
    B = rn(b, L, G, N) / math.sqrt(N)
    C = rn(b, L, G, N) / math.sqrt(N)
    dr = dr_scale * rn(b, L, H) + dr_shift
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    out = {"u": u.to(dtype), "A": A, "B": B.to(dtype), "C": C.to(dtype), "delta_raw": dr}
    out["h_init"] = 0.1 * rn(b, H, P, N) if h_init else None
    out["delta_bias"] = 0.1 * rn(H) if delta_bias else None
    out["y_grad"] = rn(b, L, H, P)
    out["h_last_grad"] = 0.1 * rn(b, H, P, N)
    return out


def run_bwd(inp, length, chunk_size, use_sp=True, limit=(0.0, INF)):
    names = ("u", "A", "B", "C", "delta_raw", "delta_bias", "h_init")
    leaves = {k: (None if inp[k] is None else inp[k].float().clone().requires_grad_(True)) for k in names}
    y, h_last = REF["SSDScanFn"].apply(leaves["u"], leaves["A"], leaves["B"], leaves["C"], leaves["delta_raw"],
                                       leaves["delta_bias"], leaves["h_init"], length, chunk_size, use_sp, limit,
                                       True)
    torch.autograd.backward([y, h_last], [inp["y_grad"], inp["h_last_grad"]])
    return {k + "_grad": (None if leaves[k] is None else leaves[k].grad.detach()) for k in names}


CASES = {
    # c0 head shape (P32 N16 cs64), h_init and dt bias, full rows
    "c0_fp32": dict(seed=11, b=2, L=256, H=4, P=32, N=16, G=1, cs=64, h_init=True, delta_bias=True),
    # partial last chunk, per-row length (one row ends inside a chunk, one on a boundary), groups
    "ragged_fp32": dict(seed=12, b=3, L=200, H=4, P=32, N=16, G=2, cs=64, length=[200, 150, 64],
                        h_init=True, delta_bias=True),
    # dt clamped on both sides of delta_limit
    "clamp_fp32": dict(seed=13, b=1, L=128, H=2, P=32, N=16, G=1, cs=64, limit=(0.01, 0.05), delta_bias=True),
    # no softplus: dt = clamp(delta_raw + bias, 0, inf), negative values clamp to 0
    "nosoftplus_fp32": dict(seed=14, b=1, L=128, H=2, P=32, N=16, G=1, cs=64, use_sp=False, dr_shift=0.03,
                            dr_scale=0.05, delta_bias=True),
    # the production head shape (P64 N128 cs256), bf16-rounded inputs
    "p64_bf16": dict(seed=15, b=1, L=512, H=2, P=64, N=128, G=1, cs=256, dtype=torch.bfloat16),
    # production head shape, two groups, a ragged row, h_init
    "p64_groups_ragged_bf16": dict(seed=16, b=2, L=384, H=4, P=64, N=128, G=2, cs=256, length=[384, 300],
                                   h_init=True, delta_bias=True, dtype=torch.bfloat16),
}


def main(only=None):
    for name, cfg in CASES.items():
        if only and name not in only:
            continue
        t0 = time.time()
        cfg = dict(cfg)
        seed, b, L, H, P, N, G, cs = (cfg.pop(k) for k in ("seed", "b", "L", "H", "P", "N", "G", "cs"))
        length = torch.tensor(cfg.pop("length", [L] * b), dtype=torch.long)
        use_sp = cfg.pop("use_sp", True)
        limit = cfg.pop("limit", (0.0, INF))
        inp = gen(seed, b, L, H, P, N, G, **cfg)
        grads = run_bwd(inp, length, cs, use_sp, limit)
        rec = dict(inp, length=length, chunk_size=cs, use_delta_softplus=use_sp, delta_limit=limit, **grads)
        torch.save(rec, os.path.join(HERE, f"ssd_bwd_{name}.pt"))
        print(f"{name}: {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
