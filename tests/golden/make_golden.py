"""Generate the golden vectors in this directory from the reference implementation.

Runs nmquan1503/selective-attention's own Triton kernels on CPU under the Triton
interpreter (see ``oracle/ref_interp.py``) through its public boundary
(``SSDScanFn.apply``, ``SSUFn.forward``) and its stage functions in
``triton_kernels/ssd_scan/forward.py``, on seeded inputs, and saves inputs and
outputs as ``<case>.pt``. Needs the reference checkout; run from the repository
root:  ``python tests/golden/make_golden.py``.

bf16 cases: the reference SSD cannot take bf16 operands (its ``tl.dot`` mixes bf16
with fp32 and Triton rejects that), so inputs are drawn in fp32, rounded to bf16,
stored as bf16 and fed to the reference upcast to fp32.
"""
from __future__ import annotations

import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_interp  # noqa: E402  (sets TRITON_INTERPRET before triton loads)

REF = ref_interp.load()

import torch  # noqa: E402

INF = float("inf")


def gen(seed, b, L, H, P, N, G, *, dtype=torch.float32, D=True, z=False, h_init=False, delta_bias=False):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    u = rn(b, L, H, P)
    B = rn(b, L, G, N) / math.sqrt(N)
    C = rn(b, L, G, N) / math.sqrt(N)
    dr = rn(b, L, H) - 4.0
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    out = {"u": u.to(dtype), "A": A, "B": B.to(dtype), "C": C.to(dtype), "delta_raw": dr}
    out["D"] = rn(H * P) if D else None
    out["z"] = rn(b, L, H * P).to(dtype) if z else None
    out["h_init"] = 0.1 * rn(b, H, P, N) if h_init else None
    out["delta_bias"] = 0.1 * rn(H) if delta_bias else None
    return out


def f32(t):
    return None if t is None else t.float()


def run_ssd(inp, length, chunk_size, use_sp=True, limit=(0.0, INF), stages=False):
    u, A, B, C, dr = f32(inp["u"]), inp["A"], f32(inp["B"]), f32(inp["C"]), inp["delta_raw"]
    db, hi = inp["delta_bias"], inp["h_init"]
    y, h_last = REF["SSDScanFn"].apply(u, A, B, C, dr, db, hi, length, chunk_size, use_sp, limit, True)
    res = {"y": y.detach(), "h_last": h_last.detach()}
    if stages:
        b, L, H, P = u.shape
        nc = math.ceil(L / chunk_size)
        cum, dt = REF["chunk_cumsum_forward"](A, dr, db, length, chunk_size, use_sp, limit)
        states = REF["chunk_state_forward"](u, B, dt, cum)
        res["cum"], res["dt"], res["states"] = cum.clone(), dt.clone(), states.clone()
        prev, _ = REF["state_passing_forward"](states.view(b, nc, H, -1),
                                               None if hi is None else hi.view(b, H, -1), cum[:, :, :, -1])
        res["prev"] = prev.view(b, nc, H, P, -1).clone()
        res["CB"] = REF["bmm_chunk_forward"](B, C, chunk_size, True).clone()
        res["y_stage"] = REF["chunk_scan_forward"](u, dt, cum, C, res["prev"], res["CB"]).clone()
    return res


def save(name, **kw):
    path = os.path.join(HERE, f"{name}.pt")
    torch.save(kw, path)
    print(f"{name}: {os.path.getsize(path) / 1024:.0f} KB")


def main():
    # c0: fp32 2x256, H4 P32 N16 G1 cs64, D (benchmark config c0), with every stage output.
    inp = gen(0, 2, 256, 4, 32, 16, 1)
    length = torch.tensor([256, 256])
    out = run_ssd(inp, length, 64, stages=True)
    save("ssd_c0_fp32", inputs=inp, length=length, chunk_size=64, use_sp=True, limit=(0.0, INF), **out)

    # ragged: partial last chunk, length < L, 2 groups, h_init, delta_bias, both clamps active
    inp = gen(1, 3, 200, 4, 32, 16, 2, h_init=True, delta_bias=True)
    length = torch.tensor([200, 150, 64])
    limit = (0.01, 0.1)
    out = run_ssd(inp, length, 64, limit=limit, stages=True)
    save("ssd_ragged_fp32", inputs=inp, length=length, chunk_size=64, use_sp=True, limit=limit, **out)

    # softplus threshold: raw values around 20 pass through unchanged above it
    inp = gen(2, 2, 96, 2, 16, 8, 1, D=False)
    inp["delta_raw"][0, 3] = 19.5
    inp["delta_raw"][0, 40] = 20.0
    inp["delta_raw"][1, 7] = 20.5
    inp["delta_raw"][1, 70] = 30.0
    length = torch.tensor([96, 90])
    out = run_ssd(inp, length, 32)
    save("ssd_threshold_fp32", inputs=inp, length=length, chunk_size=32, use_sp=True, limit=(0.0, INF), **out)

    # no softplus: dt = clamp(delta_raw) with positive raw values
    inp = gen(3, 2, 128, 2, 16, 8, 1, D=False)
    inp["delta_raw"] = inp["delta_raw"].abs() * 0.02
    length = torch.tensor([128, 100])
    out = run_ssd(inp, length, 32, use_sp=False)
    save("ssd_nosoftplus_fp32", inputs=inp, length=length, chunk_size=32, use_sp=False, limit=(0.0, INF), **out)

    # bf16, c1-shaped heads (P64 N128 cs256), 2 chunks, ragged length, D + z epilogue checked in tests
    inp = gen(4, 2, 512, 2, 64, 128, 1, dtype=torch.bfloat16, z=True)
    length = torch.tensor([512, 300])
    out = run_ssd(inp, length, 256)
    save("ssd_bf16_c1slice", inputs=inp, length=length, chunk_size=256, use_sp=True, limit=(0.0, INF), **out)

    # bf16, c4-shaped groups (G2, 2 heads per group), partial second chunk, h_init, delta_bias
    inp = gen(5, 1, 384, 4, 64, 128, 2, dtype=torch.bfloat16, z=True, h_init=True, delta_bias=True)
    length = torch.tensor([384])
    out = run_ssd(inp, length, 256)
    save("ssd_bf16_groups", inputs=inp, length=length, chunk_size=256, use_sp=True, limit=(0.0, INF), **out)

    # packed varlen (c2-shaped heads): 3 sequences 300 / 77 / 135; reference = padded rows + length
    lens = [300, 77, 135]
    T = sum(lens)
    inp = gen(6, 1, T, 2, 64, 128, 1, dtype=torch.bfloat16, z=True)
    cu = torch.tensor([0, 300, 377, 512], dtype=torch.int32)
    maxlen = max(lens)

    def pad(x):
        o = torch.zeros((len(lens), maxlen) + tuple(x.shape[2:]), dtype=torch.float32)
        for i, n in enumerate(lens):
            o[i, :n] = x[0, cu[i]:cu[i] + n].float()
        return o

    pinp = {"u": pad(inp["u"]), "A": inp["A"], "B": pad(inp["B"]), "C": pad(inp["C"]),
            "delta_raw": pad(inp["delta_raw"]), "delta_bias": None, "h_init": None}
    pout = run_ssd(pinp, torch.tensor(lens), 256)
    y_packed = torch.cat([pout["y"][i, :n] for i, n in enumerate(lens)], 0)[None]
    save("ssd_varlen_bf16", inputs=inp, cu_seqlens=cu, chunk_size=256, use_sp=True, limit=(0.0, INF),
         y=y_packed, h_last=pout["h_last"])

    # SSU bf16 x/B/C with fp32 state and delta_bias (c3-shaped heads)
    g = torch.Generator().manual_seed(7)
    b, H, P, N, G = 2, 4, 64, 128, 1
    rn = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    sinp = {"u": rn(b, H, P).bfloat16(), "B": (rn(b, G, N) / math.sqrt(N)).bfloat16(),
            "C": (rn(b, G, N) / math.sqrt(N)).bfloat16(), "delta_raw": rn(b, H) - 4.0,
            "A": -torch.exp(torch.rand(H, generator=g) * math.log(16.0)), "delta_bias": 0.1 * rn(H),
            "h": 0.1 * rn(b, H, P, N), "D": rn(H * P), "z": rn(b, H * P).bfloat16()}
    h = sinp["h"].clone()
    y, h_new = REF["SSUFn"].forward(sinp["u"], sinp["A"], sinp["B"], sinp["C"], sinp["delta_raw"],
                                    sinp["delta_bias"], h)
    save("ssu_bf16", inputs=sinp, y=y.clone(), h_new=h_new.clone())

    # SSU fp32, 2 groups, no bias, clamp active
    g = torch.Generator().manual_seed(8)
    b, H, P, N, G = 3, 4, 32, 16, 2
    sinp = {"u": rn(b, H, P), "B": rn(b, G, N) / math.sqrt(N), "C": rn(b, G, N) / math.sqrt(N),
            "delta_raw": rn(b, H) - 3.0, "A": -torch.exp(torch.rand(H, generator=g) * math.log(16.0)),
            "delta_bias": None, "h": 0.1 * rn(b, H, P, N), "D": None, "z": None}
    h = sinp["h"].clone()
    limit = (0.0, 0.05)
    y, h_new = REF["SSUFn"].forward(sinp["u"], sinp["A"], sinp["B"], sinp["C"], sinp["delta_raw"], None, h,
                                    True, limit)
    save("ssu_fp32_groups", inputs=sinp, limit=limit, y=y.clone(), h_new=h_new.clone())


if __name__ == "__main__":
    main()
