"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The reference publishes no dataset for this path; these stand in for it:
x ~ N(0,1); B, C ~ N(0,1)/sqrt(N); delta_raw ~ N(0,1) - 4 (dt = softplus(delta_raw));
A = -exp(U(log 1, log 16)); D ~ N(0,1) per channel (H*P,); z ~ N(0,1);
decode state ~ 0.1 N(0,1) fp32 and delta_bias = 0.1 N(0,1).
Tensors are drawn in fp32 in a fixed order (x, B, C, delta_raw, A, D, z, h_init,
delta_bias) from one ``torch.Generator`` on ``gen_device`` and then cast; CPU
generation gives the values parity tests use, GPU generation is used for the
full-size benchmark shapes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional

import torch

DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


@dataclass(frozen=True)
class SSDConfig:
    name: str
    dtype: str
    batch: int
    seqlen: int
    nheads: int
    headdim: int
    dstate: int
    ngroups: int
    chunk: int
    D: bool
    z: bool
    varlen: bool = False
    minlen: int = 128
    maxlen: int = 4096
    delta_bias: bool = False
    h_init: bool = False

    @property
    def tokens(self) -> int:
        return self.batch * self.seqlen


@dataclass(frozen=True)
class SSUConfig:
    name: str
    dtype: str
    batch: int
    nheads: int
    headdim: int
    dstate: int
    ngroups: int
    D: bool = True
    z: bool = True
    delta_bias: bool = True


CONFIGS = {
    # fp32 2x256, H4 P32 N16 G1 cs64, D, no z
    "c0": SSDConfig("c0", "f32", 2, 256, 4, 32, 16, 1, 64, D=True, z=False),
    # Mamba-2-130M shaped: bf16 8x2048, H24 P64 N128 G1 cs256, z-gate (+D)
    "c1": SSDConfig("c1", "bf16", 8, 2048, 24, 64, 128, 1, 256, D=True, z=True),
    # Mamba-2-2.7B shaped varlen: 32768 packed tokens, H80 P64 N128 G1 cs256, D + z
    "c2": SSDConfig("c2", "bf16", 1, 32768, 80, 64, 128, 1, 256, D=True, z=True, varlen=True),
    # long context sharded by heads: bf16 8x65536, H128 P64 N128 G8 cs256, D + z
    "c4": SSDConfig("c4", "bf16", 8, 65536, 128, 64, 128, 8, 256, D=True, z=True),
}
SSU_CONFIGS = {
    # decode: b256 H80 P64 N128 G1, fp32 state, bf16 x/B/C/z, dt_bias, D + z
    "c3": SSUConfig("c3", "bf16", 256, 80, 64, 128, 1),
}


def varlen_lengths(total: int, lo: int, hi: int, seed: int) -> list:
    """Integers U[lo, hi] drawn until the sum reaches ``total``; the last is truncated."""
    g = torch.Generator().manual_seed(seed + 7919)
    out = []
    s = 0
    while s < total:
        n = int(torch.randint(lo, hi + 1, (1,), generator=g).item())
        n = min(n, total - s)
        out.append(n)
        s += n
    return out


def make_ssd_inputs(cfg: SSDConfig, seed: int = 0, device="cpu", gen_device: Optional[str] = None,
                    **overrides) -> dict:
    """Inputs for ``SSDScanFn`` as a dict (``u, A, B, C, delta_raw, delta_bias, h_init,
    length, D, z, cu_seqlens, chunk_size``)."""
    cfg = replace(cfg, **overrides) if overrides else cfg
    gdev = gen_device or "cpu"
    g = torch.Generator(device=gdev).manual_seed(seed)
    b, L, H, P, N, G = cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, cfg.dstate, cfg.ngroups
    dt = DT[cfg.dtype]

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=gdev, dtype=torch.float32)

    x = randn(b, L, H, P)
    B = randn(b, L, G, N) / math.sqrt(N)
    C = randn(b, L, G, N) / math.sqrt(N)
    delta_raw = randn(b, L, H) - 4.0
    A = -torch.exp(torch.rand(H, generator=g, device=gdev) * math.log(16.0))
    D = randn(H * P) if cfg.D else None
    z = randn(b, L, H * P) if cfg.z else None
    h_init = 0.1 * randn(b, H, P, N) if cfg.h_init else None
    delta_bias = 0.1 * randn(H) if cfg.delta_bias else None
    cu = None
    if cfg.varlen:
        lens = varlen_lengths(cfg.tokens, cfg.minlen, cfg.maxlen, seed)
        cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int32), 0)
        if cfg.h_init:
            h_init = 0.1 * randn(len(lens), H, P, N)
    out = {
        "u": x.to(dt), "A": A, "B": B.to(dt), "C": C.to(dt),
        "delta_raw": delta_raw,  # fp32 (the configs keep dt in fp32)
        "delta_bias": delta_bias, "h_init": h_init, "length": None,
        "D": D, "z": None if z is None else z.to(dt), "cu_seqlens": cu, "chunk_size": cfg.chunk,
    }
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in out.items()}


def make_ssu_inputs(cfg: SSUConfig, seed: int = 0, device="cpu", gen_device: Optional[str] = None,
                    **overrides) -> dict:
    """Inputs for ``SSUFn`` (``u, A, B, C, delta_raw, delta_bias, h, D, z``)."""
    cfg = replace(cfg, **overrides) if overrides else cfg
    gdev = gen_device or "cpu"
    g = torch.Generator(device=gdev).manual_seed(seed)
    b, H, P, N, G = cfg.batch, cfg.nheads, cfg.headdim, cfg.dstate, cfg.ngroups
    dt = DT[cfg.dtype]

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=gdev, dtype=torch.float32)

    x = randn(b, H, P)
    B = randn(b, G, N) / math.sqrt(N)
    C = randn(b, G, N) / math.sqrt(N)
    delta_raw = randn(b, H) - 4.0
    A = -torch.exp(torch.rand(H, generator=g, device=gdev) * math.log(16.0))
    D = randn(H * P) if cfg.D else None
    z = randn(b, H * P) if cfg.z else None
    h = 0.1 * randn(b, H, P, N)
    delta_bias = 0.1 * randn(H) if cfg.delta_bias else None
    out = {"u": x.to(dt), "A": A, "B": B.to(dt), "C": C.to(dt), "delta_raw": delta_raw,
           "delta_bias": delta_bias, "h": h, "D": D, "z": None if z is None else z.to(dt)}
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in out.items()}


def ssd_algorithmic_bytes(cfg: SSDConfig, y_bytes: Optional[int] = None, nseq: Optional[int] = None) -> int:
    """Minimum HBM bytes of one fused SSD forward: read x, z, B, C, dt (+ h_init), write y
    and h_last. ``T*H*P*(s_x + s_z + s_y) + 2*T*G*N*s_x + s_dt*T*H + 4*rows*H*P*N``."""
    T = cfg.tokens
    sx = torch.finfo(DT[cfg.dtype]).bits // 8
    sy = y_bytes if y_bytes is not None else (sx if (cfg.D or cfg.z) else 4)
    sz = sx if cfg.z else 0
    rows = nseq if nseq is not None else cfg.batch
    total = T * cfg.nheads * cfg.headdim * (sx + sz + sy)
    total += 2 * T * cfg.ngroups * cfg.dstate * sx
    total += 4 * T * cfg.nheads
    total += 4 * rows * cfg.nheads * cfg.headdim * cfg.dstate
    if cfg.h_init:
        total += 4 * rows * cfg.nheads * cfg.headdim * cfg.dstate
    return total


def ssd_flops(cfg: SSDConfig) -> int:
    """``T * (4*H*P*N + G*cs*N + H*cs*P)`` (causal halves counted once)."""
    T = cfg.tokens
    return T * (4 * cfg.nheads * cfg.headdim * cfg.dstate + cfg.ngroups * cfg.chunk * cfg.dstate
                + cfg.nheads * cfg.chunk * cfg.headdim)


def ssu_algorithmic_bytes(cfg: SSUConfig, state_bytes: int = 4) -> int:
    """State read + write, x, y (and z), B, C, dt per decode step."""
    b, H, P, N, G = cfg.batch, cfg.nheads, cfg.headdim, cfg.dstate, cfg.ngroups
    sx = torch.finfo(DT[cfg.dtype]).bits // 8
    total = 2 * state_bytes * b * H * P * N
    total += b * H * P * (sx + sx + (sx if cfg.z else 0))
    total += 2 * b * G * N * sx + 4 * b * H
    return total
