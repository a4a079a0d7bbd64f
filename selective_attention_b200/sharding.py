"""Splitting one SSD forward across the GPUs of a box (one process per GPU).

The scan has no exchange between batch rows or between head groups: each (row, group)
slice is a complete problem of its own (its heads read only their group's B and C,
``forward_kernel.py:107-185,350-455``). So a global problem is split with no
collective on the data path:

- ``group_range``: by whole head groups when the groups divide among the ranks (a rank
  takes groups ``[r*G/W, (r+1)*G/W)``, i.e. their heads, B / C columns, A, D and z
  columns): the strong-scaling split of one long-context batch;
- ``row_range``: by batch rows (a rank takes rows ``[r*b/W, (r+1)*b/W)``): the
  weak-scaling split when every rank gets a fixed share of a global batch.

Inputs are drawn per group (or per row) from generators seeded by the shared seed and
the group (row) index, so any rank builds exactly its own slice of the one global
problem without the others, and the slices agree with a one-GPU build of the whole
problem. ``gather_heads`` / ``gather_rows`` collect the ranks' outputs (NCCL
``all_gather`` on GPUs, gloo on CPU), which the benchmark uses outside its timed region
to check the split against a one-GPU run.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Dict, List, Optional, Tuple

import torch

from . import workloads

_MIX = 1_000_003  # keeps the per-group / per-row seeds of different base seeds apart


def group_range(rank: int, world: int, ngroups: int) -> Tuple[int, int]:
    """Head groups ``[g0, g1)`` of ``rank``; the groups must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if ngroups % world != 0:
        raise ValueError(f"{ngroups} head groups do not split evenly over {world} ranks")
    per = ngroups // world
    return rank * per, (rank + 1) * per


def row_range(rank: int, world: int, batch: int) -> Tuple[int, int]:
    """Batch rows ``[r0, r1)`` of ``rank``; the rows must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if batch % world != 0:
        raise ValueError(f"{batch} rows do not split evenly over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def _alloc_like(cfg, b, L, H, G, device, dt):
    P, N = cfg.headdim, cfg.dstate
    return {
        "u": torch.empty(b, L, H, P, dtype=dt, device=device),
        "B": torch.empty(b, L, G, N, dtype=dt, device=device),
        "C": torch.empty(b, L, G, N, dtype=dt, device=device),
        "delta_raw": torch.empty(b, L, H, dtype=torch.float32, device=device),
        "A": torch.empty(H, dtype=torch.float32, device=device),
        "D": torch.empty(H * P, dtype=torch.float32, device=device) if cfg.D else None,
        "z": torch.empty(b, L, H * P, dtype=dt, device=device) if cfg.z else None,
    }


def make_group_inputs(cfg: workloads.SSDConfig, seed: int, groups: Tuple[int, int], device="cpu",
                      gen_device: Optional[str] = None) -> Dict[str, torch.Tensor]:
    """Inputs of head groups ``[g0, g1)`` of the global problem ``cfg`` (padded rows,
    no h_init / delta_bias): group g's tensors come from ``make_ssd_inputs`` with one
    group of ``H/G`` heads and seed ``seed * 1000003 + g``."""
    if cfg.varlen or cfg.h_init or cfg.delta_bias:
        raise ValueError("group sharding covers padded batches without h_init / delta_bias")
    g0, g1 = groups
    hpg = cfg.nheads // cfg.ngroups
    Gl, Hl, P = g1 - g0, (g1 - g0) * hpg, cfg.headdim
    out = _alloc_like(cfg, cfg.batch, cfg.seqlen, Hl, Gl, device, workloads.DT[cfg.dtype])
    sub = replace(cfg, nheads=hpg, ngroups=1)
    for i, g in enumerate(range(g0, g1)):
        part = workloads.make_ssd_inputs(sub, seed=seed * _MIX + g, device=device, gen_device=gen_device)
        hs = slice(i * hpg, (i + 1) * hpg)
        out["u"][:, :, hs] = part["u"]
        out["B"][:, :, i:i + 1] = part["B"]
        out["C"][:, :, i:i + 1] = part["C"]
        out["delta_raw"][:, :, hs] = part["delta_raw"]
        out["A"][hs] = part["A"]
        if cfg.D:
            out["D"][i * hpg * P:(i + 1) * hpg * P] = part["D"]
        if cfg.z:
            out["z"][:, :, i * hpg * P:(i + 1) * hpg * P] = part["z"]
        del part
    out.update(delta_bias=None, h_init=None, length=None, cu_seqlens=None, chunk_size=cfg.chunk)
    return out


def make_row_inputs(cfg: workloads.SSDConfig, seed: int, rows: Tuple[int, int], device="cpu",
                    gen_device: Optional[str] = None) -> Dict[str, torch.Tensor]:
    """Inputs of batch rows ``[r0, r1)`` of the global problem ``cfg`` (padded rows):
    row i's x, B, C, delta_raw, z come from ``make_ssd_inputs`` with batch 1 and seed
    ``seed * 1000003 + i``; the per-head parameters A and D, shared by all rows, from
    seed ``seed * 1000003 - 1``."""
    if cfg.varlen or cfg.h_init or cfg.delta_bias:
        raise ValueError("row sharding covers padded batches without h_init / delta_bias")
    r0, r1 = rows
    one = replace(cfg, batch=1)
    out = _alloc_like(cfg, r1 - r0, cfg.seqlen, cfg.nheads, cfg.ngroups, device, workloads.DT[cfg.dtype])
    params = workloads.make_ssd_inputs(replace(one, seqlen=1), seed=seed * _MIX - 1, device=device,
                                       gen_device=gen_device)
    out["A"].copy_(params["A"])
    if cfg.D:
        out["D"].copy_(params["D"])
    for i, r in enumerate(range(r0, r1)):
        part = workloads.make_ssd_inputs(one, seed=seed * _MIX + r, device=device, gen_device=gen_device)
        for k in ("u", "B", "C", "delta_raw") + (("z",) if cfg.z else ()):
            out[k][i:i + 1] = part[k]
        del part
    out.update(delta_bias=None, h_init=None, length=None, cu_seqlens=None, chunk_size=cfg.chunk)
    return out


def _all_gather(t: torch.Tensor, world: int) -> List[torch.Tensor]:
    import torch.distributed as dist

    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous())
    return parts


def gather_heads(local: torch.Tensor, world: int, head_dim: int) -> torch.Tensor:
    """All ranks' head slices of one output (``y`` (b, L, Hl, P) with ``head_dim=2``,
    ``h_last`` (b, Hl, P, N) with ``head_dim=1``), concatenated in rank order along the
    head axis: the global tensor of a group split. Every rank must call it."""
    if world == 1:
        return local
    return torch.cat(_all_gather(local, world), dim=head_dim)


def gather_rows(local: torch.Tensor, world: int) -> torch.Tensor:
    """All ranks' batch rows of one output, in rank order (dimension 0)."""
    if world == 1:
        return local
    return torch.cat(_all_gather(local, world), dim=0)


def compare(got: torch.Tensor, want: torch.Tensor) -> Dict[str, float]:
    """Bitwise agreement and the largest difference of two outputs of the same kernels."""
    same = bool(torch.equal(got, want))
    diff = 0.0 if same else float((got.float() - want.float()).abs().max())
    return {"bit_identical": same, "max_abs_diff": diff}

