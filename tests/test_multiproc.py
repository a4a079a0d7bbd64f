"""Multi-process host logic on CPU (gloo, world size 2): the bench's barrier and
max-over-ranks timing reduction, and the torchrun path of the reference arm (rank 0
prints the one JSON line, the other rank exits cleanly)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(world)
        slowest = bench.max_over_ranks(float(rank + 1) * 1.5, world)
        q.put((rank, slowest))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_barrier_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=5) for _ in range(world))
    assert got == [(0, 3.0), (1, 3.0)]


@pytest.mark.skipif(torch.cuda.is_available(), reason="CPU-only check of the gloo torchrun path")
def test_reference_arm_under_torchrun_gloo():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["h2d_bytes_per_step"] == 0


def _shard_worker(rank, world, port, q):
    """One gloo rank of a split SSD forward on the CPU: builds its own group slice and
    row slice of two small global problems from the shared seed, runs the oracle on
    them and gathers the outputs; rank 0 compares with the oracle on the whole problem."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import dataclasses
    import datetime

    import torch.distributed as dist

    from oracle import ssd_ref
    from selective_attention_b200 import sharding, workloads

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        res = {}
        c4 = dataclasses.replace(workloads.CONFIGS["c4"], dtype="f32", batch=2, seqlen=300, nheads=8, ngroups=4,
                                 headdim=32, dstate=16, chunk=64)
        c1 = dataclasses.replace(workloads.CONFIGS["c1"], dtype="f32", batch=4, seqlen=200, nheads=3, headdim=32,
                                 dstate=16, chunk=64)

        def run(inp, cfg):
            y, h = ssd_ref.ssd_scan_forward(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None,
                                            None, cfg.chunk)
            b, L, H, P = y.shape
            return ssd_ref.gate_epilogue(y, inp["u"], inp["D"], inp["z"]).reshape(b, L, H, P), h

        groups = sharding.group_range(rank, world, c4.ngroups)
        y, h = run(sharding.make_group_inputs(c4, 5, groups), c4)
        y_all, h_all = sharding.gather_heads(y, world, 2), sharding.gather_heads(h, world, 1)
        rows = sharding.row_range(rank, world, c1.batch)
        yr, hr = run(sharding.make_row_inputs(c1, 6, rows), c1)
        yr_all, hr_all = sharding.gather_rows(yr, world), sharding.gather_rows(hr, world)
        if rank == 0:
            y1, h1 = run(sharding.make_group_inputs(c4, 5, (0, c4.ngroups)), c4)
            res["groups"] = (sharding.compare(y_all, y1), sharding.compare(h_all, h1), groups, tuple(y_all.shape))
            y1, h1 = run(sharding.make_row_inputs(c1, 6, (0, c1.batch)), c1)
            res["rows"] = (sharding.compare(yr_all, y1), sharding.compare(hr_all, h1), rows, tuple(yr_all.shape))
        q.put((rank, res, groups, rows))
    finally:
        dist.destroy_process_group()


def test_group_and_row_split_gathers_to_the_whole_problem_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = {r: (res, g, rw) for r, res, g, rw in (q.get(timeout=5) for _ in range(world))}
    assert got[0][1] == (0, 2) and got[1][1] == (2, 4)
    assert got[0][2] == (0, 2) and got[1][2] == (2, 4)
    res = got[0][0]
    for key, shape in (("groups", (2, 300, 8, 32)), ("rows", (4, 200, 3, 32))):
        ycmp, hcmp, _, yshape = res[key]
        assert yshape == shape
        # slices computed alone equal the same slices of the whole problem: the oracle
        # is exact per (row, group), so the gathered result is bit-identical
        assert ycmp["bit_identical"], (key, ycmp)
        assert hcmp["bit_identical"], (key, hcmp)


def test_split_ranges_reject_uneven_splits():
    from selective_attention_b200 import sharding

    assert sharding.group_range(3, 8, 8) == (3, 4)
    assert sharding.row_range(1, 4, 8) == (2, 4)
    with pytest.raises(ValueError):
        sharding.group_range(0, 3, 8)
    with pytest.raises(ValueError):
        sharding.row_range(2, 2, 8)
