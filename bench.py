#!/usr/bin/env python
"""Benchmark of the SSD chunked-scan forward (and the decode state update) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1|c2|c4]

One JSON line on stdout (rank 0). A "step" is one SSD forward over one batch of
the workload (default: benchmark config c1, 8 x 2048 tokens, H24 P64 N128 cs256,
bf16 with D + z).

Multi-GPU (torchrun, one process per GPU; the scan has no cross-row or cross-group
exchange, so nothing crosses NVLink on the data path):
- headline: one global batch of ``8 N`` rows split by batch rows, 8 rows per rank
  (weak scaling; at N = 1 it is config c1 itself); ``value`` = all ranks' tokens / the
  slowest rank's device time. After the timed loop the ranks' ``y`` / ``h_last`` are
  gathered over NCCL and rank 0 checks them against its own run of each rank's rows
  (``verify``);
- ``c4``: config c4 (8 x 65536, H128 over G8) as ONE global problem split by whole
  head groups over the N ranks (strong scaling), tokens/s of that problem from the
  slowest rank, and with N > 1 an NCCL gather of the outputs checked against rank 0's
  one-GPU run of the whole problem. At N = 1 the line also carries c2, the c1 shape in
  fp32 (the reference's own precision), the decode step and the other rows' kernels.

Timing: CUDA events on the launching stream around each step, L2 flushed
(256 MiB write) between steps outside the events, barrier + synchronize on both
sides of the timed loop, max over ranks. ``e2e`` repeats the measurement through
the public API with pinned host inputs copied in and ``y``/``h_last`` copied out
inside the timed region: ``HostStreamScan`` (row slices whose copies overlap the
scan) for padded batches, ``SSDScanFn`` with explicit copies for packed ones. ``--impl reference`` times the CPU
restatement of the reference's five stages (``oracle/``) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

INF = float("inf")
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2", "c4"], default="c1")
    ap.add_argument("--kernel-impl", choices=["auto", "tc", "tc_staged", "simt"], default="auto")
    ap.add_argument("--no-ssu", action="store_true", help="skip the decode (config 3) measurement")
    ap.add_argument("--no-front", action="store_true", help="skip the prefill front-end (conv) measurement")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-bwd", action="store_true", help="skip the SSD backward measurement")
    ap.add_argument("--no-sattn", action="store_true", help="skip the selective-attention decode measurement")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-c4 (head-group split) measurement")
    ap.add_argument("--no-extra", action="store_true", help="skip the one-GPU c2 and fp32 measurements")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's own Triton SSD on the GPU (secondary comparison)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    return ap.parse_args()


# ---------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() and args.impl == "ours" else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed loop runs."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            pr = torch.cuda.get_device_properties(device_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", bus], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi unavailable"}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                rows.append((ts, float(parts[1]), float(parts[2]), parts[4:8]))
            except ValueError:
                continue
        window = [r for r in rows if self.t0 is not None and self.t0 - 1 <= r[0] <= (self.t1 or r[0]) + 1] or rows
        if not window:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({self.REASONS[i] for r in window for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in window), "sm_max_mhz": max(r[2] for r in window),
                "reasons": reasons, "samples": len(window)}


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_baseline(cfg, seconds: float, max_steps=None):
    """Time the fp32 CPU restatement of the reference's five stages (oracle/ssd_ref.py)
    on one batch row of the workload, repeated until ``seconds`` of work; returns
    tokens/s with all host threads."""
    from oracle import ssd_ref
    from selective_attention_b200 import workloads

    torch.set_num_threads(os.cpu_count() or 1)
    rows = 1
    seqlen = cfg.seqlen if not cfg.varlen else 4096
    inp = workloads.make_ssd_inputs(cfg, seed=1, batch=rows, seqlen=seqlen, varlen=False)
    f = lambda t: None if t is None else t.float()  # noqa: E731

    def step():
        y, h = ssd_ref.ssd_scan_forward(f(inp["u"]), inp["A"], f(inp["B"]), f(inp["C"]), inp["delta_raw"], None,
                                        None, None, cfg.chunk)
        ssd_ref.gate_epilogue(y, inp["u"], inp["D"], inp["z"])

    step()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if (max_steps and n >= max_steps) or (not max_steps and el >= seconds):
            break
    tok = n * rows * seqlen
    return {"value": tok / el, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} x ({rows} row x {seqlen} tokens, H{cfg.nheads} P{cfg.headdim} N{cfg.dstate} "
                      f"cs{cfg.chunk}) fp32 oracle stage-by-stage restatement, {el:.1f} s",
            "cpu": _cpu_model()}


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference_arm(args, rank, world):
    from selective_attention_b200 import workloads

    cfg = workloads.CONFIGS[args.config]
    if rank != 0:
        return
    # Size the per-step sample so W + K steps fit in about two minutes.
    from oracle import ssd_ref  # noqa: F401  (import cost outside the timing)

    torch.set_num_threads(os.cpu_count() or 1)
    probe = cpu_baseline(cfg, seconds=0.0, max_steps=1)
    per_step_tokens_s = probe["value"]
    seqlen = cfg.seqlen if not cfg.varlen else 4096
    t_row = seqlen / per_step_tokens_s
    budget = 120.0 / max(1, args.steps + args.warmup)
    heads = max(1, min(cfg.nheads, int(cfg.nheads * budget / max(t_row, 1e-9))))
    sub = workloads.SSDConfig(**{**cfg.__dict__, "nheads": heads, "ngroups": 1 if cfg.ngroups < 2 else
                                 max(1, min(cfg.ngroups, heads // max(1, cfg.nheads // cfg.ngroups)))})
    res_w = cpu_baseline(sub, seconds=0.0, max_steps=max(1, args.warmup))
    del res_w
    t0 = time.perf_counter()
    res = cpu_baseline(sub, seconds=0.0, max_steps=max(1, args.steps))
    el = time.perf_counter() - t0
    scale = heads / cfg.nheads  # a sampled token carries heads/H of a full token's work
    value = res["value"] * scale
    line = {
        "impl": "reference", "metric": "SSD chunked-scan fwd tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.name} sampled on host cores", "heads_per_sample": heads},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": res["cores"], "kind": "port",
                         "sample": res["sample"] + f"; scaled by {heads}/{cfg.nheads} heads",
                         "cpu": res.get("cpu")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def main():
    args = parse()
    rank, world, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference_arm(args, rank, world)
            return
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def time_steps(fn, steps, flush_buf, stream):
    """Sum of per-step CUDA-event durations (ms); L2 flushed before each step, untimed."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s, e in evs:
        flush_buf.fill_(1)
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def _peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


class SSDRun:
    """One SSD forward problem resident on the device, its outputs and workspace, and a
    ``step`` that runs ``kernels.ssd_scan_forward`` on it (the C-ABI ``ssd_scan_fwd``)."""

    def __init__(self, cfg, inp, kernel_impl, dev):
        from selective_attention_b200 import kernels

        self.cfg, self.inp, self.dev = cfg, inp, dev
        u = inp["u"]
        b, L, H, P = u.shape
        G, N = inp["B"].shape[2], inp["B"].shape[3]
        self.shape = (b, L, H, P, N, G)
        cu = inp["cu_seqlens"]
        self.nseq = None if cu is None else cu.numel() - 1
        self.y = torch.empty(b, L, H, P, dtype=u.dtype, device=dev)
        self.h_last = torch.empty(self.nseq or b, H, P, N, dtype=torch.float32, device=dev)
        p, self._keep, _ = kernels.ssd_scan_params(u, inp["A"], inp["B"], inp["C"], inp["delta_raw"], None, None,
                                                   None, cfg.chunk, True, (0.0, INF), inp["D"], inp["z"], cu,
                                                   kernel_impl)
        self.ws = torch.empty(kernels.workspace_size(p), dtype=torch.uint8, device=dev)
        self.tc = kernels.uses_tensor_cores(p)
        self.path = kernels.scan_path(p)
        self.kernel_impl = kernel_impl
        self.launches = {"tc_fused": 2, "tc_staged": 3, "simt": 5, "tc_split": 5}[self.path] + (1 if cu is not None else 0)

    def step(self, events=None):
        from selective_attention_b200 import kernels

        i = self.inp
        kernels.ssd_scan_forward(i["u"], i["A"], i["B"], i["C"], i["delta_raw"], None, None, None, self.cfg.chunk,
                                 True, (0.0, INF), True, i["D"], i["z"], i["cu_seqlens"], self.kernel_impl,
                                 out=(self.y, self.h_last), workspace=self.ws, events=events)


def measure_ssd(run, args, world, flush, hbm_peak, peak_src, global_tokens, steps, clocks=None):
    """Device time of ``steps`` SSD forwards (L2 flushed between them, barrier and
    synchronize around the loop, max over ranks) and the per-stage split of a second
    pass, with the dominant kernel's roofline. ``value`` = ``global_tokens`` / step time."""
    import selective_attention_b200 as sab

    dev, stream = run.dev, torch.cuda.current_stream(run.dev)
    for _ in range(max(3, args.warmup)):
        run.step()
    torch.cuda.synchronize()
    sab.check_device_error(dev)
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_start()
    per_step = time_steps(run.step, steps, flush, stream)
    torch.cuda.synchronize()
    barrier(world)
    if clocks is not None:
        clocks.mark_end()
    ms_total = max_over_ranks(sum(per_step), world)
    ms_step = ms_total / steps

    stage_ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in stage_ev:
        e.record(stream)  # materialise the handles
    handles = [e.cuda_event for e in stage_ev]
    n_stage = min(steps, 50)
    st = []
    for _ in range(n_stage):
        flush.fill_(1)
        run.step(events=handles)
        torch.cuda.synchronize()
        st.append([stage_ev[j].elapsed_time(stage_ev[j + 1]) for j in range(5)])
    stage_ms = [statistics.median(r[j] for r in st) for j in range(5)]
    sab.check_device_error(dev)

    cfg, path, nseq = run.cfg, run.path, run.nseq
    tc = path in ("tc_fused", "tc_staged")  # the 16-bit chain: cumsum and bmm fused into neighbours
    b, L, H, P, N, G = run.shape
    T = b * L
    sx = run.inp["u"].element_size()
    cu = run.inp["cu_seqlens"]
    nck = (T + cfg.chunk - 1) // cfg.chunk + (nseq or 0) if cu is not None else b * math.ceil(L / cfg.chunk)
    s_prev = 2 if tc else 4
    # algorithmic bytes per launch of each stage (fp32 intermediates on the CUDA-core chain)
    scan_bytes = (T * H * P * (sx + sx + run.y.element_size()) + 2 * T * G * N * sx + 8 * T * H
                  + s_prev * nck * H * P * N)
    state_bytes = T * H * P * sx + T * G * N * sx + 8 * T * H + 4 * nck * H * P * N
    pass_bytes = 4 * nck * H * P * N + s_prev * nck * H * P * N + 4 * (nseq or b) * H * P * N + 4 * nck * H
    cums_bytes = 4 * T * H + 8 * nck * H * cfg.chunk
    # fused chunk_state + state_passing: x, B, raw dt in; dt, cum, prev16, h_last out
    sp_bytes = (T * H * P * sx + T * G * N * sx + 4 * T * H + 8 * nck * H * cfg.chunk + 2 * nck * H * P * N
                + 4 * (nseq or b) * H * P * N)
    names = ["chunk_cumsum", "chunk_state", "state_passing", "bmm_chunk", "chunk_scan"]
    bytes_ = [cums_bytes, state_bytes, pass_bytes, 0, scan_bytes]
    if path == "tc_fused":
        names[2] = "chunk_state+state_passing"
        bytes_[2] = sp_bytes
    stages = {}
    for n_, ms_, by in zip(names, stage_ms, bytes_):
        if tc and n_ in ("bmm_chunk", "chunk_cumsum"):
            continue  # fused: cumsum into chunk_state, bmm into chunk_scan
        if path == "tc_fused" and n_ == "chunk_state":
            continue  # fused into the chain kernel timed as stage [2, 3)
        if tc and n_ == "chunk_state":
            by += cums_bytes
        gbs = by / (ms_ / 1e3) / 1e9 if ms_ > 0 else None
        stages[n_] = {"us": ms_ * 1e3, "alg_bytes": by, "gbs": gbs, "frac": (gbs / hbm_peak) if gbs else None}
    dom = max(stages, key=lambda k: stages[k]["us"])
    roof = {"kernel": dom, "bound": "hbm", "achieved": stages[dom]["gbs"], "peak": hbm_peak, "unit": "GB/s",
            "frac": stages[dom]["frac"],
            # the committed captures are of the tensor-core chain; the CUDA-core chain has none
            "traffic": _traffic_from_profiles(dom, cfg.name, T, H) if tc else None,
            "peak_source": peak_src, "alg_bytes_per_launch": stages[dom]["alg_bytes"],
            "us_per_launch": stages[dom]["us"]}
    from selective_attention_b200 import workloads

    local_cfg = workloads.SSDConfig(**{**cfg.__dict__, "batch": b, "seqlen": L, "nheads": H, "ngroups": G})
    fused_min = workloads.ssd_algorithmic_bytes(local_cfg, y_bytes=run.y.element_size(), nseq=nseq)
    whole = {"alg_min_bytes": fused_min, "gbs": fused_min / (ms_step / 1e3) / 1e9,
             "frac_of_fused_roof": fused_min / (ms_step / 1e3) / 1e9 / hbm_peak}
    return {"value": global_tokens / (ms_step / 1e3), "unit": "tokens/s", "ms_per_step": ms_step, "steps": steps,
            "path": {"tc_fused": "tcgen05, chunk_state+state_passing fused", "tc_staged": "tcgen05",
                     "simt": "cuda-core", "tc_split": "tcgen05, split-bf16 products of fp32"}[path],
            "roofline": roof, "stages": stages, "whole_step": whole, "launches_per_step": run.launches}


def _row_split_inputs(cfg, rank, world, dev):
    """This rank's rows of the global batch (``cfg.batch`` rows per rank), or for packed
    varlen configs its own packed batch (batch ``rank`` of the global problem)."""
    from selective_attention_b200 import sharding, workloads

    if cfg.varlen:
        return workloads.make_ssd_inputs(cfg, seed=1 + rank, device=dev, gen_device="cuda")
    glob = workloads.SSDConfig(**{**cfg.__dict__, "batch": cfg.batch * world})
    return sharding.make_row_inputs(glob, 1, sharding.row_range(rank, world, glob.batch), device=dev,
                                    gen_device="cuda")


def verify_row_split(run, cfg, rank, world, dev, args):
    """NCCL all_gather of every rank's y and h_last (outside the timed region); rank 0
    rebuilds each other rank's rows from the shared seed, runs them through the same
    kernels and compares."""
    from selective_attention_b200 import sharding

    y_all = sharding.gather_rows(run.y, world)
    h_all = sharding.gather_rows(run.h_last, world)
    if rank != 0:
        return None
    worst = {"bit_identical": True, "max_abs_diff": 0.0}
    b = run.y.shape[0]
    for r in range(1, world):
        other = SSDRun(cfg, _row_split_inputs(cfg, r, world, dev), args.kernel_impl, dev)
        other.step()
        torch.cuda.synchronize()
        for got, want in ((y_all[r * b:(r + 1) * b], other.y), (h_all[r * b:(r + 1) * b], other.h_last)):
            c = sharding.compare(got, want)
            worst["bit_identical"] &= c["bit_identical"]
            worst["max_abs_diff"] = max(worst["max_abs_diff"], c["max_abs_diff"])
        del other
    return {"collective": "nccl all_gather of y and h_last", "checked_ranks": list(range(1, world)),
            "against": "rank 0 re-running each rank's rows from the shared seed", **worst}


def c4_measure(args, rank, world, dev, flush, hbm_peak, peak_src):
    """Config c4 (bf16 8 x 65536, H128 P64 N128 G8 cs256, D + z), one global problem split
    by whole head groups over the ranks (strong scaling: rank r takes groups
    [8r/N, 8(r+1)/N)); tokens/s for the global problem from the slowest rank's device
    time. With N > 1, the ranks' y and h_last are gathered over NCCL after the timed
    loop, batch row by batch row, and rank 0 compares them with its own one-GPU run of
    the whole problem."""
    from selective_attention_b200 import sharding, workloads

    cfg = workloads.CONFIGS["c4"]
    groups = sharding.group_range(rank, world, cfg.ngroups)
    inp = sharding.make_group_inputs(cfg, 1, groups, device=dev, gen_device="cuda")
    run = SSDRun(cfg, inp, args.kernel_impl, dev)
    steps = max(5, min(args.steps, 50))
    res = measure_ssd(run, args, world, flush, hbm_peak, peak_src, cfg.tokens, steps)
    res.update(workload=_workload_name(cfg), scaling="strong", n_gpus=world,
               split=f"head groups {groups[0]}..{groups[1] - 1} of {cfg.ngroups} on rank {rank}" if world > 1
               else "whole problem on one GPU", dtype="bf16")
    if world > 1:
        full = None
        if rank == 0:
            torch.cuda.empty_cache()
            full = SSDRun(cfg, sharding.make_group_inputs(cfg, 1, (0, cfg.ngroups), device=dev, gen_device="cuda"),
                          args.kernel_impl, dev)
            full.step()
            torch.cuda.synchronize()
        worst = {"bit_identical": True, "max_abs_diff": 0.0}
        for r in range(cfg.batch):
            got = sharding.gather_heads(run.y[r:r + 1], world, 2)
            if full is not None:
                c = sharding.compare(got, full.y[r:r + 1])
                worst["bit_identical"] &= c["bit_identical"]
                worst["max_abs_diff"] = max(worst["max_abs_diff"], c["max_abs_diff"])
            del got
        got = sharding.gather_heads(run.h_last, world, 1)
        if full is not None:
            c = sharding.compare(got, full.h_last)
            worst["bit_identical"] &= c["bit_identical"]
            worst["max_abs_diff"] = max(worst["max_abs_diff"], c["max_abs_diff"])
            res["verify"] = {"collective": "nccl all_gather of y (per batch row) and h_last",
                             "against": "rank 0's one-GPU run of the whole c4 problem", **worst}
        del full, got
    del run, inp
    torch.cuda.empty_cache()
    return res


def c2_measure(args, dev, flush, hbm_peak, peak_src):
    """Config c2 (32768 packed tokens, H80 P64 N128 G1 cs256, D + z, bf16) on one GPU."""
    from selective_attention_b200 import workloads

    cfg = workloads.CONFIGS["c2"]
    inp = workloads.make_ssd_inputs(cfg, seed=1, device=dev, gen_device="cuda")
    run = SSDRun(cfg, inp, args.kernel_impl, dev)
    res = measure_ssd(run, args, 1, flush, hbm_peak, peak_src, cfg.tokens, max(5, min(args.steps, 100)))
    res.update(workload=_workload_name(cfg), n_gpus=1, dtype="bf16")
    del run, inp
    torch.cuda.empty_cache()
    return res


def fp32_measure(args, dev, flush, hbm_peak, peak_src):
    """Config c1's shape in fp32 (the reference's own precision: its SSD takes fp32
    operands only) on one GPU: fp32 u, B, C, z in and y out, on the default fp32 chain
    (tensor cores with split-bf16 products; ``--kernel-impl simt`` does not change it), and
    the backward on the same inputs unless ``--no-bwd``."""
    from selective_attention_b200 import workloads

    cfg = workloads.SSDConfig(**{**workloads.CONFIGS["c1"].__dict__, "dtype": "f32"})
    inp = workloads.make_ssd_inputs(cfg, seed=1, device=dev, gen_device="cuda")
    run = SSDRun(cfg, inp, "auto", dev)
    res = measure_ssd(run, args, 1, flush, hbm_peak, peak_src, cfg.tokens, max(5, min(args.steps, 50)))
    res.update(workload=_workload_name(cfg), n_gpus=1, dtype="f32")
    del run
    # the CUDA-core chain on the same inputs (fp32 FFMA products), for comparison
    run = SSDRun(cfg, inp, "simt", dev)
    simt = measure_ssd(run, args, 1, flush, hbm_peak, peak_src, cfg.tokens, 5)
    res["cuda_core_chain"] = {"ms_per_step": simt["ms_per_step"], "value": simt["value"], "path": simt["path"],
                              "stages_us": {k: v["us"] for k, v in simt["stages"].items()}}
    del run
    if not args.no_bwd:
        # the backward on the same fp32 inputs (split-bf16 tcgen05 products, CUDA-core rest)
        res["bwd"] = bwd_measure(args, cfg, inp, dev, flush)
    del inp
    torch.cuda.empty_cache()
    return res


def run_ours(args, rank, world, local):
    dev = torch.device("cuda", local)
    from selective_attention_b200 import workloads

    cfg = workloads.CONFIGS[args.config]
    peaks = _peaks()
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    # Headline: the workload split by batch rows, cfg.batch rows per rank (weak scaling);
    # at one GPU it is the benchmark config itself.
    inp = _row_split_inputs(cfg, rank, world, dev)
    run = SSDRun(cfg, inp, args.kernel_impl, dev)
    clocks = ClockSampler(local)
    time.sleep(1.0)  # let the sampler start before the timed loop
    head = measure_ssd(run, args, world, flush, hbm_peak, peak_src, world * cfg.tokens, args.steps, clocks)
    clk = clocks.stop()
    sx = inp["u"].element_size()
    parallelism = "single" if world == 1 else f"dp{world}: batch rows split, {cfg.batch} rows per rank"
    if cfg.varlen and world > 1:
        parallelism = f"dp{world}: one packed batch per rank"
    line = {
        "metric": "SSD chunked-scan fwd tokens/s", "value": head["value"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if sx == 2 else "f32", "data": "synthetic",
        "config": {"workload": _workload_name(cfg), "global_batch": cfg.batch * world, "seq_len": cfg.seqlen,
                   "parallelism": parallelism, "path": head["path"],
                   "l2": "flushed between timed steps (256 MiB write)"},
        "roofline": head["roofline"], "stages": head["stages"], "whole_step": head["whole_step"], "clocks": clk,
        "gpu_launches": args.steps * run.launches,
    }
    if world > 1 and not cfg.varlen:
        line["verify"] = verify_row_split(run, cfg, rank, world, dev, args)
    if not args.no_e2e:
        line["e2e"] = e2e_measure(args, cfg, inp, dev, world, flush)
    del run
    torch.cuda.empty_cache()
    if not args.no_c4:
        line["c4"] = c4_measure(args, rank, world, dev, flush, hbm_peak, peak_src)
    if world == 1:
        if not args.no_extra and args.config != "c2":
            line["c2"] = c2_measure(args, dev, flush, hbm_peak, peak_src)
        if not args.no_extra:
            line["fp32"] = fp32_measure(args, dev, flush, hbm_peak, peak_src)
        if not args.no_ssu:
            line["ssu"] = ssu_measure(args, dev, flush, hbm_peak, world)
        if not args.no_front:
            line["front"] = front_measure(args, dev, flush, hbm_peak)
        if not args.no_bwd:
            line["bwd"] = bwd_measure(args, cfg, inp, dev, flush)
        if not args.no_sattn:
            line["sattn_decode"] = sattn_measure(args, dev, flush, hbm_peak)
            line["sattn_prefill"] = sattn_prefill_measure(args, dev, flush, peaks.get("bf16_tflops", 1590.0))
            line["sattn_train"] = sattn_train_measure(args, dev, flush, peaks.get("bf16_tflops", 1590.0))
        if not args.no_ref_gpu:
            line["reference_gpu"] = ref_gpu_measure(args, dev, flush)
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)


def _workload_name(cfg):
    extra = "+D" if cfg.D else ""
    extra += "+z" if cfg.z else ""
    shape = f"{cfg.tokens} packed tokens" if cfg.varlen else f"{cfg.batch}x{cfg.seqlen}"
    return (f"{cfg.name}: SSD fwd {cfg.dtype} {shape} H{cfg.nheads} P{cfg.headdim} N{cfg.dstate} "
            f"G{cfg.ngroups} cs{cfg.chunk} {extra}").strip()


def _traffic_from_profiles(kernel, cfg_name, tokens, heads):
    """DRAM bytes per launch of ``kernel`` from the committed ncu summary
    (``profiles/dram_traffic.json``: per config, the bytes of one captured launch and the
    token-heads it processed), scaled to this launch's token-heads; None without a capture."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        d = json.load(open(path)).get(cfg_name, {}).get(kernel)
    except (OSError, ValueError):
        return None
    if d is None:
        return None
    if isinstance(d, dict):
        return d["bytes"] * (tokens * heads) / d["token_heads"]
    return d


E2E_SLICES = 4


def e2e_measure(args, cfg, inp, dev, world, flush):
    """Same metric through the public API with pinned host inputs and outputs: the
    streaming entry ``HostStreamScan`` (row slices, copies overlapped with the scan) for
    padded batches, ``SSDScanFn`` with explicit copies for packed ones."""
    import selective_attention_b200 as sab

    names = ["u", "B", "C", "delta_raw", "z"]
    host = {k: inp[k].cpu().pin_memory() for k in names if inp[k] is not None}
    dev_in = {k: torch.empty_like(inp[k]) for k in host}
    small = {k: inp[k] for k in ("A", "D")}
    cu = inp["cu_seqlens"]
    y_h = torch.empty(cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, dtype=inp["u"].dtype).pin_memory()
    nrow = cfg.batch if cu is None else cu.numel() - 1
    h_h = torch.empty(nrow, cfg.nheads, cfg.headdim, cfg.dstate, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    scanner = sab.HostStreamScan(dev, slices=E2E_SLICES, in_flight=3) if cu is None else None
    A_h, D_h = small["A"].cpu(), small["D"].cpu()

    def step():
        if scanner is not None:
            scanner(host["u"], A_h, host["B"], host["C"], host["delta_raw"], None, None, None, cfg.chunk, True,
                    (0.0, INF), D_h, host.get("z"), out=(y_h, h_h))
            return
        for k, t in host.items():
            dev_in[k].copy_(t, non_blocking=True)
        y, h = sab.SSDScanFn.apply(dev_in["u"], small["A"], dev_in["B"], dev_in["C"], dev_in["delta_raw"], None,
                                   None, None, cfg.chunk, True, (0.0, INF), True, small["D"], dev_in.get("z"), cu)
        y_h.copy_(y, non_blocking=True)
        h_h.copy_(h, non_blocking=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 50))
    barrier(world)
    per = time_steps(step, steps, flush, stream)
    barrier(world)
    ms = max_over_ranks(sum(per), world) / steps
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = y_h.numel() * y_h.element_size() + h_h.numel() * h_h.element_size()
    return {"value": world * cfg.tokens / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "steps": steps,
            "note": ("pinned host -> device inputs, scan, device -> pinned host y and h_last, per step; "
                     + (f"HostStreamScan, {E2E_SLICES} row slices, copy-in / scan / copy-out streams"
                        if scanner is not None else "SSDScanFn"))}


def front_measure(args, dev, flush, hbm_peak):
    """SSM prefill front end at config 1's widths (b 8, L 2048, inner 1536, G*N 128, K 4,
    bf16): SiLU + depthwise causal conv + split into x, B, C and the decode cache, read
    from a slice of the input projection's output. Achieved HBM GB/s on its bytes."""
    from selective_attention_b200 import kernels

    b, L, inner, gn, K, H = 8, 2048, 1536, 128, 4, 24
    conv_dim = inner + 2 * gn
    g = torch.Generator(device=dev).manual_seed(1)
    proj = torch.randn(b, L, conv_dim + inner + H, device=dev, generator=g).to(torch.bfloat16)
    hBC = proj[..., :conv_dim]
    w = torch.randn(conv_dim, 1, K, device=dev, generator=g) * 0.5
    bias = torch.randn(conv_dim, device=dev, generator=g) * 0.1
    x = torch.empty(b, L, inner, device=dev, dtype=torch.bfloat16)
    Bo = torch.empty(b, L, gn, device=dev, dtype=torch.bfloat16)
    Co = torch.empty(b, L, gn, device=dev, dtype=torch.bfloat16)

    ctx = torch.empty(b, conv_dim, K, device=dev, dtype=torch.bfloat16)
    kernels.ssm_conv_prefill(hBC, w, bias, inner, gn, build_ctx=True, out=(x, Bo, Co))  # checks the wrapper once
    # Timed through the C ABI with the arguments prepared once: the kernel pair takes
    # ~10 us, less than the Python wrapper's own per-call cost, which would otherwise
    # leave the GPU idle inside the timed interval.
    from selective_attention_b200 import _lib

    fn, w2 = _lib.lib().ssm_conv_prefill, w.reshape(conv_dim, K).contiguous()
    cargs = (_lib.ptr(hBC), hBC.stride(1), _lib.ptr(w2), _lib.ptr(bias), _lib.ptr(x), _lib.ptr(Bo), _lib.ptr(Co),
             _lib.ptr(ctx), None, b, L, inner, gn, K, _lib.dtype_code(torch.bfloat16, "hBC"),
             torch.cuda.current_stream(dev).cuda_stream)

    def step():
        _lib.check(fn(*cargs), "ssm_conv_prefill")

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 200))
    per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
    us = statistics.median(per) * 1e3
    by = 2 * b * L * conv_dim * 2 + conv_dim * (K + 1) * 4 + b * conv_dim * K * 2
    gbs = by / (us / 1e6) / 1e9
    return {"config": "c1 widths: b8 L2048 conv_dim 1792 (x 1536 + B 128 + C 128) K4 bf16, projection slice in",
            "us_per_step": us, "alg_bytes": by, "gbs": gbs, "peak_gbs": hbm_peak, "frac": gbs / hbm_peak,
            "steps": steps, "timing": "median of per-step CUDA events around the C-ABI call (arguments prepared once), "
                                     "L2 flushed between steps"}


FFMA_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # CUDA-core fp32 FMA, nominal (no measured figure)


def bwd_measure(args, cfg, inp, dev, flush):
    """SSD backward (row f1) on the bench workload's inputs: y_grad fp32 (the reference's
    y dtype) and h_last_grad, through ``kernels.ssd_scan_backward`` (the C-ABI
    ``ssd_scan_bwd``). For 16-bit u / B / C at headdim 64, dstate 128, chunk 256 (the bench
    workload) the contractions run on tcgen05 with 16-bit operands; reported in TFLOP/s of
    the algorithmic FLOPs, with the per-stage split from the C-ABI's events; fp32 u / B / C
    at that shape run them on tcgen05 with split-bf16 products. The FFMA fraction is kept for
    comparison with the CUDA-core path."""
    from selective_attention_b200 import kernels

    u, A, B, C, dr = inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"]
    b, L, H, P = u.shape
    G, N = B.shape[2], B.shape[3]
    cu = inp.get("cu_seqlens")
    nrows = b if cu is None else cu.numel() - 1
    g = torch.Generator(device=dev).manual_seed(2)
    yg = torch.randn(b, L, H, P, device=dev, generator=g)
    hlg = 0.1 * torch.randn(nrows, H, P, N, device=dev, generator=g)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in ev:
        e.record()
    handles = [e.cuda_event for e in ev]
    ws = torch.empty(0, dtype=torch.uint8, device=dev)

    def step(events=None):
        kernels.ssd_scan_backward(u, A, B, C, dr, None, None, yg, hlg, None, cfg.chunk, cu_seqlens=cu,
                                  events=events)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 20))
    per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
    split = []
    for _ in range(3):
        step(handles)
        torch.cuda.synchronize()
        split.append([ev[i].elapsed_time(ev[i + 1]) for i in range(5)])
    names = ["cumsum+states", "state_pass+cb", "state_grad", "intra", "bmm+reduce"]
    stages = {n: statistics.median(x[i] for x in split) for i, n in enumerate(names)}
    ms = statistics.median(per)
    cs = cfg.chunk
    if cu is None:
        nk = b * ((L + cs - 1) // cs)
    else:
        nk = sum((n + cs - 1) // cs for n in (cu[1:] - cu[:-1]).tolist())
    # per (chunk, head): five cs x P x N products (S, HG, accS, B_grad, C_grad terms) and two
    # causal cs x cs x P ones (CB^T y_grad, y_grad u^T); per (chunk, group): CB and the two
    # bmm-backward products, causal cs x cs x N. Counted on whole chunks.
    flops = nk * H * (10 * cs * P * N + 2 * cs * cs * P) + nk * G * 3 * cs * cs * N
    tf = flops / (ms * 1e-3) / 1e12
    del ws
    return {"config": f"{cfg.name} inputs, y_grad fp32 + h_last_grad, no D/z", "ms_per_step": ms,
            "tokens_per_s": b * L / (ms * 1e-3), "stages_ms": stages, "alg_flops": flops, "tflops": tf,
            "ffma_nominal_tflops": FFMA_NOMINAL_TFLOPS, "frac_of_nominal_ffma": tf / FFMA_NOMINAL_TFLOPS,
            "steps": steps, "timing": "median of per-step CUDA events, L2 flushed between steps"}


def sattn_measure(args, dev, flush, hbm_peak):
    """Selective-attention decode step (row f4): b 64, H 16, head_dim 64, an fp32 cache
    (the reference allocates its cache in fp32) holding 4000 keys; each step writes the
    token's key / value / log-gate and attends over the 4001 keys. Achieved HBM GB/s on the
    step's bytes, through the C-ABI call with arguments prepared once."""
    from selective_attention_b200 import _lib, kernels

    b, H, D, cap, w = 64, 16, 64, 4096, 4000
    g = torch.Generator(device=dev).manual_seed(3)
    kc = torch.randn(b, H, cap, D, device=dev, generator=g)
    vc = torch.randn(b, H, cap, D, device=dev, generator=g)
    lgc = torch.log(torch.sigmoid(torch.randn(b, H, cap, device=dev, generator=g) + 2.0)) * 2.0
    q, kn, vn = (torch.randn(b, H, D, device=dev, generator=g) for _ in range(3))
    lgn = torch.zeros(b, H, device=dev)
    out = kernels.sattn_decode_step(q, kn, vn, lgn, kc, vc, lgc, w)  # checks the wrapper once
    fn = _lib.lib().sattn_decode_step
    cargs = (_lib.ptr(q), _lib.ptr(kn), _lib.ptr(vn), _lib.ptr(lgn), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(lgc), w,
             cap, _lib.ptr(out), b, H, D, D ** -0.5, 0, torch.cuda.current_stream(dev).cuda_stream)

    def step():
        _lib.check(fn(*cargs), "sattn_decode_step")

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 200))
    per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
    us = statistics.median(per) * 1e3
    n = w + 1
    by = b * H * (n * D * 4 * 2 + n * 4 + 4 * D * 4 + 4 + D * 4 * 2)  # K, V, gates read; q, new k/v/gate, out
    gbs = by / (us / 1e6) / 1e9
    return {"config": "b64 H16 D64, fp32 cache of 4096 slots, 4001 keys attended", "us_per_step": us,
            "alg_bytes": by, "gbs": gbs, "peak_gbs": hbm_peak, "frac": gbs / hbm_peak, "steps": steps,
            "timing": "median of per-step CUDA events around the C-ABI call (arguments prepared once), "
                      "L2 flushed between steps"}


def sattn_prefill_measure(args, dev, flush, tc_peak):
    """Selective-attention prefill (row f4, inference): b 2, H 16, L 2048, head_dim 64, bf16
    inputs, 10 % of the keys dropped. TFLOP/s of the causal attention's 2 L^2 D FLOPs per
    (row, head), for the tensor-core kernel (against the measured bf16 dense peak) and the
    CUDA-core one (against the nominal FFMA rate)."""
    from selective_attention_b200 import kernels

    b, H, L, D = 2, 16, 2048, 64
    g = torch.Generator(device=dev).manual_seed(4)
    q, k, v = (torch.randn(b, H, L, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    lg = torch.log(torch.sigmoid(torch.randn(b, H, L, device=dev, generator=g) + 2.0)) * 2.0
    lg = torch.where(torch.rand(b, H, L, device=dev, generator=g) < 0.1, torch.full_like(lg, -math.inf), lg)
    out = torch.empty_like(q)
    flops = 2 * b * H * L * L * D
    res = {"config": "b2 H16 L2048 D64 bf16, 10% of keys dropped", "alg_flops": flops,
           "timing": "median of per-step CUDA events, L2 flushed between steps"}
    for impl, peak, peak_name in (("tc", tc_peak, "bf16 dense, measured"),
                                  ("simt", FFMA_NOMINAL_TFLOPS, "fp32 FFMA, nominal")):
        def step():
            kernels.sattn_prefill(q, k, v, lg, out=out, impl=impl)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        steps = max(5, min(args.steps, 50))
        per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
        ms = statistics.median(per)
        tf = flops / (ms * 1e-3) / 1e12
        res[impl] = {"ms_per_step": ms, "tflops": tf, "peak_tflops": peak, "peak": peak_name, "frac": tf / peak,
                     "steps": steps}
    return res


def sattn_train_measure(args, dev, flush, tc_peak):
    """Selective attention in training mode (row f4, training): b 2, H 16, L 2048, head_dim 64,
    causal, ragged lengths, bf16 inputs; one step = ``SelectiveAttnTrainFn`` forward + backward
    (tcgen05 kernels for this shape). TFLOP/s of the algorithmic FLOPs over the causal pairs
    (forward: statistics q k^T, attention q k^T and P v = 3 x 2 L^2 D / 2; backward as the
    reference's autograd runs it: q k^T, dO v^T, dv, dq, dk = 5 x 2 L^2 D / 2) against the
    measured bf16 dense peak, and the CUDA-core path (``impl="simt"``) against the nominal FFMA
    rate."""
    import selective_attention_b200 as sab

    b, H, L, D = 2, 16, 2048, 64
    g = torch.Generator(device=dev).manual_seed(5)
    q, k, v = (torch.randn(b, H, L, D, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
               for _ in range(3))
    sel = torch.sigmoid(torch.randn(b, H, L, device=dev, generator=g) + 2.0).to(torch.bfloat16).requires_grad_(True)
    lengths = torch.tensor([L, 3 * L // 4], device=dev)
    dout = torch.randn(b, H, L, D, device=dev, generator=g).to(torch.bfloat16)

    flops = 8 * b * H * L * L * D
    res = {"config": "b2 H16 L2048 D64 bf16 causal, lengths (2048, 1536)", "alg_flops": flops,
           "timing": "median of per-step CUDA events, L2 flushed between steps"}
    for impl, peak, peak_name in (("tc", tc_peak, "bf16 dense, measured"),
                                  ("simt", FFMA_NOMINAL_TFLOPS, "fp32 FFMA, nominal")):
        def fwd():
            return sab.selective_attn_train(q, k, v, sel, lengths, 1.0, True, impl=impl)

        def step():
            out, _ = fwd()
            out.backward(dout)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        steps = max(5, min(args.steps, 20))
        per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
        per_f = time_steps(fwd, steps, flush, torch.cuda.current_stream(dev))
        ms, ms_f = statistics.median(per), statistics.median(per_f)
        tf = flops / (ms * 1e-3) / 1e12
        res[impl] = {"ms_per_step": ms, "fwd_ms": ms_f, "bwd_ms": ms - ms_f, "tflops": tf, "peak_tflops": peak,
                     "peak": peak_name, "frac": tf / peak, "steps": steps}
    return res


def ref_gpu_measure(args, dev, flush):
    """Secondary comparison on this GPU: the reference's own Triton SSD (``SSDScanFn`` of the
    package ``baseline/install_reference.sh`` installs into ``baseline/_ref``; ``ops/ssd_scan.py``
    over ``triton_kernels/ssd_scan``) at config 1's shape in fp32, its operand type, forward
    and forward + backward, beside this library's ``SSDScanFn`` on the same fp32 inputs (the
    split-bf16 tensor-core forward, and the CUDA-core forward with ``impl="simt"``; the backward
    is the same in both: split-bf16 tcgen05 stages and CUDA-core stages for fp32) and on bf16 inputs (tensor cores). No D / z (the
    reference op has none).
    The reference runs its stock code path; Triton compiles and autotunes it on first use,
    outside the timed steps."""
    import selective_attention_b200 as sab
    from selective_attention_b200 import workloads

    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "selective_attention")):
        return {"unavailable": "reference package not installed in baseline/_ref"}
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        from selective_attention.ops import SSDScanFn as RefSSD
    except Exception as e:  # noqa: BLE001 - recorded, not raised: the entry is optional
        return {"unavailable": f"reference import failed: {e!r}"[:300]}
    cfg = workloads.SSDConfig(**{**workloads.CONFIGS["c1"].__dict__, "dtype": "f32", "D": False, "z": False})
    inp = workloads.make_ssd_inputs(cfg, seed=7, device=dev, gen_device="cuda")
    b, L = cfg.batch, cfg.seqlen
    length = torch.full((b,), L, dtype=torch.long, device=dev)
    g = torch.Generator(device=dev).manual_seed(8)
    res = {"config": "c1 shape (8x2048 H24 P64 N128 G1 cs256), no D / z; fp32 unless noted",
           "timing": "median of per-step CUDA events, L2 flushed between steps"}
    steps = max(3, min(args.steps, 10))
    stream = torch.cuda.current_stream(dev)

    def run(name, op, dtype, extra=()):
        leaves = [inp[k].to(dtype) if k in ("u", "B", "C") else inp[k] for k in ("u", "A", "B", "C", "delta_raw")]
        bias = inp.get("delta_bias")
        yg = torch.randn(inp["u"].shape, device=dev, generator=g)

        def fwd():
            with torch.no_grad():
                return op.apply(*leaves, bias, None, length, cfg.chunk, *extra)

        def fwd_bwd():
            xs = [t.detach().requires_grad_(True) for t in leaves]
            y, h = op.apply(*xs, bias, None, length, cfg.chunk, *extra)
            torch.autograd.backward([y], [yg.to(y.dtype)])

        try:
            for f in (fwd, fwd_bwd):
                f()
            torch.cuda.synchronize()
            tf = statistics.median(time_steps(fwd, steps, flush, stream))
            tb = statistics.median(time_steps(fwd_bwd, steps, flush, stream))
            res[name] = {"fwd_ms": tf, "fwd_bwd_ms": tb, "tokens_per_s_fwd": b * L / (tf * 1e-3)}
        except Exception as e:  # noqa: BLE001 - recorded, the other lines still run
            res[name] = {"error": f"{e!r}"[:300]}

    run("reference_triton_fp32", RefSSD, torch.float32)
    run("ours_fp32", sab.SSDScanFn, torch.float32)
    run("ours_fp32_cuda_core", sab.SSDScanFn, torch.float32, (True, (0.0, INF), True, None, None, None, "simt"))
    run("ours_bf16", sab.SSDScanFn, torch.bfloat16)
    r, o = res.get("reference_triton_fp32", {}), res.get("ours_bf16", {})
    if "fwd_ms" in r and "fwd_ms" in o:
        res["speedup_bf16_vs_reference_fwd"] = r["fwd_ms"] / o["fwd_ms"]
        res["speedup_bf16_vs_reference_fwd_bwd"] = r["fwd_bwd_ms"] / o["fwd_bwd_ms"]
    if "fwd_ms" in r and "fwd_ms" in res.get("ours_fp32", {}):
        res["speedup_fp32_vs_reference_fwd"] = r["fwd_ms"] / res["ours_fp32"]["fwd_ms"]
        res["speedup_fp32_vs_reference_fwd_bwd"] = r["fwd_bwd_ms"] / res["ours_fp32"]["fwd_bwd_ms"]
    del inp
    torch.cuda.empty_cache()
    return res


def ssu_measure(args, dev, flush, hbm_peak, world):
    """Decode state update, benchmark config c3: achieved HBM GB/s on the algorithmic bytes."""
    from selective_attention_b200 import kernels, workloads

    cfg = workloads.SSU_CONFIGS["c3"]
    inp = workloads.make_ssu_inputs(cfg, seed=2, device=dev, gen_device="cuda")
    y = torch.empty_like(inp["u"])
    h = inp["h"]

    def step():
        kernels.ssu_forward(inp["u"], inp["A"], inp["B"], inp["C"], inp["delta_raw"], inp["delta_bias"], h, True,
                            (0.0, INF), inp["D"], inp["z"], y=y)

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 200))
    per = time_steps(step, steps, flush, torch.cuda.current_stream(dev))
    us = statistics.median(per) * 1e3
    by = workloads.ssu_algorithmic_bytes(cfg)
    gbs = by / (us / 1e6) / 1e9
    return {"config": "c3: decode b256 H80 P64 N128 G1, fp32 state in place, bf16 x/B/C/z, D+z",
            "us_per_step": us, "alg_bytes": by, "gbs": gbs, "peak_gbs": hbm_peak, "frac": gbs / hbm_peak,
            "steps": steps, "timing": "median of per-step CUDA events, L2 flushed between steps",
            "front": decode_front_measure(args, dev, flush, cfg)}


def decode_front_measure(args, dev, flush, cfg):
    """The decode step's front end before the SSU at config 3's widths (conv cache update,
    SiLU, weighted sum, split; K 4): one launch through the C ABI, arguments prepared once
    (the kernel is a few microseconds, below the Python wrapper's own cost)."""
    from selective_attention_b200 import _lib, kernels

    b, inner, gn, K = cfg.batch, cfg.nheads * cfg.headdim, cfg.ngroups * cfg.dstate, 4
    conv_dim = inner + 2 * gn
    g = torch.Generator(device=dev).manual_seed(3)
    proj = torch.randn(b, conv_dim + inner + cfg.nheads, device=dev, generator=g).to(torch.bfloat16)
    ctx = torch.randn(b, conv_dim, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(conv_dim, K, device=dev, generator=g) * 0.5).contiguous()
    bias = torch.randn(conv_dim, device=dev, generator=g) * 0.1
    x = torch.empty(b, inner, device=dev, dtype=torch.bfloat16)
    Bo = torch.empty(b, gn, device=dev, dtype=torch.bfloat16)
    Co = torch.empty(b, gn, device=dev, dtype=torch.bfloat16)
    kernels.ssm_conv_decode(proj[:, :conv_dim], ctx, w, bias, inner, gn, out=(x, Bo, Co))
    fn = _lib.lib().ssm_conv_decode
    cargs = (_lib.ptr(proj), proj.stride(0), _lib.ptr(ctx), _lib.ptr(w), _lib.ptr(bias), _lib.ptr(x), _lib.ptr(Bo),
             _lib.ptr(Co), b, inner, gn, K, _lib.dtype_code(torch.bfloat16, "hBC"),
             torch.cuda.current_stream(dev).cuda_stream)

    def step():
        _lib.check(fn(*cargs), "ssm_conv_decode")

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    per = time_steps(step, max(10, min(args.steps, 200)), flush, torch.cuda.current_stream(dev))
    us = statistics.median(per) * 1e3
    by = b * conv_dim * (2 * 2 * K + 2 + 2) + conv_dim * (K + 1) * 4  # cache r/w, input, output, weights
    return {"config": f"b{b} conv_dim {conv_dim} (x {inner} + B {gn} + C {gn}) K{K} bf16, cache in place",
            "us_per_step": us, "alg_bytes": by, "gbs": by / (us / 1e6) / 1e9,
            "note": "replaces the reference's cache roll, silu, product, sum, bias add and split (6 torch launches)"}


if __name__ == "__main__":
    main()
