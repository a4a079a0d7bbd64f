"""SSD forward on inputs that live in (pinned) host memory.

``HostStreamScan`` runs ``ssd_scan_forward`` over a padded batch whose tensors are in
host memory. The batch is cut into row slices that flow through a three-stream
pipeline:

    copy-in stream    H2D(0) H2D(1) H2D(2) ...            (never waits on a copy back)
    compute stream           scan(0) scan(1) scan(2) ...
    copy-out stream                 D2H(0) D2H(1) ...

so the host -> device link stays busy from the first slice to the last while scans
and device -> host copies of earlier slices run beside it (PCIe is full duplex).
Slices use a ring of ``in_flight`` device buffer sets; slice i reuses the set of
slice i - in_flight once that slice's copy back has finished. Rows are independent in
the scan, so the result equals one ``ssd_scan_forward`` over the whole batch (the
kernel chain chosen per slice may differ, with the same tolerance as between chains).

There is no reference counterpart: the reference takes device tensors only. This is
the entry for callers whose data is not resident on the GPU.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import kernels

INF = float("inf")


class HostStreamScan:
    """Reusable host -> device -> host streaming SSD forward for one problem shape.

    ``slices`` row slices per call, ``in_flight`` device buffer sets (each with its own
    workspace). Buffers are allocated on first use for a shape and kept, so repeated
    calls allocate nothing on the device.
    """

    def __init__(self, device=None, slices: int = 4, in_flight: int = 3):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.slices = max(1, int(slices))
        self.in_flight = max(2, int(in_flight))
        self._key = None
        self._bufs = None
        self._copy_in = torch.cuda.Stream(self.device)
        self._compute = torch.cuda.Stream(self.device)
        self._copy_out = torch.cuda.Stream(self.device)

    def _buffers(self, key, rows, L, H, P, G, N, dtypes, have):
        if self._key == key:
            return self._bufs
        dev = self.device
        bufs = []
        for _ in range(self.in_flight):
            b = {
                "u": torch.empty(rows, L, H, P, device=dev, dtype=dtypes["u"]),
                "B": torch.empty(rows, L, G, N, device=dev, dtype=dtypes["u"]),
                "C": torch.empty(rows, L, G, N, device=dev, dtype=dtypes["u"]),
                "delta_raw": torch.empty(rows, L, H, device=dev, dtype=dtypes["delta_raw"]),
                "y": torch.empty(rows, L, H, P, device=dev, dtype=dtypes["y"]),
                "h_last": torch.empty(rows, H, P, N, device=dev, dtype=torch.float32),
            }
            if have["z"]:
                b["z"] = torch.empty((rows,) + have["z"], device=dev, dtype=dtypes["u"])
            if have["h_init"]:
                b["h_init"] = torch.empty(rows, H, P, N, device=dev, dtype=torch.float32)
            if have["length"]:
                b["length"] = torch.empty(rows, device=dev, dtype=torch.int64)
            b["workspace"] = torch.empty(0, device=dev, dtype=torch.uint8)
            bufs.append(b)
        self._key, self._bufs = key, bufs
        return bufs

    def __call__(self, u, A, B, C, delta_raw, delta_bias=None, h_init=None, length=None, chunk_size=256,
                 use_delta_softplus=True, delta_limit=(0.0, INF), D=None, z=None, impl: str = "auto",
                 out: Optional[Sequence[torch.Tensor]] = None):
        """Same arguments and results as ``ssd_scan_forward`` (padded rows only), with
        u, B, C, delta_raw, z, h_init and length in host memory; results land in host
        memory (``out`` or new pinned tensors). A, D and delta_bias may be on either side.
        Returns once the work is queued; synchronize the current stream before reading."""
        if u.dim() != 4 or B.dim() != 4 or C.dim() != 4 or delta_raw.dim() != 3:
            raise ValueError("expected u (b, L, H, P), B and C (b, L, G, N), delta_raw (b, L, H)")
        for t, n in ((u, "u"), (B, "B"), (C, "C"), (delta_raw, "delta_raw"), (z, "z"), (h_init, "h_init"),
                     (length, "length")):
            if t is not None and t.is_cuda:
                raise ValueError(f"[{n}] HostStreamScan takes host tensors; use ssd_scan_forward for device ones")
        b, L, H, P = u.shape
        G, N = B.shape[2], B.shape[3]
        dev = self.device
        y_dtype = u.dtype if (D is not None or z is not None) else torch.float32
        if out is None:
            y_h = torch.empty(b, L, H, P, dtype=y_dtype).pin_memory()
            h_h = torch.empty(b, H, P, N, dtype=torch.float32).pin_memory()
        else:
            y_h, h_h = out
        cur = torch.cuda.current_stream(dev)
        small = {}
        for n, t in (("A", A), ("D", D), ("delta_bias", delta_bias)):
            small[n] = None if t is None else t.to(dev, dtype=torch.float32, non_blocking=True)
        rows = math.ceil(b / self.slices)
        # z keeps its own trailing shape: (L, H, P) or the SSM layer's (L, H * P)
        have = {"z": None if z is None else tuple(z.shape[1:]), "h_init": h_init is not None,
                "length": length is not None}
        key = (rows, L, H, P, G, N, u.dtype, delta_raw.dtype, y_dtype, have["z"], have["h_init"], have["length"])
        bufs = self._buffers(key, rows, L, H, P, G, N, {"u": u.dtype, "delta_raw": delta_raw.dtype, "y": y_dtype},
                             have)
        start = torch.cuda.Event()
        start.record(cur)  # after the small tensors' copies and the caller's earlier work
        for s in (self._copy_in, self._compute, self._copy_out):
            s.wait_event(start)
        out_done = []
        for i, r0 in enumerate(range(0, b, rows)):
            r1 = min(b, r0 + rows)
            n = r1 - r0
            d = bufs[i % self.in_flight]
            # host -> device; the buffer set is free once its previous slice was copied back
            with torch.cuda.stream(self._copy_in):
                if i >= self.in_flight:
                    self._copy_in.wait_event(out_done[i - self.in_flight])
                dv = {}
                for name, t in (("u", u), ("B", B), ("C", C), ("delta_raw", delta_raw), ("z", z), ("h_init", h_init),
                                ("length", length)):
                    if t is None:
                        dv[name] = None
                        continue
                    dv[name] = d[name][:n]
                    dv[name].copy_(t[r0:r1], non_blocking=True)
                in_done = torch.cuda.Event()
                in_done.record(self._copy_in)
            y_d, h_d = d["y"][:n], d["h_last"][:n]
            with torch.cuda.stream(self._compute):
                self._compute.wait_event(in_done)
                p, keep, _ = kernels.ssd_scan_params(dv["u"], small["A"], dv["B"], dv["C"], dv["delta_raw"],
                                                     small["delta_bias"], dv["h_init"], dv["length"], chunk_size,
                                                     use_delta_softplus, delta_limit, small["D"], dv["z"], None, impl)
                need = kernels.workspace_size(p)
                if d["workspace"].numel() < need:
                    d["workspace"] = torch.empty(need, device=dev, dtype=torch.uint8)
                kernels.ssd_scan_forward(dv["u"], small["A"], dv["B"], dv["C"], dv["delta_raw"], small["delta_bias"],
                                         dv["h_init"], dv["length"], chunk_size, use_delta_softplus, delta_limit,
                                         True, small["D"], dv["z"], None, impl, out=(y_d, h_d),
                                         workspace=d["workspace"])
                del keep
                scanned = torch.cuda.Event()
                scanned.record(self._compute)
            # device -> host
            with torch.cuda.stream(self._copy_out):
                self._copy_out.wait_event(scanned)
                y_h[r0:r1].copy_(y_d, non_blocking=True)
                h_h[r0:r1].copy_(h_d, non_blocking=True)
                done = torch.cuda.Event()
                done.record(self._copy_out)
                out_done.append(done)
        if out_done:
            cur.wait_event(out_done[-1])  # the copy-out stream runs the slices in order
        return y_h, h_h
