"""Route an installed reference package through the B200 kernels.

``install()`` rebinds ``SSDScanFn`` and ``SSUFn`` in ``selective_attention.ops`` and in
the module that calls them, ``selective_attention.modules.ssm`` (``ssm.py:7``), so the
reference's SSM layer and decode cache path (``ssm.py:136-139,195-197``) run on the
CUDA library without other changes. ``uninstall()`` restores the originals.
"""
from __future__ import annotations

import importlib

from .ops import SSDScanFn, SSUFn

_saved = {}


def install(package: str = "selective_attention") -> None:
    for modname in (f"{package}.ops", f"{package}.ops.ssd_scan", f"{package}.ops.ssu", f"{package}.modules.ssm"):
        try:
            mod = importlib.import_module(modname)
        except ImportError:
            continue
        for name, repl in (("SSDScanFn", SSDScanFn), ("SSUFn", SSUFn)):
            if hasattr(mod, name):
                _saved.setdefault((modname, name), getattr(mod, name))
                setattr(mod, name, repl)


def uninstall() -> None:
    for (modname, name), orig in list(_saved.items()):
        setattr(importlib.import_module(modname), name, orig)
    _saved.clear()
