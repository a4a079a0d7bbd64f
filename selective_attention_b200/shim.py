"""Route an installed reference package through the B200 kernels.

``install()`` rebinds ``SSDScanFn`` and ``SSUFn`` in ``selective_attention.ops`` and in
the module that calls them, ``selective_attention.modules.ssm`` (``ssm.py:7``), so the
reference's SSM layer and decode cache path (``ssm.py:136-139,195-197``) run on the
CUDA library without other changes. ``uninstall()`` restores the originals.

``install()`` raises ``ImportError`` when the package, its ``ops`` module or its
``modules.ssm`` module cannot be imported, or when they do not define both names: a
misspelt package name must not leave the caller silently on the reference's kernels.
"""
from __future__ import annotations

import importlib

from .ops import SSDScanFn, SSUFn

_saved = {}

# Modules that must exist and bind both names (the ops package and its caller), and
# modules that are rebound when present (the op's own defining modules).
_REQUIRED = ("ops", "modules.ssm")
_OPTIONAL = ("ops.ssd_scan", "ops.ssu")
_NAMES = (("SSDScanFn", SSDScanFn), ("SSUFn", SSUFn))


def install(package: str = "selective_attention") -> None:
    targets = []
    for sub in _REQUIRED:
        modname = f"{package}.{sub}"
        mod = importlib.import_module(modname)  # ImportError propagates
        missing = [name for name, _ in _NAMES if not hasattr(mod, name)]
        if missing:
            raise ImportError(f"{modname} does not define {', '.join(missing)}")
        targets.append((modname, mod))
    for sub in _OPTIONAL:
        modname = f"{package}.{sub}"
        try:
            targets.append((modname, importlib.import_module(modname)))
        except ModuleNotFoundError as e:
            if e.name != modname:
                raise  # the module exists but one of its own imports failed
    for modname, mod in targets:
        for name, repl in _NAMES:
            if hasattr(mod, name):
                _saved.setdefault((modname, name), getattr(mod, name))
                setattr(mod, name, repl)


def installed() -> bool:
    return bool(_saved)


def uninstall() -> None:
    for (modname, name), orig in list(_saved.items()):
        setattr(importlib.import_module(modname), name, orig)
    _saved.clear()
