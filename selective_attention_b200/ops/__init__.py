"""Reference-compatible op entry points (mirrors ``selective_attention.ops``)."""
from .ssd_scan import SSDScanFn
from .ssu import SSUFn

__all__ = ["SSDScanFn", "SSUFn"]
