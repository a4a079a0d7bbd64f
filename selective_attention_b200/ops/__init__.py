"""Reference-compatible op entry points (mirrors ``selective_attention.ops``)."""
from .ssd_scan import SSDScanFn
from .selective_attn import SelectiveAttnTrainFn, selective_attn_train
from .ssu import SSUFn

__all__ = ["SSDScanFn", "SSUFn", "SelectiveAttnTrainFn", "selective_attn_train"]
