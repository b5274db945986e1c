"""kvquant: nuq KV quantisation, the compact paged pool and the fused decode,
with the call signatures of xFuzzitx/helix-lite ``src/kvquant``
(exports of src/kvquant/__init__.py:24-33 plus the pool, selector and hooks).

All compute runs in the CUDA library ``libhelix_kv.so`` (sm_100a); there is
no CPU path.
"""
from .nuq import dequantize_nuq, find_outliers, quantize_nuq, round_to_nearest_pole
from .scales import KVScales, PerChannelScale, PerTokenScale

__all__ = [
    "quantize_nuq",
    "dequantize_nuq",
    "find_outliers",
    "round_to_nearest_pole",
    "KVScales",
    "PerChannelScale",
    "PerTokenScale",
]
