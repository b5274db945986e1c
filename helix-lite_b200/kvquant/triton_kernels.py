"""Import-compatible module name for src/kvquant/triton_kernels.py.

The per-head (T, D) functions are the CUDA implementations in
:mod:`kvquant.batched`; no Triton is involved.
"""
from .batched import (  # noqa: F401
    pack_keys_per_channel,
    pack_values_per_token,
    unpack_keys_per_channel,
    unpack_values_per_token,
)
