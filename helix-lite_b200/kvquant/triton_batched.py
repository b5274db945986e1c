"""Import-compatible module name for src/kvquant/triton_batched.py.

The functions are the CUDA implementations in :mod:`kvquant.batched`; no
Triton is involved.
"""
from .batched import (  # noqa: F401
    pack_keys_per_channel_batched,
    pack_values_per_token_batched,
    unpack_keys_per_channel_batched,
    unpack_values_per_token_batched,
)
