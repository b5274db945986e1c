"""Bit-packed code rows (test infrastructure only).

The reference stores one code per byte (src/kvquant/compact_pool.py:9-12) and
only plans bit-packing (src/kvquant/vllm_integration.md:51: ``head_size//2``
bytes for nuq4, ``//4`` for nuq2). The build pins the order:

  * nuq4: byte i = code[2i] | code[2i+1] << 4
  * nuq2: byte i = code[4i] | code[4i+1] << 2 | code[4i+2] << 4 | code[4i+3] << 6

applied along the last axis (head_dim) of a code array.
"""
from __future__ import annotations

import numpy as np


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    per = 8 // bits
    assert c.shape[-1] % per == 0
    c = c.reshape(c.shape[:-1] + (c.shape[-1] // per, per))
    out = np.zeros(c.shape[:-1], dtype=np.uint8)
    for j in range(per):
        out |= (c[..., j] & ((1 << bits) - 1)) << (bits * j)
    return out


def unpack_codes(packed: np.ndarray, bits: int) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    per = 8 // bits
    out = np.empty(p.shape + (per,), dtype=np.uint8)
    for j in range(per):
        out[..., j] = (p >> (bits * j)) & ((1 << bits) - 1)
    return out.reshape(p.shape[:-1] + (p.shape[-1] * per,))
