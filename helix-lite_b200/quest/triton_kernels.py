"""Import-compatible module name for src/quest/triton_kernels.py.

``page_upper_bound_triton`` keeps the reference's fp16 output
(triton_kernels.py:57) on top of the CUDA bound kernel; no Triton is involved.
"""
from __future__ import annotations

import torch

from .reference import page_upper_bound


def page_upper_bound_triton(query: torch.Tensor, K_min: torch.Tensor, K_max: torch.Tensor) -> torch.Tensor:
    if query.dim() != 2 or K_min.dim() != 3 or K_max.shape != K_min.shape:
        raise ValueError(
            f"shape mismatch: query={tuple(query.shape)}, K_min={tuple(K_min.shape)}, K_max={tuple(K_max.shape)}")
    return page_upper_bound(query.to(torch.float16), K_min.to(torch.float16), K_max.to(torch.float16)).to(
        torch.float16)
