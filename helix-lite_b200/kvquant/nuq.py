"""nuq quantisation API of src/kvquant/nuq.py, computed by CUDA kernels.

Same signatures and broadcasting as the reference:
  * ``round_to_nearest_pole(values, poles)``                 nuq.py:22-38
  * ``find_outliers(values, upper, lower, cap, first_few, seq_dim)``  :41-94
  * ``quantize_nuq(values, poles, upper, lower, ...)``       :97-132
  * ``dequantize_nuq(codes, outliers, outlier_mask, poles)`` :135-156

Inputs must be CUDA tensors (fp32 or fp16); there is no CPU path. Broadcast
operands are expanded on the device, then one flat kernel does the work.
Differences |x - pole| are rounded in the input dtype, as torch does, so the
nearest pole (lowest index on ties) equals the reference's. With
``cap_outliers`` ties in deviation go to the lower index (the reference's
``torch.topk`` leaves that order unspecified).
"""
from __future__ import annotations

import torch

import hxlib
from hxlib import call, ptr, stream

_DT = {torch.float32: 0, torch.float16: 1}


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"nuq kernels take float32 or float16, got {t.dtype}")
    return _DT[t.dtype]


def _quantize(values, poles, upper, lower, cap_outliers=-1, first_few_fp16=-1, seq_dim=-2):
    hxlib.require_cuda(values, poles, upper, lower)
    dt = values.dtype
    _dtype_code(values)
    shape = values.shape
    L = poles.shape[-1]
    p = poles.to(dt).expand(*shape, L).contiguous()
    up = upper.to(dt).expand(shape).contiguous()
    lo = lower.to(dt).expand(shape).contiguous()
    v = values.contiguous()
    n = v.numel()
    recon = torch.empty_like(v)
    mask = torch.empty(shape, dtype=torch.uint8, device=v.device)
    row = shape[-1] if len(shape) else 1
    scratch = torch.empty(n, dtype=torch.uint8, device=v.device) if cap_outliers > 0 else None
    seq_stride, seq_size, ff = 1, 1, 0
    if first_few_fp16 > 0:
        sd = seq_dim % len(shape)
        seq_size = shape[sd]
        seq_stride = 1
        for s in shape[sd + 1:]:
            seq_stride *= s
        ff = int(first_few_fp16)
    with torch.cuda.device(v.device):
        call("hx_nuq_quantize_flat", stream(v.device), _dtype_code(v), ptr(v), ptr(p), ptr(up), ptr(lo), n, L,
             int(cap_outliers), row, seq_stride, seq_size, ff, ptr(recon), ptr(mask), ptr(scratch))
    return recon, mask.bool()


def find_outliers(values, upper_threshold, lower_threshold, cap_outliers: int = -1,
                  first_few_fp16: int = -1, seq_dim: int = -2):
    """Boolean outlier mask (nuq.py:41-94)."""
    poles = values.unsqueeze(-1)  # any single level: the mask does not depend on it
    _, mask = _quantize(values, poles, upper_threshold, lower_threshold, cap_outliers, first_few_fp16, seq_dim)
    return mask


def round_to_nearest_pole(values, poles):
    """Pole value nearest to each element (nuq.py:22-38)."""
    inf = torch.full((), float("inf"), dtype=values.dtype, device=values.device)
    recon, _ = _quantize(values, poles, inf, -inf)
    return recon


def quantize_nuq(values, poles, upper_threshold, lower_threshold, cap_outliers: int = -1,
                 first_few_fp16: int = -1, seq_dim: int = -2):
    """``(where(mask, values, nearest pole), mask)`` (nuq.py:97-132)."""
    return _quantize(values, poles, upper_threshold, lower_threshold, cap_outliers, first_few_fp16, seq_dim)


def dequantize_nuq(codes, outliers, outlier_mask, poles):
    """``where(mask, outliers, poles[code])`` in the dtype of ``outliers`` (nuq.py:135-156)."""
    hxlib.require_cuda(codes, outliers, outlier_mask, poles)
    dt = outliers.dtype
    shape = codes.shape
    L = poles.shape[-1]
    c = codes.to(torch.int64).contiguous()
    o = outliers.expand(shape).contiguous()
    m = outlier_mask.to(torch.uint8).expand(shape).contiguous()
    p = poles.to(dt).expand(*shape, L).contiguous()
    out = torch.empty(shape, dtype=dt, device=c.device)
    with torch.cuda.device(c.device):
        call("hx_nuq_dequantize_flat", stream(c.device), _dtype_code(o), ptr(c), ptr(o), ptr(m), ptr(p),
             c.numel(), L, ptr(out), ptr(hxlib.err_word(c.device)))
    return out
