"""Dense pack / unpack API of the reference's Triton kernels, on CUDA.

Batched (T, H, D) forms, src/kvquant/triton_batched.py:
  * ``pack_keys_per_channel_batched(values, poles (H, D, L), upper, lower)``  :125-148
  * ``unpack_keys_per_channel_batched(codes, outlier_v, outlier_m, poles)``  :151-171
  * ``pack_values_per_token_batched(values, poles (H, T, L), upper, lower)`` :275-303
  * ``unpack_values_per_token_batched(codes, outlier_v, outlier_m, poles)``  :306-326
Per-head (T, D) forms, src/kvquant/triton_kernels.py:96-339:
  * ``pack_keys_per_channel`` / ``unpack_keys_per_channel`` (poles (D, L))
  * ``pack_values_per_token`` / ``unpack_values_per_token`` (poles (T, L))

Outputs match the reference bit for bit: uint8 codes (nearest pole by fp32
|x - pole|, first level on ties), fp16 outlier values (0 elsewhere) and a
uint8 outlier mask.
"""
from __future__ import annotations

import torch

import hxlib
from hxlib import call, ptr, stream


def _pack(mode, values, poles, upper, lower):
    if not values.is_cuda or values.dtype != torch.float16:
        raise AssertionError("values must be a CUDA float16 tensor")
    if not values.is_contiguous():
        raise AssertionError("values must be contiguous (T, H, D)")
    T, H, D = values.shape
    L = poles.shape[-1]
    if mode == 1 and tuple(poles.shape) != (H, T, L):
        raise AssertionError(f"poles shape {tuple(poles.shape)} != ({H},{T},{L})")
    p = poles.to(torch.float16).contiguous()
    up = upper.to(torch.float16).contiguous()
    lo = lower.to(torch.float16).contiguous()
    hxlib.require_cuda(p, up, lo)
    codes = torch.empty((T, H, D), dtype=torch.uint8, device=values.device)
    outv = torch.empty((T, H, D), dtype=torch.float16, device=values.device)
    outm = torch.empty((T, H, D), dtype=torch.uint8, device=values.device)
    with torch.cuda.device(values.device):
        call("hx_nuq_pack_dense", stream(values.device), mode, ptr(values), ptr(p), ptr(up), ptr(lo), T, H, D, L,
             ptr(codes), ptr(outv), ptr(outm))
    return codes, outv, outm


def _unpack(mode, codes, outlier_v, outlier_m, poles):
    if not codes.is_cuda or codes.dtype != torch.uint8:
        raise AssertionError("codes must be a CUDA uint8 tensor")
    if not codes.is_contiguous():
        raise AssertionError("codes must be contiguous")
    T, H, D = codes.shape
    L = poles.shape[-1]
    ov = outlier_v.to(torch.float16).contiguous()
    om = outlier_m.to(torch.uint8).contiguous()
    p = poles.to(torch.float16).contiguous()
    out = torch.empty((T, H, D), dtype=torch.float16, device=codes.device)
    with torch.cuda.device(codes.device):
        call("hx_nuq_unpack_dense", stream(codes.device), mode, ptr(codes), ptr(ov), ptr(om), ptr(p), T, H, D, L,
             ptr(out))
    return out


def pack_keys_per_channel_batched(values, poles, upper, lower):
    return _pack(0, values, poles, upper, lower)


def unpack_keys_per_channel_batched(codes, outlier_v, outlier_m, poles):
    return _unpack(0, codes, outlier_v, outlier_m, poles)


def pack_values_per_token_batched(values, poles, upper, lower):
    return _pack(1, values, poles, upper, lower)


def unpack_values_per_token_batched(codes, outlier_v, outlier_m, poles):
    return _unpack(1, codes, outlier_v, outlier_m, poles)


# -- per-head (T, D) forms: a head axis of one ----------------------------------

def _one_head(fn, values, poles, upper, lower, per_token):
    v = values.unsqueeze(1).contiguous()
    p = poles.unsqueeze(0)
    c, ov, om = fn(v, p, upper.unsqueeze(0), lower.unsqueeze(0))
    return c[:, 0], ov[:, 0], om[:, 0]


def pack_keys_per_channel(values, poles, upper, lower):
    """(T, D) values, poles (D, L), thresholds (D,) (triton_kernels.py:96-172)."""
    return _one_head(pack_keys_per_channel_batched, values, poles, upper, lower, False)


def pack_values_per_token(values, poles, upper, lower):
    """(T, D) values, poles (T, L), thresholds (T,) (triton_kernels.py:258-318)."""
    return _one_head(pack_values_per_token_batched, values, poles, upper, lower, True)


def unpack_keys_per_channel(codes, outlier_v, outlier_m, poles):
    out = unpack_keys_per_channel_batched(codes.unsqueeze(1).contiguous(), outlier_v.unsqueeze(1),
                                          outlier_m.unsqueeze(1), poles.unsqueeze(0))
    return out[:, 0]


def unpack_values_per_token(codes, outlier_v, outlier_m, poles):
    out = unpack_values_per_token_batched(codes.unsqueeze(1).contiguous(), outlier_v.unsqueeze(1),
                                          outlier_m.unsqueeze(1), poles.unsqueeze(0))
    return out[:, 0]
