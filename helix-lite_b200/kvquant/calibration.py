"""On-device calibration statistics for nuq scales.

Mirrors the statistics step of src/kvquant/calibration.py:127-188
(``_calibrate_keys`` / ``_calibrate_values``) on the GPU: the outlier band of
every group is numpy's linear-interpolation quantile at p and 1 - p (the
same doubles the reference's ``np.quantile`` returns), and the group's
codebook is a 1-D k-means of its in-band samples, here the exact optimum
(dynamic programming over the sorted, duplicate-merged samples, or 4,096 of
them stratified by rank) refined by Lloyd steps over every in-band sample.
The reference fits sklearn's KMeans on a random subsample of 5,000; the
exact optimum never has a larger SSE than that fit. Groups are sorted on the
device and reduced by one kernel (hx_calib_rows, one CTA per group). Model loading and the prompt set (the
reference's :60-104) stay with the caller: the functions take the captured
K / V tensors.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

import hxlib

from .scales import PerChannelScale, PerTokenScale


@dataclass
class CalibrationConfig:
    """The statistics fields of the reference's CalibrationConfig
    (calibration.py:45-60); ``max_iter`` bounds Lloyd's iterations (the
    reference's KMeans max_iter)."""
    num_bits: int = 2
    outlier_pct: float = 0.005
    max_iter: int = 20


def calibrate_rows(rows: torch.Tensor, num_levels: int, outlier_pct: float, max_iter: int = 20):
    """rows (R, n) float32 on the GPU, one group per row -> (lower (R,),
    upper (R,), centres (R, num_levels) sorted, iterations (R,)) float32."""
    if not rows.is_cuda:
        raise hxlib.HelixError("calibrate_rows needs a CUDA tensor")
    if rows.dim() != 2 or rows.shape[1] < 1:
        raise ValueError("rows must be (groups, samples)")
    dev = rows.device
    R, n = rows.shape
    srt = torch.sort(rows.to(torch.float32).contiguous(), dim=1).values
    lower = torch.empty((R,), dtype=torch.float32, device=dev)
    upper = torch.empty((R,), dtype=torch.float32, device=dev)
    cent = torch.empty((R, num_levels), dtype=torch.float32, device=dev)
    its = torch.empty((R,), dtype=torch.int32, device=dev)
    nbytes = int(hxlib.lib().hx_calib_scratch_bytes(R, n))
    prefix = torch.empty((nbytes // 8,), dtype=torch.float64, device=dev)
    with torch.cuda.device(dev):
        hxlib.call("hx_calib_rows", hxlib.stream(dev), hxlib.ptr(srt), R, n, float(outlier_pct),
                   float(1.0 - outlier_pct), int(num_levels), int(max_iter), hxlib.ptr(lower), hxlib.ptr(upper),
                   hxlib.ptr(cent), hxlib.ptr(prefix), hxlib.ptr(its))
    return lower, upper, cent, its


def calibrate_keys(K_concat: torch.Tensor, cfg: CalibrationConfig) -> PerChannelScale:
    """K_concat (total_tokens, H, D): one group per (head, channel) over the
    tokens (calibration.py:127-155)."""
    T, H, D = K_concat.shape
    rows = K_concat.permute(1, 2, 0).reshape(H * D, T)
    lo, up, c, _ = calibrate_rows(rows, 2 ** cfg.num_bits, cfg.outlier_pct, cfg.max_iter)
    return PerChannelScale(poles=c.view(H, D, -1), upper_threshold=up.view(H, D), lower_threshold=lo.view(H, D),
                           num_bits=cfg.num_bits)


def calibrate_values(V_stack: torch.Tensor, cfg: CalibrationConfig) -> PerTokenScale:
    """V_stack (num_prompts, seqlen, H, D): one group per (head, position)
    over prompts x channels (calibration.py:158-188)."""
    P, T, H, D = V_stack.shape
    rows = V_stack.permute(2, 1, 0, 3).reshape(H * T, P * D)
    lo, up, c, _ = calibrate_rows(rows, 2 ** cfg.num_bits, cfg.outlier_pct, cfg.max_iter)
    return PerTokenScale(poles=c.view(H, T, -1), upper_threshold=up.view(H, T), lower_threshold=lo.view(H, T),
                         num_bits=cfg.num_bits)
