"""Seeded synthetic KV workloads with the shapes of the benchmark configs.

Stand-in for real Qwen2.5-7B-1M activations and calibrated scale files (the
reference's ``scales/*.pt`` are not available): K and V are N(0, 1) times a
per-channel scale drawn log-uniform in [0.1, 10], and a seeded fraction of
positions is multiplied by 10 so the outlier band catches them. Codebooks
are the sorted N(0, 1) quantiles z_l = Phi^-1((l + 0.5) / L) scaled by the
group's standard deviation; thresholds are the group quantiles at
``side`` and ``1 - side`` (the recipe of src/kvquant/calibration.py:141-142),
taken over a calibration prefix of the data.
"""
from __future__ import annotations

import torch

from .scales import KVScales, PerChannelScale, PerTokenScale


def make_kv(T: int, H: int, D: int, seed: int, outlier_frac: float = 0.01, device="cuda",
            chan_scale: torch.Tensor | None = None, chan_seed: int | None = None):
    """(K, V) fp16 (T, H, D) sampled with ``seed``. The per-channel scales
    (2, H, D) are ``chan_scale`` if given, else drawn from ``chan_seed``
    (default ``seed``); data meant for the scales of ``make_scales(seed=s)``
    layer i uses chan_seed = s + 1000 * i."""
    g = torch.Generator(device=device).manual_seed(seed)
    if chan_scale is None:
        chan_scale = channel_scales(H, D, seed if chan_seed is None else chan_seed, device)
    out = []
    for i in range(2):
        x = torch.randn((T, H, D), generator=g, device=device, dtype=torch.float32) * chan_scale[i]
        if outlier_frac > 0:
            hit = torch.rand((T, H, D), generator=g, device=device) < outlier_frac
            x = torch.where(hit, x * 10.0, x)
        out.append(x.to(torch.float16))
    return out[0], out[1]


def channel_scales(H: int, D: int, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed + 7919)
    u = torch.rand((2, H, D), generator=g, device=device)
    return torch.exp(torch.log(torch.tensor(0.1)) + u * (torch.log(torch.tensor(10.0)) - torch.log(torch.tensor(0.1))))


def codebook(levels: int, device="cuda") -> torch.Tensor:
    l = torch.arange(levels, device=device, dtype=torch.float64)
    return torch.special.ndtri((l + 0.5) / levels).to(torch.float32)


def _quantiles(x: torch.Tensor, qs, dim: int) -> torch.Tensor:
    # torch.quantile caps its input size; sort-based quantiles along one dim
    s, _ = torch.sort(x.float(), dim=dim)
    n = s.shape[dim]
    out = []
    for q in qs:
        pos = q * (n - 1)
        lo = int(pos)
        hi = min(lo + 1, n - 1)
        w = pos - lo
        a = s.select(dim, lo)
        b = s.select(dim, hi)
        out.append(a + (b - a) * w)
    return out


def layer_scales(K_cal: torch.Tensor, V_cal: torch.Tensor, levels: int, side: float, t_cal: int):
    """Scales of one layer from calibration K/V (T, H, D) (T >= t_cal)."""
    z = codebook(levels, K_cal.device)
    k = K_cal.float()
    v = V_cal[:t_cal].float()
    ks = k.std(dim=0)                                     # (H, D)
    k_poles = (ks.unsqueeze(-1) * z).to(torch.float16)    # (H, D, L), ascending
    k_lo, k_hi = _quantiles(k, (side, 1.0 - side), dim=0)
    vs = v.std(dim=2).t()                                 # (H, T_cal)
    v_poles = (vs.unsqueeze(-1) * z).to(torch.float16)    # (H, T_cal, L)
    v_lo, v_hi = _quantiles(v, (side, 1.0 - side), dim=2)  # (T_cal, H)
    return (PerChannelScale(k_poles, k_hi.to(torch.float16), k_lo.to(torch.float16), num_bits=levels.bit_length() - 1),
            PerTokenScale(v_poles, v_hi.t().contiguous().to(torch.float16), v_lo.t().contiguous().to(torch.float16),
                          num_bits=levels.bit_length() - 1))


# layer mixes of the benchmark configs: (levels, outlier fraction, band side)
NUQ4 = (16, 0.01, 0.005)
NUQ2 = (4, 0.05, 0.025)


def mixed_layout(num_layers: int = 28, cut: int = 16):
    """Layers [0, cut) nuq2, [cut, num_layers) nuq4 (benchmarks/pr1c/mix_scales.py:59-68)."""
    return [NUQ2 if i < cut else NUQ4 for i in range(num_layers)]


def make_scales(layout, H: int, D: int, t_cal: int, seed: int, device="cuda", calib_tokens: int | None = None):
    """KVScales for a list of (levels, outlier_frac, side), calibrated on a
    seeded sample of each layer's distribution."""
    keys, vals = [], []
    T = max(t_cal, calib_tokens or t_cal)
    for i, (levels, frac, side) in enumerate(layout):
        cs = channel_scales(H, D, seed + 1000 * i, device)
        K, V = make_kv(T, H, D, seed + 1000 * i, frac, device, chan_scale=cs)
        ks, vs = layer_scales(K, V, levels, side, t_cal)
        keys.append(ks)
        vals.append(vs)
    return KVScales(keys, vals, first_few_fp16=4, num_bits=4)
