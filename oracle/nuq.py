"""nuq quantisation restated in numpy (test infrastructure only).

Follows the reference:
  * ``round_to_nearest_pole``  src/kvquant/nuq.py:22-38
  * ``find_outliers``          src/kvquant/nuq.py:41-94
  * ``quantize_nuq``           src/kvquant/nuq.py:97-132
  * ``dequantize_nuq``         src/kvquant/nuq.py:135-156
  * GPU rule for the code: fp32 |x - pole|, strict ``<`` over levels in order,
    so the first minimum wins (src/kvquant/triton_batched.py:65-72,
    src/kvquant/compact_pool.py:258-268).
"""
from __future__ import annotations

import numpy as np


def nearest_codes(values: np.ndarray, poles: np.ndarray) -> np.ndarray:
    """Index of the nearest pole, computed as the reference's GPU kernels do.

    ``values`` has shape ``S``; ``poles`` broadcasts to ``S + (L,)``. Both are
    converted to float32 first; the difference is rounded to float32 and the
    lowest level index wins ties (numpy ``argmin`` returns the first
    occurrence, like the strict ``<`` scan in triton_batched.py:70). A NaN
    value keeps code 0, as the scan does (no diff compares below +inf).
    """
    v = np.asarray(values, dtype=np.float32)
    p = np.asarray(poles, dtype=np.float32)
    diff = np.abs(v[..., None] - p)
    # NaN diffs never win the strict-< scan: replace them by +inf so argmin
    # picks the first finite minimum, or 0 when everything is inf/NaN.
    diff = np.where(np.isnan(diff), np.float32(np.inf), diff)
    codes = np.argmin(diff, axis=-1)
    # a row whose every diff is +inf keeps code 0 in the scan; argmin agrees.
    return codes.astype(np.uint8)


def band_outliers(values: np.ndarray, upper: np.ndarray, lower: np.ndarray) -> np.ndarray:
    """``(x < lower) | (x > upper)`` (nuq.py:72), compared in float32.

    fp16 operands convert exactly to float32, so this equals the fp16
    comparison the reference makes.
    """
    v = np.asarray(values, dtype=np.float32)
    return (v < np.asarray(lower, dtype=np.float32)) | (v > np.asarray(upper, dtype=np.float32))


def round_to_nearest_pole(values: np.ndarray, poles: np.ndarray) -> np.ndarray:
    """nuq.py:22-38: the pole value at the nearest-pole code."""
    codes = nearest_codes(values, poles)
    p = np.broadcast_to(poles, np.asarray(values).shape + (np.asarray(poles).shape[-1],))
    return np.take_along_axis(p, codes[..., None].astype(np.int64), axis=-1)[..., 0]


def cap_outlier_mask(values, upper, lower, mask, cap: int) -> np.ndarray:
    """nuq.py:74-87 with a pinned tie rule.

    The reference keeps the ``cap`` largest ``|normalised| * mask`` entries per
    row with ``torch.topk`` (tie order unspecified). Here ties are broken by
    the lower index. Computation is in float32.
    """
    v = np.asarray(values, dtype=np.float32)
    up = np.asarray(upper, dtype=np.float32)
    lo = np.asarray(lower, dtype=np.float32)
    zp = (up + lo) / np.float32(2)
    half = np.maximum((up - lo) / np.float32(2), np.float32(1e-8))
    mag = np.abs((v - zp) / half) * mask.astype(np.float32)
    mag = np.broadcast_to(mag, v.shape)
    n = mag.shape[-1]
    k = min(cap, n)
    flat = mag.reshape(-1, n)
    out = np.zeros_like(flat, dtype=bool)
    idx = np.arange(n)
    for r in range(flat.shape[0]):
        order = np.lexsort((idx, -flat[r]))
        out[r, order[:k]] = True
    return out.reshape(mag.shape)


def find_outliers(values, upper, lower, cap_outliers: int = -1,
                  first_few_fp16: int = -1, seq_dim: int = -2) -> np.ndarray:
    """nuq.py:41-94 (band test, optional cap, optional first-N rows)."""
    mask = np.broadcast_to(band_outliers(values, upper, lower), np.asarray(values).shape).copy()
    if cap_outliers > 0:
        mask = cap_outlier_mask(values, upper, lower, mask, cap_outliers)
    if first_few_fp16 > 0:
        idx = [slice(None)] * mask.ndim
        idx[seq_dim] = slice(0, first_few_fp16)
        mask[tuple(idx)] = True
    return mask


def quantize_nuq(values, poles, upper, lower, cap_outliers: int = -1,
                 first_few_fp16: int = -1, seq_dim: int = -2):
    """nuq.py:97-132: ``(where(mask, x, pole[code]), mask)``."""
    mask = find_outliers(values, upper, lower, cap_outliers, first_few_fp16, seq_dim)
    q = round_to_nearest_pole(values, poles)
    v = np.asarray(values)
    return np.where(mask, v, q.astype(v.dtype)), mask


def dequantize_nuq(codes, outliers, outlier_mask, poles):
    """nuq.py:135-156: ``where(mask, outliers, poles[code])``."""
    c = np.asarray(codes).astype(np.int64)
    p = np.broadcast_to(poles, c.shape + (np.asarray(poles).shape[-1],))
    rec = np.take_along_axis(p, c[..., None], axis=-1)[..., 0]
    o = np.asarray(outliers)
    return np.where(outlier_mask, o, rec.astype(o.dtype))


# --- dense (T, H, D) pack / unpack, the reference's batched Triton API ----------

def pack_keys_per_channel(values, poles, upper, lower):
    """triton_batched.py:28-82 / :125-148: K with per-channel poles (H, D, L).

    Returns ``(codes u8, outlier_v fp16, outlier_m u8)``, each (T, H, D).
    """
    v = np.asarray(values, dtype=np.float16)
    codes = nearest_codes(v, np.asarray(poles)[None])
    m = band_outliers(v, np.asarray(upper)[None], np.asarray(lower)[None])
    outv = np.where(m, v, np.float16(0)).astype(np.float16)
    return codes, outv, m.astype(np.uint8)


def pack_values_per_token(values, poles, upper, lower):
    """triton_batched.py:179-232 / :275-303: V with per-token poles (H, T, L)."""
    v = np.asarray(values, dtype=np.float16)               # (T, H, D)
    p = np.transpose(np.asarray(poles), (1, 0, 2))         # (T, H, L)
    codes = nearest_codes(v, p[:, :, None, :])
    up = np.transpose(np.asarray(upper))[:, :, None]       # (T, H, 1)
    lo = np.transpose(np.asarray(lower))[:, :, None]
    m = band_outliers(v, up, lo)
    outv = np.where(m, v, np.float16(0)).astype(np.float16)
    return codes, outv, m.astype(np.uint8)


def unpack_keys_per_channel(codes, outv, outm, poles):
    """triton_batched.py:85-122: dequantise K, fp16 output."""
    p = np.broadcast_to(np.asarray(poles)[None], codes.shape + (np.asarray(poles).shape[-1],))
    rec = np.take_along_axis(p, codes[..., None].astype(np.int64), axis=-1)[..., 0]
    return np.where(outm != 0, outv, rec).astype(np.float16)


def unpack_values_per_token(codes, outv, outm, poles):
    """triton_batched.py:235-272: dequantise V with per-token poles (H, T, L)."""
    p = np.transpose(np.asarray(poles), (1, 0, 2))[:, :, None, :]
    p = np.broadcast_to(p, codes.shape + (p.shape[-1],))
    rec = np.take_along_axis(p, codes[..., None].astype(np.int64), axis=-1)[..., 0]
    return np.where(outm != 0, outv, rec).astype(np.float16)
