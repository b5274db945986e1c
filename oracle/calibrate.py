"""Calibration statistics restated in numpy (TEST INFRASTRUCTURE ONLY: the
tests compare hx_calib_rows with it; nothing of the product imports it).

The band follows xFuzzitx/helix-lite src/kvquant/calibration.py:139-142 /
:176-179 literally (``np.quantile`` of the group's float32 samples at p and
1 - p, the samples with lo <= x <= up kept). The codebook is the algorithm
the device kernel runs: the exact (globally optimal) 1-D k-means of the
in-band samples, or of 4,096 of them stratified by rank, by dynamic
programming over the sorted, duplicate-merged points (split points searched
middle-first, the smallest optimal split on ties), then Lloyd steps over
every in-band sample. The reference fits sklearn's KMeans (k-means++, 3
starts, 20 iterations) on a random subsample of 5,000 (calibration.py:106-125,
143-147), which no other implementation reproduces sample for sample; the
tests hold this oracle to sklearn's SSE. Groups with fewer in-band samples
than levels follow the reference's padding rule (:117-122).
"""
from __future__ import annotations

import numpy as np


def band(vals, pct: float):
    """(lower, upper) as the reference computes them (Python floats)."""
    v = np.asarray(vals, dtype=np.float32)
    return float(np.quantile(v, pct)), float(np.quantile(v, 1 - pct))


DP_MAX = 4096   # points the exact k-means runs on (rank-stratified beyond)


def _points(x_sorted):
    """The exact k-means' points: every sample, or DP_MAX stratified by rank,
    equal values merged; returns values, and the sequential prefix sums of
    count, sum and square sum (float64, in order)."""
    m = x_sorted.size
    if m > DP_MAX:
        idx = ((2 * np.arange(DP_MAX, dtype=np.int64) + 1) * m) // (2 * DP_MAX)
        p = x_sorted[idx]
    else:
        p = x_sorted
    vals, counts = [], []
    for v in p.astype(np.float32):
        if not vals or v != vals[-1]:
            vals.append(v)
            counts.append(0)
        counts[-1] += 1
    W, S1, S2 = [0.0], [0.0], [0.0]
    w = s1 = s2 = 0.0
    for v, c in zip(vals, counts):
        dv = float(v)
        for _ in range(c):          # the device adds sample by sample
            w += 1.0
            s1 += dv
            s2 += dv * dv
        W.append(w)
        S1.append(s1)
        S2.append(s2)
    return np.array(vals, np.float64), np.array(W), np.array(S1), np.array(S2)


def _cost(W, S1, S2, s, e):
    n, sm, ss = W[e] - W[s], S1[e] - S1[s], S2[e] - S2[s]
    return ss - (sm * sm) / n


def exact_kmeans_points(vals, W, S1, S2, k: int):
    """Optimal 1-D k-means of weighted points (k < len(vals)): centres as the
    clusters' weighted means, ascending. Split points: the smallest optimal,
    searched middle-first over a segment tree as the device does."""
    U = len(vals)
    dprev = np.array([_cost(W, S1, S2, 0, i) if i >= 1 else 0.0 for i in range(U + 1)])
    T = np.zeros((k + 1, U + 1), np.int64)
    for j in range(2, k + 1):
        dcur = np.full(U + 1, np.inf)
        tj = T[j]
        R_lo, R_hi = j, U

        # level by level, as the device
        for lvl in range(14):
            for seg in range(1 << lvl):
                lo, hi = R_lo, R_hi
                for bit in range(lvl - 1, -1, -1):
                    if lo > hi:
                        break
                    mid = (lo + hi) >> 1
                    if (seg >> bit) & 1:
                        lo = mid + 1
                    else:
                        hi = mid - 1
                if lo > hi:
                    continue
                mid = (lo + hi) >> 1
                s_lo = j - 1 if lo == R_lo else int(tj[lo - 1])
                s_hi = min(mid - 1, R_hi - 1 if hi == R_hi else int(tj[hi + 1]))
                ss = np.arange(s_lo, s_hi + 1)
                n = W[mid] - W[ss]
                sm = S1[mid] - S1[ss]
                q = S2[mid] - S2[ss]
                v = dprev[ss] + (q - (sm * sm) / n)
                b = int(np.argmin(v))          # first minimum: the smallest s
                dcur[mid] = v[b]
                tj[mid] = ss[b]
        dprev = dcur
    c = np.zeros(k)
    e = U
    for j in range(k, 0, -1):
        s_ = 0 if j == 1 else int(T[j][e])
        c[j - 1] = (S1[e] - S1[s_]) / (W[e] - W[s_])
        e = s_
    return c


def kmeans_1d(mass, k: int, max_iter: int = 20):
    """Sorted centres (float64) and Lloyd steps run: the exact k-means of the
    points above, then Lloyd steps over every sample (a sample on a midpoint
    joins the lower centre; an empty cluster keeps its centre; stop when no
    centre moves). Fewer samples than k: the reference's padding rule."""
    x = np.sort(np.asarray(mass, dtype=np.float32))
    m = x.size
    if m < k:
        pad = np.zeros(k, dtype=np.float32)
        pad[:m] = x
        return np.sort(pad).astype(np.float64), 0
    vals, W, S1, S2 = _points(x)
    U = len(vals)
    if U <= k:
        c = np.array([vals[min(i, U - 1)] for i in range(k)], np.float64)
    else:
        c = exact_kmeans_points(vals, W, S1, S2, k)
    xd = x.astype(np.float64)
    pre = np.concatenate([[0.0], np.cumsum(xd)])
    it = 0
    while it < max_iter:
        mids = 0.5 * (c[:-1] + c[1:])
        cuts = np.concatenate([[0], np.searchsorted(xd, mids, side="right"), [m]])
        cnt = cuts[1:] - cuts[:-1]
        nc = c.copy()
        nz = cnt > 0
        nc[nz] = (pre[cuts[1:]] - pre[cuts[:-1]])[nz] / cnt[nz]
        if np.array_equal(nc, c):
            break
        c = nc
        it += 1
    return c, it


def calibrate_group(vals, k: int, pct: float, max_iter: int = 20):
    lo, up = band(vals, pct)
    v = np.asarray(vals, dtype=np.float32)
    mass = v[(v >= lo) & (v <= up)]
    c, it = kmeans_1d(mass, k, max_iter)
    return lo, up, c, it


def inertia(mass, centres) -> float:
    """Sum of squared distances to the nearest centre."""
    x = np.asarray(mass, dtype=np.float64)[:, None]
    return float(((x - np.asarray(centres, np.float64)[None, :]) ** 2).min(axis=1).sum())
