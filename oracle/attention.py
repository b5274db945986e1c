"""Dequantise-then-attend decode attention in float64 (test infrastructure only).

Generalises src/quest/reference.py:136-168 (``selected_attention``: softmax of
``q . K^T / sqrt(D)`` over the selected pages, times V) to grouped-query
attention: query head i reads KV head ``i // G``. The softmax is exact float64,
the reference for the build's 2e-3 max-abs tolerance.

Also restates the split-KV combine the build adds: each shard returns the
normalised output o_r and its log-sum-exp lse_r (natural log); the merged
output is sum_r exp(lse_r - M) o_r / sum_r exp(lse_r - M), M = max_r lse_r.
"""
from __future__ import annotations

import math

import numpy as np


def decode_attention(q, K, V, token_mask=None, scale=None):
    """q (Hq, D); K, V (N, H, D); token_mask (H, N) bool or None.

    Returns (o (Hq, D) float64, lse (Hq,) float64 natural log). Heads whose
    mask is empty get o = 0 and lse = -inf.
    """
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    hq, d = q.shape
    n, h, _ = K.shape
    g = hq // h
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    o = np.zeros((hq, V.shape[-1]))
    lse = np.full(hq, -np.inf)
    for i in range(hq):
        kv = i // g
        m = np.ones(n, bool) if token_mask is None else np.asarray(token_mask[kv], bool)
        if not m.any():
            continue
        s = (K[m, kv] @ q[i]) * scale
        mx = s.max()
        p = np.exp(s - mx)
        tot = p.sum()
        o[i] = (p @ V[m, kv]) / tot
        lse[i] = mx + math.log(tot)
    return o, lse


def page_mask_to_token_mask(selected_pages_per_head, n_tokens, page_size):
    """(H lists of logical page ids) -> (H, n_tokens) bool."""
    h = len(selected_pages_per_head)
    m = np.zeros((h, n_tokens), bool)
    for kv, pages in enumerate(selected_pages_per_head):
        for p in pages:
            a = int(p) * page_size
            m[kv, a:min(a + page_size, n_tokens)] = True
    return m


def merge_partials(o_parts, lse_parts):
    """(R, Hq, D), (R, Hq) -> merged (Hq, D), (Hq,). Empty shards have lse=-inf."""
    o_parts = np.asarray(o_parts, np.float64)
    lse_parts = np.asarray(lse_parts, np.float64)
    M = lse_parts.max(axis=0)
    Mz = np.where(np.isfinite(M), M, 0.0)
    w = np.exp(lse_parts - Mz[None])
    w = np.where(np.isfinite(lse_parts), w, 0.0)
    tot = w.sum(axis=0)
    o = (w[..., None] * o_parts).sum(axis=0) / np.where(tot > 0, tot, 1.0)[:, None]
    lse = np.where(tot > 0, Mz + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    return o, lse
