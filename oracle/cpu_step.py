"""One layer of the decode step on CPU, vectorised numpy (test infrastructure).

The timed CPU baseline of bench.py (its ``cpu_baseline`` leg and the
``--impl reference`` arm). Same algorithm as the reference path, stated in
oracle/quest.py and oracle/attention.py:
  1. page bounds from the fp16 K min / max of every page (reference.py:59-93,
     GQA sum over the group; pinned fp32 order),
  2. per KV head: the sinks + best k pages (reference.py:96-133),
  3. dequantise the selected pages: codes -> poles, outliers patched
     (compact_pool.py:293-395),
  4. softmax(q K^T / sqrt(D)) V over them, grouped-query (reference.py:136-168).
Inputs are the packed pool arrays of one layer copied to host.
"""
from __future__ import annotations

import math

import numpy as np

from .packing import unpack_codes
from .quest import group_terms, page_scores, select_pages


class HostLayer:
    """Host copy of one pool layer for a sequence of n pages (pages 0..n-1)."""

    def __init__(self, k_rows, v_rows, stats, k_out, v_out, k_poles, v_poles, bits_k, bits_v, t_cal):
        self.k_rows, self.v_rows = k_rows, v_rows          # (H, n, S, RB) uint8
        self.stats = stats                                 # (H, n, 2, D) fp16
        self.k_out, self.v_out = k_out, v_out              # (H, n) lists of (slot, d, value) arrays
        self.k_poles, self.v_poles = k_poles, v_poles      # (H, D, L), (H, Tc, L) fp16
        self.bits_k, self.bits_v, self.t_cal = bits_k, bits_v, t_cal


def algorithmic_bytes(layer: HostLayer, pages_per_head, hq: int, D: int) -> int:
    """Bytes the step must read / write for this layer (bench roofline unit)."""
    H, n = layer.stats.shape[:2]
    b = H * n * 2 * D * 2                       # stats scan
    seg = layer.k_rows.shape[2] * (layer.k_rows.shape[3] + layer.v_rows.shape[3])
    for h in range(H):
        for p in pages_per_head[h]:
            b += seg + 32 + 4 * (len(layer.k_out[h][p][0]) + len(layer.v_out[h][p][0]))
    b += hq * D * 2 + hq * D * 4 + hq * 4       # q in, o and lse out
    return b


def decode_layer(layer: HostLayer, q, seq_len: int, group: int, k_frac=(1, 4), sinks: int = 4):
    """(o (Hq, D) float32, selected pages per head) for one decode token."""
    H, n, S, _ = layer.k_rows.shape
    D = layer.stats.shape[-1]
    kmin = layer.stats[:, :, 0].transpose(1, 0, 2)
    kmax = layer.stats[:, :, 1].transpose(1, 0, 2)
    qp, qn = group_terms(q, group, "sum")
    sc = page_scores(qp, qn, kmin, kmax)
    k = n * k_frac[0] // k_frac[1]
    o = np.zeros((H * group, D), np.float32)
    chosen = []
    for h in range(H):
        pages = select_pages(sc[:, h], k, sinks)
        chosen.append(pages)
        kc = unpack_codes(layer.k_rows[h, pages], layer.bits_k).astype(np.int64)     # (m, S, D)
        vc = unpack_codes(layer.v_rows[h, pages], layer.bits_v).astype(np.int64)
        Kd = layer.k_poles[h][np.arange(D)[None, None, :], kc]                        # (m, S, D)
        pos = np.minimum(pages[:, None] * S + np.arange(S)[None, :], layer.t_cal - 1)  # (m, S)
        Vd = np.take_along_axis(layer.v_poles[h][pos], vc, axis=-1)
        for i, p in enumerate(pages):
            for arr, lst in ((Kd, layer.k_out[h][p]), (Vd, layer.v_out[h][p])):
                if len(lst[0]):
                    arr[i, lst[0], lst[1]] = lst[2]
        Kf = Kd.reshape(-1, D).astype(np.float32)
        Vf = Vd.reshape(-1, D).astype(np.float32)
        valid = (pages[:, None] * S + np.arange(S)[None, :]).reshape(-1) < seq_len
        qh = q[h * group:(h + 1) * group].astype(np.float32)
        s = (qh @ Kf.T) * np.float32(1.0 / math.sqrt(D))
        s[:, ~valid] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        o[h * group:(h + 1) * group] = (p @ Vf) / p.sum(axis=1, keepdims=True)
    return o, chosen
