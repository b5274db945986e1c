"""Quest page scoring and top-K selection restated in numpy (test infra only).

Follows the reference:
  * ``compute_page_stats``     src/quest/reference.py:38-56
  * ``page_upper_bound``       src/quest/reference.py:59-93
    (``q+ . kmax + q- . kmin`` summed over head_dim)
  * ``topk_pages_with_sinks``  src/quest/reference.py:96-133
  * GQA contraction            src/kvquant/compact_backend.py:225-231 (mean of
    the group queries) and BASELINE config 2 (sum of per-query-head bounds)
  * ``select_top_blocks_for_layer`` src/kvquant/quest_selector.py:38-90

Pinned arithmetic (so selection can be compared bit-exactly):
  * group terms, float32, sequential over the G group heads:
      sum mode:  Qp[d] = sum_g (q_gd > 0 ? q_gd : 0),  Qn[d] = sum_g (q_gd < 0 ? q_gd : 0)
      mean mode: m[d] = fp16((sum_g q_gd) / G);  Qp = m > 0 ? m : 0;  Qn = m < 0 ? m : 0
  * score of one (page, kv head): 32 lanes, lane l owns channels
    d = V*l + j (V = ceil(D/32), j = 0..V-1, d < D); each lane runs
      acc = 0; for j: acc = acc + Qp[d]*kmax[d]; acc = acc + Qn[d]*kmin[d]
    with every product and sum rounded to float32 (no fused multiply-add),
    then a butterfly: for m in 16, 8, 4, 2, 1: acc = acc + acc[lane ^ m].
  * order key: k32 = orderable_bits(score + 0.0f), NaN -> 0; larger is better;
    equal keys rank the lower page index first.
  * selection: the first ``sinks = min(sink_pages, n)`` pages always; the best
    ``k_eff = min(k, n - sinks)`` of the others; output ascending.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def compute_page_stats(K_pages):
    """reference.py:38-56: amin / amax over the slot axis of (P, S, H, D)."""
    K = np.asarray(K_pages)
    if K.ndim != 4:
        raise ValueError("expected (P, page, H, D)")
    return K.min(axis=1), K.max(axis=1)


def group_terms(q, group: int, mode: str = "sum"):
    """(Hq, D) query -> (Qp, Qn), each (Hq // group, D) float32."""
    q = np.asarray(q).astype(F32)
    hq, d = q.shape
    h = hq // group
    qg = q.reshape(h, group, d)
    if mode == "sum":
        qp = np.zeros((h, d), F32)
        qn = np.zeros((h, d), F32)
        for g in range(group):
            x = qg[:, g]
            qp = (qp + np.where(x > 0, x, F32(0))).astype(F32)
            qn = (qn + np.where(x < 0, x, F32(0))).astype(F32)
        return qp, qn
    if mode == "mean":
        s = np.zeros((h, d), F32)
        for g in range(group):
            s = (s + qg[:, g]).astype(F32)
        m = (s / F32(group)).astype(F32).astype(np.float16).astype(F32)
        return np.where(m > 0, m, F32(0)), np.where(m < 0, m, F32(0))
    raise ValueError(mode)


def page_scores(qp, qn, kmin, kmax):
    """Pinned-order bound: (H, D) terms x (P, H, D) stats -> (P, H) float32."""
    kmin = np.asarray(kmin).astype(F32)
    kmax = np.asarray(kmax).astype(F32)
    P, H, D = kmin.shape
    V = -(-D // 32)
    acc = np.zeros((P, H, 32), F32)
    for j in range(V):
        for lane in range(32):
            d = V * lane + j
            if d >= D:
                continue
            a = acc[:, :, lane]
            a = (a + (qp[None, :, d] * kmax[:, :, d]).astype(F32)).astype(F32)
            a = (a + (qn[None, :, d] * kmin[:, :, d]).astype(F32)).astype(F32)
            acc[:, :, lane] = a
    for m in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, :, np.arange(32) ^ m]).astype(F32)
    return acc[:, :, 0]


def order_keys(scores):
    """float32 scores -> uint32 keys, larger key = better page; NaN -> 0."""
    s = (np.asarray(scores, dtype=F32) + F32(0.0)).astype(F32)
    u = s.view(np.uint32)
    k = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    return np.where(np.isnan(s), np.uint32(0), k).astype(np.uint32)


def select_pages(scores_1d, k: int, sink_pages: int):
    """One head: sorted page indices = sinks + best k_eff of the rest."""
    s = np.asarray(scores_1d)
    n = s.shape[0]
    sinks = max(0, min(sink_pages, n))
    k_eff = max(0, min(k, n - sinks))
    keys = order_keys(s).astype(np.int64)
    idx = np.arange(sinks, n)
    order = np.lexsort((idx, -keys[sinks:]))   # key desc, then index asc
    chosen = idx[order[:k_eff]]
    return np.sort(np.concatenate([np.arange(sinks), chosen])).astype(np.int64)


def topk_pages_with_sinks(bound, k: int, sink_pages: int = 1):
    """reference.py:96-133 with the pinned tie rule: (sinks + k_eff, H)."""
    b = np.asarray(bound).astype(F32)
    if b.ndim != 2:
        raise ValueError("bound should be (P, H)")
    cols = [select_pages(b[:, h], k, sink_pages) for h in range(b.shape[1])]
    return np.stack(cols, axis=1)


def sharded_selection(scores_1d, n_ranks: int, frac_num: int, frac_den: int, sink_pages: int):
    """Split-KV selection: rank r owns a contiguous page range and keeps the
    best ``floor(n_r * frac)`` of its pages; rank 0 also keeps the sinks.

    Returns the union of the per-rank choices (sorted) and the per-rank lists.
    """
    n = len(scores_1d)
    bounds = shard_bounds(n, n_ranks)
    per_rank = []
    for r in range(n_ranks):
        a, b = bounds[r], bounds[r + 1]
        local = np.asarray(scores_1d[a:b])
        kr = (b - a) * frac_num // frac_den
        sinks = sink_pages if r == 0 else 0
        sel = select_pages(local, kr, sinks) + a
        per_rank.append(sel)
    return np.sort(np.concatenate(per_rank)), per_rank


def shard_bounds(n_pages: int, n_ranks: int):
    """Contiguous page ranges: rank r owns [b[r], b[r+1])."""
    base, rem = divmod(n_pages, n_ranks)
    b = [0]
    for r in range(n_ranks):
        b.append(b[-1] + base + (1 if r < rem else 0))
    return b


def keys64(scores_1d, first_page: int = 0):
    """64-bit page keys: order key << 32 | ~(global page index); larger = better."""
    k = order_keys(scores_1d).astype(np.uint64) << np.uint64(32)
    idx = (np.arange(len(scores_1d), dtype=np.int64) + first_page).astype(np.uint64)
    return k | (~idx & np.uint64(0xFFFFFFFF))


def threshold64(scores_1d, k: int, sink_pages: int) -> int:
    """The selection as one 64-bit threshold over the non-sink pages' keys:
    a page is chosen iff its key >= T (0: every page, 2^64-1: none)."""
    s = np.asarray(scores_1d)
    n = len(s)
    sinks = max(0, min(sink_pages, n))
    k_eff = max(0, min(k, n - sinks))
    if k_eff == 0:
        return (1 << 64) - 1
    if k_eff >= n - sinks:
        return 0
    keys = np.sort(keys64(s)[sinks:])[::-1]
    return int(keys[k_eff - 1])


def shard_threshold(T: int, base: int) -> int:
    """A global threshold restated for a shard whose page 0 is global page
    `base` (hx_quest_localize): keys with local indices select exactly the
    global choice's pages in the shard."""
    if T in (0, (1 << 64) - 1):
        return T
    kT, low = T >> 32, T & 0xFFFFFFFF
    if kT == 0xFFFFFFFF:
        return T
    gmax = (~low) & 0xFFFFFFFF
    if gmax < base:
        return (kT + 1) << 32
    return (kT << 32) | ((~(gmax - base)) & 0xFFFFFFFF)


def select_by_threshold(scores_1d, T: int, sink_pages: int):
    """Ascending local pages: the sinks and every other page with key >= T."""
    s = np.asarray(scores_1d)
    n = len(s)
    sinks = max(0, min(sink_pages, n))
    keys = keys64(s)
    chosen = np.nonzero(keys[sinks:] >= np.uint64(T))[0] + sinks
    return np.concatenate([np.arange(sinks), chosen]).astype(np.int64)


def global_selection_per_shard(scores_1d, n_ranks: int, k: int, sink_pages: int):
    """The single-GPU selection split at the shard bounds, as local indices."""
    sel = select_pages(scores_1d, k, sink_pages)
    b = shard_bounds(len(scores_1d), n_ranks)
    return [sel[(sel >= b[r]) & (sel < b[r + 1])] - b[r] for r in range(n_ranks)]


def slice_counts(local_sel, n: int, sinks: int, C: int):
    """Exclusive prefix (C + 1 entries) of the selected non-sink pages per
    slice of ceil((n - sinks) / C) pages (the decode's slices)."""
    n_ns = n - sinks
    per = (n_ns + C - 1) // C if n_ns > 0 else 1
    sel = np.asarray(local_sel)
    sel = sel[sel >= sinks]
    cnt = np.bincount((sel - sinks) // per, minlength=C)[:C]
    return np.concatenate([[0], np.cumsum(cnt)]).astype(np.int64)


def shard_sinks(sink_pages: int, base: int, n: int) -> int:
    """The global sinks that fall on a shard of n pages starting at `base`."""
    return max(0, min(sink_pages - base, n))
