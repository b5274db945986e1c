"""Quest decode-time page selection API (src/quest/reference.py), on CUDA.

Same functions, shapes and errors as the reference:
  * ``compute_page_stats(K_pages (P, S, H, D)) -> (K_min, K_max)``      :38-56
  * ``page_upper_bound(query (H, D), K_min, K_max (P, H, D)) -> (P, H)`` :59-93
  * ``topk_pages_with_sinks(bound (P, H), k, sink_pages=1)``            :96-133
  * ``selected_attention(query, K_pages, V_pages, page_indices)``       :136-168

Kernels: the pinned-order score of hx_quest_scores (fp32 products and sums,
so a bound matches the reference within fp32 rounding), the exact radix
top-k of hx_quest_threshold (ties to the lower page; ``torch.topk`` leaves
that order open) and an fp32 attention over the selected pages. Query head
i reads KV head i // (Hq // H), which reduces to the reference's per-head
loop when Hq == H. CUDA tensors only.
"""
from __future__ import annotations

import math

import torch

import hxlib
from hxlib import call, ptr, stream

_DT = {torch.float32: 0, torch.float16: 1}


def _dt(t):
    if t.dtype not in _DT:
        raise TypeError(f"expected float32 or float16, got {t.dtype}")
    return _DT[t.dtype]


def compute_page_stats(K_pages: torch.Tensor):
    if K_pages.dim() != 4:
        raise ValueError(f"expected (P, page, H, D), got {tuple(K_pages.shape)}")
    hxlib.require_cuda(K_pages)
    K = K_pages.contiguous()
    P, S, H, D = K.shape
    kmin = torch.empty((P, H, D), dtype=K.dtype, device=K.device)
    kmax = torch.empty_like(kmin)
    with torch.cuda.device(K.device):
        call("hx_page_stats", stream(K.device), _dt(K), ptr(K), P, S, H, D, ptr(kmin), ptr(kmax))
    return kmin, kmax


def _scores(query, K_min, K_max, group=1, mode=0):
    H = K_min.shape[1]
    P, _, D = K_min.shape
    dt = torch.promote_types(K_min.dtype, K_max.dtype)
    if dt not in _DT:
        dt = torch.float32
    kmin = K_min.to(dt).contiguous()
    kmax = K_max.to(dt).contiguous()
    q = query.to(torch.float16).reshape(1, H * group, D).contiguous()
    if query.dtype == torch.float32 and not torch.equal(q.reshape(query.shape).float(), query):
        # the kernels take fp16 queries; an fp32 query that is not fp16-exact
        # is scored through the fp32 group terms instead
        return _scores_fp32_query(query, kmin, kmax)
    scores = torch.empty((1, H, P), dtype=torch.float32, device=kmin.device)
    sl = torch.tensor([P], dtype=torch.int32, device=kmin.device)
    with torch.cuda.device(kmin.device):
        call("hx_quest_scores", stream(kmin.device), ptr(q), 1, H, group, D, mode, _dt(kmin), ptr(kmin), ptr(kmax),
             H * D, D, None, 0, ptr(sl), 1, P, 0, ptr(scores), None)
    return scores[0].t()


def _scores_fp32_query(query, kmin, kmax):
    # fold the query into the stats: max(q,0)*kmax + min(q,0)*kmin ==
    # 1 * (qp*kmax) + (-1) * (-(qn*kmin)) is not exact; instead score with
    # unit group terms on pre-multiplied stats (products rounded to fp32 as
    # the kernel does), then the pinned sum order.
    qp = query.clamp(min=0).float()
    qn = query.clamp(max=0).float()
    a = (kmax.float() * qp.unsqueeze(0)).contiguous()
    b = (kmin.float() * qn.unsqueeze(0)).contiguous()
    P, H, D = a.shape
    ones = torch.ones((1, H, D), dtype=torch.float16, device=a.device)
    scores = torch.empty((1, H, P), dtype=torch.float32, device=a.device)
    sl = torch.tensor([P], dtype=torch.int32, device=a.device)
    # kmax slot <- products with q+, kmin slot <- products with q- negated;
    # with unit queries Qp = 1 and Qn = 0 only the kmax slot counts, so run
    # twice and add (two pinned partial sums).
    with torch.cuda.device(a.device):
        call("hx_quest_scores", stream(a.device), ptr(ones), 1, H, 1, D, 0, 0, ptr(b), ptr(a), H * D, D, None, 0,
             ptr(sl), 1, P, 0, ptr(scores), None)
        s2 = torch.empty_like(scores)
        call("hx_quest_scores", stream(a.device), ptr(ones), 1, H, 1, D, 0, 0, ptr(a), ptr(b), H * D, D, None, 0,
             ptr(sl), 1, P, 0, ptr(s2), None)
    return (scores[0] + s2[0]).t()


def page_upper_bound(query: torch.Tensor, K_min: torch.Tensor, K_max: torch.Tensor) -> torch.Tensor:
    if query.dim() != 2:
        raise ValueError(f"query should be (H, D), got {tuple(query.shape)}")
    if K_min.shape != K_max.shape or K_min.dim() != 3:
        raise ValueError(
            f"K_min/K_max should be (P, H, D), got {tuple(K_min.shape)} and {tuple(K_max.shape)}")
    hxlib.require_cuda(query, K_min, K_max)
    out_dt = torch.promote_types(query.dtype, torch.promote_types(K_min.dtype, K_max.dtype))
    return _scores(query, K_min, K_max).to(out_dt)


def topk_pages_with_sinks(bound: torch.Tensor, k: int, sink_pages: int = 1) -> torch.Tensor:
    if bound.dim() != 2:
        raise ValueError(f"bound should be (P, H), got {tuple(bound.shape)}")
    hxlib.require_cuda(bound)
    P, H = bound.shape
    dev = bound.device
    sinks = max(0, min(sink_pages, P))
    k_eff = max(0, min(k, P - sinks))
    if k_eff == 0:
        return torch.arange(sinks, device=dev).unsqueeze(1).expand(-1, H)
    scores = bound.float().t().contiguous().reshape(1, H, P)
    sl = torch.tensor([P], dtype=torch.int32, device=dev)
    thresh = torch.empty((H,), dtype=torch.int64, device=dev)
    hist = hxlib.scratch(dev, "quest_hist", H * 2 * 4096 * 4)
    cand = hxlib.scratch(dev, "quest_cand", H * P * 8)
    ctr = hxlib.scratch(dev, "quest_ctr", H * 2 * 4)
    n_out = sinks + k_eff
    out = torch.empty((H, n_out), dtype=torch.int32, device=dev)
    counts = torch.empty((H,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = stream(dev)
        call("hx_quest_threshold", st, ptr(scores), 1, H, ptr(sl), 1, P, sinks, k_eff, 0, 0, 0, ptr(hist), ptr(cand),
             ptr(ctr), ptr(thresh), ptr(hxlib.err_word(dev)))
        call("hx_quest_compact", st, ptr(scores), ptr(thresh), 1, H, ptr(sl), 1, P, sinks, 0, n_out, ptr(out),
             ptr(counts))
    return out.t().to(torch.int64)


def selected_attention(query: torch.Tensor, K_pages: torch.Tensor, V_pages: torch.Tensor,
                       page_indices: torch.Tensor) -> torch.Tensor:
    hxlib.require_cuda(query, K_pages, V_pages, page_indices)
    P, S, H, D = K_pages.shape
    Hq = query.shape[0]
    if V_pages.shape[2] != H or V_pages.shape[3] != D:
        raise ValueError("V_pages must match K_pages heads and head_dim in this implementation")
    dt = query.dtype
    if dt not in _DT:
        raise TypeError(f"expected float32 or float16, got {dt}")
    q = query.contiguous()
    K = K_pages.to(dt).contiguous()
    V = V_pages.to(dt).contiguous()
    idx = page_indices.to(torch.int64).contiguous()
    k = idx.shape[0]
    if idx.shape[1] != H:
        raise ValueError(f"page_indices should be (k, H={H}), got {tuple(idx.shape)}")
    out = torch.empty((Hq, D), dtype=dt, device=q.device)
    with torch.cuda.device(q.device):
        call("hx_selected_attention", stream(q.device), _DT[dt], ptr(q), ptr(K), ptr(V), ptr(idx), k, P, S, H, Hq,
             D, 1.0 / math.sqrt(D), ptr(out))
    return out
