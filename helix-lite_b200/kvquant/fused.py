"""Quest page selection and fused-dequant decode attention over a CompactKVPool.

This is the B200 hot path that replaces, per layer and decode step,
``select_top_blocks_for_layer`` + ``unpack_to_staging`` + FlashAttention on a
fp16 staging buffer (src/kvquant/compact_backend.py:225-299):

  quest_select   page scores from the pool's fp16 K min / max (pinned fp32
                 arithmetic) and an exact per-(sequence, KV head) top-K
                 threshold: sinks + the best k pages, ties to the lower page
  decode         one decode token per sequence: the selected pages are read
                 as packed codes, dequantised on chip and attended; returns
                 normalised o (fp32) and lse (natural log)
  selected_lists the selection as ascending page lists (API / tests)

quest_select also returns, per (b, h), how many pages each slice of the
sequence contributes (the threshold kernel's blocks count them as they go),
and decode balances its splits over the selected pages with them: every CTA
gets the same number of selected pages however the selection clusters along
the sequence, and finds its pages by scanning the scores of its slices.

Everything is asynchronous on the current stream; scratch is cached per
device and left zeroed by the kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

import hxlib
from hxlib import SEL_DENSE, SEL_LIST, SEL_SLICES, SEL_THRESHOLD, call, ptr, stream

from .compact_pool import CompactKVPool, ctypes_ref

NUM_SMS = 148


@dataclass
class Selection:
    scores: torch.Tensor      # (B, H, max_pages) fp32
    thresh: torch.Tensor      # (B * H,) int64 holding uint64 thresholds
    seq_lens: torch.Tensor    # (B,) int32 tokens
    page_size: int
    max_pages: int
    sink_pages: int
    lists: torch.Tensor | None = None   # (B * H, max_pages) int32 ascending selected pages
    counts: torch.Tensor | None = None  # (B * H,) int32
    slice_off: torch.Tensor | None = None  # (B * H, slices + 1) int32 exclusive selected counts


def _i32(t, device):
    return t.to(device=device, dtype=torch.int32).contiguous()


def page_scores(pool: CompactKVPool, layer_idx: int, q: torch.Tensor, bt: torch.Tensor, sl: torch.Tensor,
                max_pages: int, sink_pages: int, scores: torch.Tensor, hist: torch.Tensor | None = None,
                gqa: str = "sum"):
    """Quest bounds of every page of each sequence into ``scores`` (B, H,
    max_pages) fp32 (one kernel); with ``hist`` also the level-1 key histogram
    the threshold kernel starts from. q (B, Hq, D) fp16 and bt / sl int32 on
    the pool's device."""
    B, Hq, D = q.shape
    H = pool.num_kv_heads
    stats = pool.layers[layer_idx].stats
    call("hx_quest_scores", stream(pool.device), ptr(q), B, H, Hq // H, D, 0 if gqa == "sum" else 1, 1,
         ptr(stats), hxlib.ctypes.c_void_p(stats.data_ptr() + 2 * D), 2 * D, pool.num_blocks * 2 * D,
         ptr(bt), bt.shape[1], ptr(sl), pool.block_size, max_pages, sink_pages, ptr(scores),
         ptr(hist) if hist is not None else None)


def quest_select(pool: CompactKVPool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, *, top_k: int | None = None, top_frac=(1, 4), sink_pages: int = 4,
                 gqa: str = "sum", max_pages: int | None = None, scores: torch.Tensor | None = None,
                 thresh: torch.Tensor | None = None, lists: bool = False,
                 list_out: tuple[torch.Tensor, torch.Tensor] | None = None,
                 slice_out: torch.Tensor | None = None) -> Selection:
    """Score every page of each sequence and fix the exact top-K thresholds.

    query (B, Hq, D) fp16 with Hq = group * H; block_table (B, >= max_pages)
    logical -> pool page; seq_lens (B,) tokens; optional preallocated
    ``scores`` (B, H, max_pages) fp32 and ``thresh`` (B*H,) int64 outputs.
    k = top_k pages if given,
    else floor(n_pages * top_frac[0] / top_frac[1]); gqa "sum" adds the
    per-query-head bounds of a group, "mean" bounds the group's mean query
    (the reference hook, compact_backend.py:231). The per-slice counts the
    decode balances over land in ``slice_out`` ((B*H, slices + 1) int32,
    slices = hx_quest_slices(max_pages)) when given. ``lists`` also writes
    the ascending page lists, into ``list_out`` = ((B*H, max_pages) int32,
    (B*H,) int32) when given.
    """
    dev = pool.device
    q = query.to(device=dev, dtype=torch.float16).contiguous()
    B, Hq, D = q.shape
    H = pool.num_kv_heads
    S = pool.block_size
    if Hq % H:
        raise ValueError("query heads must be a multiple of KV heads")
    bt = _i32(block_table, dev)
    sl = _i32(seq_lens, dev)
    mp = int(max_pages if max_pages is not None else bt.shape[1])
    if scores is None:
        scores = torch.empty((B, H, max(mp, 1)), dtype=torch.float32, device=dev)
    if thresh is None:
        thresh = torch.empty((B * H,), dtype=torch.int64, device=dev)
    hist = hxlib.scratch(dev, "quest_hist", B * H * 2 * 4096 * 4)
    cand = hxlib.scratch(dev, "quest_cand", B * H * max(mp, 1) * 8)
    ctr = hxlib.scratch(dev, "quest_ctr", B * H * 2 * 4)
    with torch.cuda.device(dev):
        st = stream(dev)
        page_scores(pool, layer_idx, q, bt, sl, mp, sink_pages, scores, hist, gqa)
        kf, fn, fd = (int(top_k), 0, 0) if top_k is not None else (0, int(top_frac[0]), int(top_frac[1]))
        nsl = int(hxlib.lib().hx_quest_slices(mp))
        if slice_out is None:
            slice_out = torch.empty((B * H, nsl + 1), dtype=torch.int32, device=dev)
        if slice_out.shape != (B * H, nsl + 1) or slice_out.dtype != torch.int32:
            raise ValueError(f"slice_out must be ({B * H}, {nsl + 1}) int32")
        call("hx_quest_threshold_slices", st, ptr(scores), B, H, ptr(sl), S, mp, sink_pages, kf, fn, fd, 1,
             ptr(hist), ptr(cand), ptr(ctr), ptr(thresh), ptr(slice_out), ptr(hxlib.err_word(dev)))
        lst = cnt = None
        if lists or list_out is not None:
            mpl = max(mp, 1)
            if list_out is not None:
                lst, cnt = list_out
            else:
                lst = torch.empty((B * H, mpl), dtype=torch.int32, device=dev)
                cnt = torch.empty((B * H,), dtype=torch.int32, device=dev)
            if lst.shape != (B * H, mpl) or cnt.shape != (B * H,) or lst.dtype != torch.int32:
                raise ValueError("list_out must be ((B*H, max_pages) int32, (B*H,) int32)")
            nch = -(-mpl // 2048)
            chunks = hxlib.scratch(dev, "quest_chunks", B * H * nch * 4)
            call("hx_quest_lists", st, ptr(scores), ptr(thresh), B, H, ptr(sl), S, mp, sink_pages, mpl, ptr(lst),
                 ptr(cnt), ptr(chunks))
    return Selection(scores, thresh, sl, S, mp, sink_pages, lst, cnt, slice_out)


def selected_lists(sel: Selection, union: bool = False, max_out: int | None = None):
    """Ascending selected logical pages: (B, H, max_out) int32 + counts (B, H);
    with union=True the union over heads: (B, max_out) + (B,)."""
    B, H, mp = sel.scores.shape
    mo = int(max_out if max_out is not None else mp)
    dev = sel.scores.device
    rows = B if union else B * H
    out = torch.full((rows, max(mo, 1)), -1, dtype=torch.int32, device=dev)
    counts = torch.empty((rows,), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        call("hx_quest_compact", stream(dev), ptr(sel.scores), ptr(sel.thresh), B, H, ptr(sel.seq_lens),
             sel.page_size, sel.max_pages, sel.sink_pages, 1 if union else 0, mo, ptr(out), ptr(counts))
    if union:
        return out, counts
    return out.view(B, H, -1), counts.view(B, H)


def default_splits(B: int, H: int, max_pages: int) -> int:
    """Splits per (sequence, head): about one decode CTA (12 warps) per SM."""
    want = max(1, math.ceil(NUM_SMS / max(1, B * H)))
    return max(1, min(want, max(1, math.ceil(max_pages / 16))))


def decode(pool: CompactKVPool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
           seq_lens: torch.Tensor, selection: Selection | None = None, *, lists: torch.Tensor | None = None,
           list_counts: torch.Tensor | None = None, page_begin: int = 0, max_pages: int | None = None,
           n_splits: int | None = None, softmax_scale: float | None = None, out16: torch.Tensor | None = None,
           o: torch.Tensor | None = None, lse: torch.Tensor | None = None, v_pos: str = "logical",
           cores: str = "tensor"):
    """Fused-dequant decode attention; returns (o (B, Hq, D) fp32, lse (B, Hq)).

    Pages attended: every page (no selection), the Quest selection (split
    over its selected pages by the selection's slice counts, else by its
    lists when it has them, else over the sequence), or explicit per-(b, h)
    logical page lists (``lists`` (B, H, L) int32 with ``list_counts`` (B,
    H)). ``page_begin`` is the absolute logical page of this pool's page 0
    (split-KV shards), used for V's position clamp. ``cores="cuda"`` runs QK
    and PV as fp32 FFMA on the CUDA cores (the comparison variant) instead of
    mma.sync on the tensor cores.
    """
    if cores not in ("tensor", "cuda"):
        raise ValueError("cores must be 'tensor' or 'cuda'")
    dev = pool.device
    q = query.to(device=dev, dtype=torch.float16).contiguous()
    B, Hq, D = q.shape
    H = pool.num_kv_heads
    bt = _i32(block_table, dev)
    sl = _i32(seq_lens, dev)
    mp = int(max_pages if max_pages is not None else bt.shape[1])
    slice_off = None
    if selection is not None and selection.slice_off is not None and lists is None:
        mp = selection.max_pages
        slice_off = selection.slice_off
        mode = SEL_SLICES
    elif selection is not None and selection.lists is not None and lists is None:
        lists, list_counts = selection.lists, selection.counts
        mode = SEL_LIST
        selection = None
    elif selection is not None:
        mp = selection.max_pages  # the scores' row stride
        mode = SEL_THRESHOLD
    elif lists is not None:
        mode = SEL_LIST
    else:
        mode = SEL_DENSE
    ns = int(n_splits or default_splits(B, H, mp if mode != SEL_LIST else lists.shape[-1]))
    scale = float(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    if o is None:
        o = torch.empty((B, Hq, D), dtype=torch.float32, device=dev)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    nbytes = hxlib.lib().hx_decode_scratch_bytes(B, H, ns)
    scr = hxlib.scratch(dev, "decode", nbytes)
    st_scales, _keep = pool.scales.device_layer(layer_idx, dev)
    if mode == SEL_LIST:
        lists_c = _i32(lists, dev).view(B * H, -1)
        counts_c = _i32(list_counts, dev)
        lstride = lists_c.shape[1]
    elif mode == SEL_SLICES:
        lists_c, counts_c = slice_off, None
        lstride = slice_off.shape[1]
    else:
        lists_c = counts_c = None
        lstride = 0
    with torch.cuda.device(dev):
        call("hx_decode_attn", stream(dev), ctypes_ref(pool.layers[layer_idx].struct), ctypes_ref(st_scales),
             ptr(q), B, Hq // H, scale, ptr(bt), bt.shape[1], ptr(sl), int(page_begin), mp,
             mode | (hxlib.VPOS_PHYSICAL if v_pos == "physical" else 0)
             | (hxlib.DECODE_CUDA_CORES if cores == "cuda" else 0),
             ptr(selection.scores) if selection is not None else None,
             ptr(selection.thresh) if selection is not None else None,
             selection.sink_pages if selection is not None else 0,
             ptr(lists_c), lstride, ptr(counts_c), ns, ptr(scr), ptr(o), ptr(lse), ptr(out16),
             ptr(hxlib.err_word(dev)))
    return o, lse


FUSED_MAX_PAGES = 16384   # rows the decode can select for itself (hx_decode_attn_select)


def quest_decode(pool: CompactKVPool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, *, top_k: int | None = None, top_frac=(1, 4), sink_pages: int = 4,
                 gqa: str = "sum", max_pages: int | None = None, scores: torch.Tensor | None = None, **kw):
    """Quest selection and fused decode in two kernels: the page scores (with
    their level-1 histogram), then the decode, whose CTAs find their row's
    exact top-K threshold themselves (hx_decode_attn_select). Same selection
    and outputs as quest_select + decode, without the threshold kernel; rows
    of at most FUSED_MAX_PAGES pages. Keyword arguments of decode_select
    pass through. Returns (o, lse)."""
    dev = pool.device
    q = query.to(device=dev, dtype=torch.float16).contiguous()
    B, Hq, D = q.shape
    H = pool.num_kv_heads
    if Hq % H:
        raise ValueError("query heads must be a multiple of KV heads")
    bt = _i32(block_table, dev)
    sl = _i32(seq_lens, dev)
    mp = int(max_pages if max_pages is not None else bt.shape[1])
    if scores is None:
        scores = torch.empty((B, H, max(mp, 1)), dtype=torch.float32, device=dev)
    hist = hxlib.scratch(dev, "quest_hist", B * H * 2 * 4096 * 4)
    with torch.cuda.device(dev):
        page_scores(pool, layer_idx, q, bt, sl, mp, sink_pages, scores, hist, gqa)
    return decode_select(pool, layer_idx, q, bt, sl, scores, top_k=top_k, top_frac=top_frac, sink_pages=sink_pages,
                         max_pages=mp, **kw)


def decode_select(pool: CompactKVPool, layer_idx: int, q: torch.Tensor, bt: torch.Tensor, sl: torch.Tensor,
                  scores: torch.Tensor, *, top_k: int | None = None, top_frac=(1, 4), sink_pages: int = 4,
                  max_pages: int | None = None, page_begin: int = 0, n_splits: int | None = None,
                  softmax_scale: float | None = None, o: torch.Tensor | None = None,
                  lse: torch.Tensor | None = None, out16: torch.Tensor | None = None, v_pos: str = "logical",
                  cores: str = "tensor", thresh_out: torch.Tensor | None = None,
                  slice_out: torch.Tensor | None = None):
    """The decode half of quest_decode: ``scores`` and the level-1 histogram
    (the "quest_hist" scratch) from page_scores; q fp16, bt / sl int32 on the
    pool's device. thresh_out (B*H,) int64 and slice_out (B*H, slices + 1)
    int32 receive the rows' thresholds and slice offsets when given."""
    dev = pool.device
    B, Hq, D = q.shape
    H = pool.num_kv_heads
    if cores not in ("tensor", "cuda"):
        raise ValueError("cores must be 'tensor' or 'cuda'")
    mp = int(max_pages if max_pages is not None else bt.shape[1])
    if mp > FUSED_MAX_PAGES:
        raise ValueError(f"decode_select selects rows of at most {FUSED_MAX_PAGES} pages; use quest_select")
    hist = hxlib.scratch(dev, "quest_hist", B * H * 2 * 4096 * 4)
    kf, fn, fd = (int(top_k), 0, 0) if top_k is not None else (0, int(top_frac[0]), int(top_frac[1]))
    ns = int(n_splits or default_splits(B, H, mp))
    scale = float(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    if o is None:
        o = torch.empty((B, Hq, D), dtype=torch.float32, device=dev)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    scr = hxlib.scratch(dev, "decode", hxlib.lib().hx_decode_scratch_bytes(B, H, ns))
    st_scales, _keep = pool.scales.device_layer(layer_idx, dev)
    flags = (hxlib.VPOS_PHYSICAL if v_pos == "physical" else 0) | (hxlib.DECODE_CUDA_CORES if cores == "cuda" else 0)
    with torch.cuda.device(dev):
        call("hx_decode_attn_select", stream(dev), ctypes_ref(pool.layers[layer_idx].struct), ctypes_ref(st_scales),
             ptr(q), B, Hq // H, scale, ptr(bt), bt.shape[1], ptr(sl), int(page_begin), mp, flags, ptr(scores),
             ptr(hist), sink_pages, kf, fn, fd, ns, ptr(scr), ptr(o), ptr(lse), ptr(out16), ptr(thresh_out),
             ptr(slice_out), ptr(hxlib.err_word(dev)))
    return o, lse


def prefill(pool: CompactKVPool, layer_idx: int, query: torch.Tensor, query_start: torch.Tensor,
            block_table: torch.Tensor, seq_lens: torch.Tensor, *, max_query_len: int | None = None,
            softmax_scale: float | None = None, v_pos: str = "logical", out: torch.Tensor | None = None,
            lse: torch.Tensor | None = None, out32: torch.Tensor | None = None):
    """Chunked-prefill attention read from the compact pool (one kernel).

    query (Tq, Hq, D) fp16: sequence b's chunk is rows query_start[b] ..
    query_start[b + 1] - 1, the last tokens of its seq_lens[b], already
    written to the pool (write_kv); each query attends causally to every
    earlier token of its sequence and to itself. Returns (out (Tq, Hq, D)
    fp16, lse (Tq, Hq) fp32 natural log); ``out32`` (Tq, Hq, D) fp32, when
    given, receives the output before its fp16 rounding. The reference's prefill reads
    vLLM's fp16 cache instead (src/kvquant/compact_backend.py:12-15).
    """
    dev = pool.device
    q = query.to(device=dev, dtype=torch.float16).contiguous()
    Tq, Hq, D = q.shape
    H = pool.num_kv_heads
    if Hq % H:
        raise ValueError("query heads must be a multiple of KV heads")
    qs = _i32(query_start, dev)
    bt = _i32(block_table, dev)
    sl = _i32(seq_lens, dev)
    B = qs.shape[0] - 1
    if max_query_len is None:
        max_query_len = int((qs[1:] - qs[:-1]).max().item()) if B > 0 else 0
    scale = float(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    if out is None:
        out = torch.empty((Tq, Hq, D), dtype=torch.float16, device=dev)
    if lse is None:
        lse = torch.empty((Tq, Hq), dtype=torch.float32, device=dev)
    st_scales, _keep = pool.scales.device_layer(layer_idx, dev)
    with torch.cuda.device(dev):
        call("hx_prefill_attn", stream(dev), ctypes_ref(pool.layers[layer_idx].struct), ctypes_ref(st_scales),
             ptr(q), ptr(qs), B, Hq // H, scale, ptr(bt), bt.shape[1], ptr(sl), int(max_query_len),
             hxlib.VPOS_PHYSICAL if v_pos == "physical" else 0, ptr(out), ptr(out32), ptr(lse),
             ptr(hxlib.err_word(dev)))
    return out, lse


def merge_partials(o_parts: torch.Tensor, lse_parts: torch.Tensor, out16: torch.Tensor | None = None):
    """Merge R shards' normalised (o, lse): (R, N, D), (R, N) -> (N, D), (N,)."""
    R, N, D = o_parts.shape
    dev = o_parts.device
    op = o_parts.to(torch.float32).contiguous()
    lp = lse_parts.to(torch.float32).contiguous()
    o = torch.empty((N, D), dtype=torch.float32, device=dev)
    lse = torch.empty((N,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        call("hx_merge_partials", stream(dev), ptr(op), ptr(lp), R, N, D, ptr(o), ptr(lse), ptr(out16))
    return o, lse
