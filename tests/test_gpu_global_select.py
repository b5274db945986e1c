"""Global top-K over split-KV shards, with the shards emulated on one GPU.

R shards' score rows are slices of one global row. The threshold kernel over
the global rows and then hx_quest_localize per shard must select, with local
page indices, exactly the oracle's single-GPU selection on each shard (ties
broken by the global page index), and write the decode's slice counts. On a
real pool the shard selections drive the decode (slice mode) and the merged
partials equal float64 attention over the single-GPU selection; the global
threshold equals the one-GPU quest_select threshold bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import make_pools, np16
from oracle import attention as oatt
from oracle import quest as oq

pytestmark = pytest.mark.gpu

S = 16


def _threshold(glob, seq, sinks, k=None, frac=(1, 4), slice_off=None):
    import hxlib
    B, H, n = glob.shape
    dev = glob.device
    thresh = torch.empty((B * H,), dtype=torch.int64, device=dev)
    hist = torch.zeros((B * H * 2 * 4096,), dtype=torch.int32, device=dev)
    cand = torch.empty((B * H * n,), dtype=torch.int64, device=dev)
    ctr = torch.zeros((B * H * 2,), dtype=torch.int32, device=dev)
    kf, fn, fd = (k, 0, 0) if k is not None else (0, frac[0], frac[1])
    hxlib.call("hx_quest_threshold_slices", hxlib.stream(dev), hxlib.ptr(glob), B, H, hxlib.ptr(seq), S, n, sinks,
               kf, fn, fd, 0, hxlib.ptr(hist), hxlib.ptr(cand), hxlib.ptr(ctr), hxlib.ptr(thresh),
               hxlib.ptr(slice_off), hxlib.ptr(hxlib.err_word(dev)))
    return thresh


def _localize(thresh_g, loc, seq_loc, sinks, begin):
    import hxlib
    B, H, n = loc.shape
    dev = loc.device
    C = int(hxlib.lib().hx_quest_slices(n))
    thresh = torch.empty((B * H,), dtype=torch.int64, device=dev)
    slice_off = torch.empty((B * H, C + 1), dtype=torch.int32, device=dev)
    hxlib.call("hx_quest_localize", hxlib.stream(dev), hxlib.ptr(thresh_g), hxlib.ptr(loc), B, H,
               hxlib.ptr(seq_loc), S, n, sinks, begin, hxlib.ptr(thresh), hxlib.ptr(slice_off))
    return thresh, slice_off, C


def _lists(loc, thresh, seq_loc, sinks):
    import hxlib
    B, H, n = loc.shape
    dev = loc.device
    out = torch.full((B * H, max(n, 1)), -1, dtype=torch.int32, device=dev)
    cnt = torch.empty((B * H,), dtype=torch.int32, device=dev)
    chunks = torch.empty((B * H * max(1, -(-n // 2048)),), dtype=torch.int32, device=dev)
    hxlib.call("hx_quest_lists", hxlib.stream(dev), hxlib.ptr(loc), hxlib.ptr(thresh), B, H, hxlib.ptr(seq_loc), S,
               n, sinks, max(n, 1), hxlib.ptr(out), hxlib.ptr(cnt), hxlib.ptr(chunks))
    return out, cnt


@pytest.mark.parametrize("P", [300, 2048, 2049, 16384, 40000])
@pytest.mark.parametrize("kind", ["randn", "ties"])
def test_threshold_slice_counts(P, kind):
    """The thresholds and the decode's slice counts of both threshold kernels
    (one CTA per row up to 2048 pages, else one per 1024 pages) against the
    oracle, with a second sequence that ends part-way."""
    import hxlib
    B, H, sinks = 2, 4, 4
    rng = np.random.default_rng(P)
    sc = rng.standard_normal((B, H, P))
    if kind == "ties":
        sc = np.round(sc * 2) / 4
    sc = sc.astype(np.float32)
    seq = np.array([P * S, (P * 2 // 3) * S - 3], dtype=np.int32)
    C = int(hxlib.lib().hx_quest_slices(P))
    so = torch.empty((B * H, C + 1), dtype=torch.int32, device="cuda")
    T = _threshold(torch.from_numpy(sc).cuda(), torch.from_numpy(seq).cuda(), sinks, slice_off=so)
    hxlib.check_device_errors("cuda")
    T, so = np16(T).view(np.uint64), np16(so)
    for b in range(B):
        nb = -(-int(seq[b]) // S)
        for h in range(H):
            want = oq.select_pages(sc[b, h, :nb], nb // 4, sinks)
            # a threshold may sit anywhere between the last page taken and the
            # next one (a bin's floor): compare what it selects
            np.testing.assert_array_equal(oq.select_by_threshold(sc[b, h, :nb], int(T[b * H + h]), sinks), want)
            np.testing.assert_array_equal(so[b * H + h], oq.slice_counts(want, nb, sinks, C))


@pytest.mark.parametrize("R,n,k,sinks,kind", [
    (2, 3000, None, 4, "randn"),     # frac 1/4 of each sequence's pages
    (4, 2048, None, 4, "ties"),      # many equal scores across shard edges
    (8, 700, 333, 4, "randn"),
    (3, 500, 0, 4, "randn"),         # k = 0: sinks only
    (5, 64, 10 ** 6, 4, "randn"),    # k >= pages: everything
    (6, 3, 5, 7, "ties"),            # the sinks spill past the first shard
    (4, 1000, None, 4, "equal"),     # one score everywhere: lowest global pages win
])
def test_localize_matches_single_gpu_selection(R, n, k, sinks, kind):
    import hxlib
    B, H = 2, 4
    rng = np.random.default_rng(R * 1000 + n)
    N = R * n
    if kind == "randn":
        sc = rng.standard_normal((B, H, N))
    elif kind == "ties":
        sc = np.round(rng.standard_normal((B, H, N)) * 2) / 4
    else:
        sc = np.ones((B, H, N))
    sc = sc.astype(np.float32)
    # sequence 1 ends part-way through shard R // 2 (a partial last page)
    seq = np.array([N * S, (R // 2) * n * S + (n // 2) * S - 5], dtype=np.int64)
    seq = np.maximum(seq, 1)
    dev = "cuda"
    glob = torch.from_numpy(sc).to(dev)
    seq_d = torch.from_numpy(seq.astype(np.int32)).to(dev)
    Tg = _threshold(glob, seq_d, sinks, k)
    for r in range(R):
        begin = r * n
        loc = glob[:, :, begin:begin + n].contiguous()
        seq_loc = np.clip(seq - begin * S, 0, n * S).astype(np.int32)
        sl = torch.from_numpy(seq_loc).to(dev)
        ls = oq.shard_sinks(sinks, begin, n)
        Tr, slice_off, C = _localize(Tg, loc, sl, ls, begin)
        out, cnt = _lists(loc, Tr, sl, ls)
        hxlib.check_device_errors(dev)
        out, cnt, so = np16(out), np16(cnt), np16(slice_off)
        for b in range(B):
            nb = -(-int(seq[b]) // S)
            kb = k if k is not None else nb // 4
            n_loc = -(-int(seq_loc[b]) // S)
            for h in range(H):
                sel = oq.select_pages(sc[b, h, :nb], kb, sinks)
                want = sel[(sel >= begin) & (sel < begin + n)] - begin
                row = b * H + h
                np.testing.assert_array_equal(out[row, :cnt[row]], want)
                np.testing.assert_array_equal(so[row], oq.slice_counts(want, n_loc, min(ls, n_loc), C))


def test_sharded_decode_over_global_selection():
    """A 32K-token nuq4 layer split over 4 emulated shards: each shard scores
    its pages, the global threshold equals the one-GPU quest_select's, each
    shard's decode over its part of the selection gives partials whose merge
    is float64 attention over the single-GPU selection (within 2e-3)."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, G, R = 4, 128, 7, 4
    T = 32 * 1024
    n_all = T // S
    n = n_all // R
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=700)
    gpu, orc = make_pools(sc, n_all, S, H, D, outlier_frac=0.02)
    K, V = make_kv(T, H, D, seed=701, chan_seed=700)
    pos = torch.arange(T, device="cuda")
    gpu.write_kv(0, K, V, pos, pos)
    k_, v_, p_ = np16(K), np16(V), np16(pos)
    for a in range(0, T, 4096):
        orc.write_kv(0, k_[a:a + 4096], v_[a:a + 4096], p_[a:a + 4096], p_[a:a + 4096])
    g = torch.Generator(device="cuda").manual_seed(702)
    q = torch.randn((1, H * G, D), generator=g, device="cuda").to(torch.float16)
    bt = torch.arange(n_all, dtype=torch.int32, device="cuda").unsqueeze(0)
    one = fused.quest_select(gpu, 0, q, bt, torch.tensor([T], dtype=torch.int32, device="cuda"), top_frac=(1, 4),
                             sink_pages=4)
    locs = []
    for r in range(R):
        loc = torch.empty((1, H, n), dtype=torch.float32, device="cuda")
        sl = torch.tensor([n * S], dtype=torch.int32, device="cuda")
        fused.page_scores(gpu, 0, q, bt[:, r * n:(r + 1) * n].contiguous(), sl, n, oq.shard_sinks(4, r * n, n), loc)
        locs.append(loc)
    glob = torch.cat(locs, dim=2).contiguous()           # the all-gather, emulated
    Tg = _threshold(glob, torch.tensor([T], dtype=torch.int32, device="cuda"), 4)
    np.testing.assert_array_equal(np16(Tg), np16(one.thresh))
    o_parts, l_parts = [], []
    for r in range(R):
        sl = torch.tensor([n * S], dtype=torch.int32, device="cuda")
        ls = oq.shard_sinks(4, r * n, n)
        Tr, slice_off, _ = _localize(Tg, locs[r], sl, ls, r * n)
        sel = fused.Selection(locs[r], Tr, sl, S, n, ls, None, None, slice_off)
        o, lse = fused.decode(gpu, 0, q, bt[:, r * n:(r + 1) * n].contiguous(), sl, sel, page_begin=r * n)
        o_parts.append(np16(o[0]))
        l_parts.append(np16(lse[0]))
    gpu.check()
    om, _ = oatt.merge_partials(np.stack(o_parts), np.stack(l_parts))
    q0 = np16(q[0])
    kmin = orc.stats[0][:, :, 0].transpose(1, 0, 2)
    kmax = orc.stats[0][:, :, 1].transpose(1, 0, 2)
    qp, qn = oq.group_terms(q0, G, "sum")
    scores = oq.page_scores(qp, qn, kmin, kmax)
    pages = [oq.select_pages(scores[:, h], n_all // 4, 4) for h in range(H)]
    Kd, Vd = orc.dequant_sequence(0, np.arange(n_all), T)
    ro, _ = oatt.decode_attention(q0.astype(np.float64), Kd, Vd, oatt.page_mask_to_token_mask(pages, T, S))
    assert np.abs(om - ro).max() < 2e-3
