"""GPU parity: Kernel C (fused-dequant split-KV decode) against fp64
dequantise-then-attend on the oracle pool, within 2e-3 max-abs; and the
cross-shard (o, lse) merge."""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import pytest
import torch

from helpers import make_pools, np16, write_both
from oracle import attention as oatt
from oracle import quest as oq

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max-abs on the normalised attention output


def _build(layout, n_tokens, seed, B=1, t_cal=4096, pages_extra=0, shuffle=False, v_layout=None):
    """A pool over `layout`; with `v_layout` the V scales (and V code width)
    of each layer come from that layout instead."""
    from kvquant.synthetic import make_kv, make_scales
    H, D, S = 4, 128, 16
    sc = make_scales(layout, H, D, t_cal=t_cal, seed=seed)
    if v_layout is not None:
        sv = make_scales(v_layout, H, D, t_cal=t_cal, seed=seed + 7)
        for li in range(len(layout)):
            sc.per_layer_values[li] = sv.per_layer_values[li]
    n_pages = [-(-n // S) for n in n_tokens]
    NB = sum(n_pages) + pages_extra
    gpu, orc = make_pools(sc, NB, S, H, D)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    perm = torch.randperm(NB, generator=g, device="cuda") if shuffle else torch.arange(NB, device="cuda")
    maxp = max(n_pages)
    bt = torch.zeros((B, maxp), dtype=torch.int32, device="cuda")
    base = 0
    for b in range(B):
        bt[b, :n_pages[b]] = perm[base:base + n_pages[b]].to(torch.int32)
        base += n_pages[b]
    for li, (levels, frac, side) in enumerate(layout):
        for b in range(B):
            K, V = make_kv(n_tokens[b], H, D, seed=seed + 10 * li + 100 * b, outlier_frac=frac,
                           chan_seed=seed + 1000 * li)
            pos = torch.arange(n_tokens[b], device="cuda")
            slots = bt[b, pos // S].to(torch.int64) * S + pos % S
            write_both(gpu, orc, li, K, V, slots, pos)
    gpu.check()
    return gpu, orc, bt, torch.tensor(n_tokens, dtype=torch.int32, device="cuda")


def _oracle_out(orc, layer, q, bt, sl, pages_per_head=None):
    B = q.shape[0]
    outs, lses = [], []
    for b in range(B):
        n = int(sl[b])
        K, V = orc.dequant_sequence(layer, np16(bt[b]), n)
        mask = None
        if pages_per_head is not None:
            mask = oatt.page_mask_to_token_mask(pages_per_head[b], n, 16)
        o, lse = oatt.decode_attention(np16(q[b]).astype(np.float64), K, V, mask)
        outs.append(o)
        lses.append(lse)
    return np.stack(outs), np.stack(lses)


def _query(B, G, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((B, 4 * G, 128), generator=g, device="cuda").to(torch.float16)


@pytest.mark.parametrize("layout_name", ["nuq4", "nuq2"])
def test_dense_decode_matches_oracle(layout_name):
    from kvquant import fused
    from kvquant.synthetic import NUQ2, NUQ4
    layout = {"nuq4": [NUQ4], "nuq2": [NUQ2]}[layout_name]
    gpu, orc, bt, sl = _build(layout, [5000 - 7], seed=20)
    q = _query(1, 7, 21)
    o, lse = fused.decode(gpu, 0, q, bt, sl)
    gpu.check()
    ro, rl = _oracle_out(orc, 0, q, bt, sl)
    assert np.abs(np16(o) - ro).max() < TOL
    np.testing.assert_allclose(np16(lse), rl, atol=1e-3)


@pytest.mark.parametrize("bits", [(4, 4), (4, 2), (2, 4), (2, 2)])
def test_cuda_core_decode_matches_oracle(bits):
    """The CUDA-core (FFMA) variant of the decode, dense and over a Quest
    selection, against the same oracle; K and V at every pair of widths."""
    from kvquant import fused
    from kvquant.synthetic import NUQ2, NUQ4
    lay = {4: NUQ4, 2: NUQ2}
    gpu, orc, bt, sl = _build([lay[bits[0]]], [6000 - 3], seed=25, v_layout=[lay[bits[1]]])
    assert (gpu.layers[0].bits_k, gpu.layers[0].bits_v) == bits
    q = _query(1, 7, 26)
    o, lse = fused.decode(gpu, 0, q, bt, sl, cores="cuda")
    ro, rl = _oracle_out(orc, 0, q, bt, sl)
    assert np.abs(np16(o) - ro).max() < TOL
    np.testing.assert_allclose(np16(lse), rl, atol=1e-3)
    sel = fused.quest_select(gpu, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4)
    lists, counts = fused.selected_lists(sel)
    o2, _ = fused.decode(gpu, 0, q, bt, sl, sel, cores="cuda")
    o3, _ = fused.decode(gpu, 0, q, bt, sl, sel)
    gpu.check()
    pages = [[np16(lists[0, h, :int(counts[0, h])]) for h in range(4)]]
    ro2, _ = _oracle_out(orc, 0, q, bt, sl, pages)
    assert np.abs(np16(o2) - ro2).max() < TOL
    assert np.abs(np16(o2) - np16(o3)).max() < TOL


def test_quest_decode_matches_oracle_config3_shape():
    """Config 3 shape at 16K context: nuq4 pool, Quest 25% + 4 sinks, G=7,
    t_cal crossing (V per-token rows then the tail row)."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    gpu, orc, bt, sl = _build([NUQ4], [16384], seed=30, t_cal=4096)
    q = _query(1, 7, 31)
    sel = fused.quest_select(gpu, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4)
    o, lse = fused.decode(gpu, 0, q, bt, sl, sel)
    lists, counts = fused.selected_lists(sel)
    gpu.check()
    n = 1024
    kmin = orc.stats[0][:, :n, 0].transpose(1, 0, 2)
    kmax = orc.stats[0][:, :n, 1].transpose(1, 0, 2)
    qp, qn = oq.group_terms(np16(q[0]), 7, "sum")
    ref = oq.page_scores(qp, qn, kmin, kmax)
    pages = [oq.select_pages(ref[:, h], n // 4, 4) for h in range(4)]
    for h in range(4):
        np.testing.assert_array_equal(np16(lists[0, h, :int(counts[0, h])]), pages[h])
    ro, rl = _oracle_out(orc, 0, q, bt, sl, [pages])
    assert np.abs(np16(o) - ro).max() < TOL
    np.testing.assert_allclose(np16(lse), rl, atol=1e-3)
    # the same selection read from the thresholds alone (splits over the sequence)
    sel_t = dataclasses.replace(sel, slice_off=None, lists=None, counts=None)
    o_t, lse_t = fused.decode(gpu, 0, q, bt, sl, sel_t)
    gpu.check()
    assert np.abs(np16(o_t) - ro).max() < TOL
    np.testing.assert_allclose(np16(lse_t), rl, atol=1e-3)


def test_batched_decode_block_tables_partial_pages():
    """Config 4 flavour: several sequences of ragged lengths, shuffled pool
    pages, partial last pages, a 1-token and an exactly-one-page sequence."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    lens = [1, 16, 777, 2048 + 5]
    gpu, orc, bt, sl = _build([NUQ4], lens, seed=40, B=len(lens), shuffle=True, pages_extra=3)
    q = _query(len(lens), 7, 41)
    o, lse = fused.decode(gpu, 0, q, bt, sl, n_splits=5)
    ro, rl = _oracle_out(orc, 0, q, bt, sl)
    assert np.abs(np16(o) - ro).max() < TOL
    sel = fused.quest_select(gpu, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4)
    lists, counts = fused.selected_lists(sel)
    o2, _ = fused.decode(gpu, 0, q, bt, sl, sel, n_splits=3)
    gpu.check()
    pages = [[np16(lists[b, h, :int(counts[b, h])]) for h in range(4)] for b in range(len(lens))]
    ro2, _ = _oracle_out(orc, 0, q, bt, sl, pages)
    assert np.abs(np16(o2) - ro2).max() < TOL


def test_list_mode_and_mixed_layers():
    """Explicit page lists (the reference hook's per-head selection) on a
    two-layer pool: nuq2 layer 0, nuq4 layer 1."""
    from kvquant import fused
    from kvquant.synthetic import NUQ2, NUQ4
    gpu, orc, bt, sl = _build([NUQ2, NUQ4], [3000], seed=50)
    q = _query(1, 7, 51)
    rng = np.random.default_rng(52)
    n = 188
    per_head = [np.sort(rng.choice(n, size=40, replace=False)) for _ in range(4)]
    lists = torch.tensor(np.stack(per_head), dtype=torch.int32, device="cuda").unsqueeze(0)
    counts = torch.full((1, 4), 40, dtype=torch.int32, device="cuda")
    for layer in (0, 1):
        o, _ = fused.decode(gpu, layer, q, bt, sl, lists=lists, list_counts=counts)
        ro, _ = _oracle_out(orc, layer, q, bt, sl, [per_head])
        assert np.abs(np16(o) - ro).max() < TOL
    gpu.check()


def test_empty_selection_gives_zero_output():
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    gpu, orc, bt, sl = _build([NUQ4], [64], seed=60)
    q = _query(1, 7, 61)
    lists = torch.zeros((1, 4, 1), dtype=torch.int32, device="cuda")
    counts = torch.zeros((1, 4), dtype=torch.int32, device="cuda")
    o, lse = fused.decode(gpu, 0, q, bt, sl, lists=lists, list_counts=counts)
    gpu.check()
    assert float(o.abs().max()) == 0.0
    assert torch.isinf(lse).all() and (lse < 0).all()


def test_merge_partials_split_kv_equals_unsharded():
    """Split-KV: shard a sequence's pages into 3 pools, decode each with its
    page_begin, merge (o, lse): equal to the unsharded decode."""
    from kvquant import fused
    from kvquant.compact_pool import CompactKVPool
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S, n = 4, 128, 16, 4000
    sc = make_scales([NUQ4], H, D, t_cal=1000, seed=70)
    K, V = make_kv(n, H, D, seed=71, chan_seed=70)
    q = _query(1, 7, 72)
    full = CompactKVPool(1, 250, S, H, D, sc)
    pos = torch.arange(n, device="cuda")
    full.write_kv(0, K, V, pos, pos)
    bt = torch.arange(250, dtype=torch.int32, device="cuda").unsqueeze(0)
    o_ref, lse_ref = fused.decode(full, 0, q, bt, torch.tensor([n], dtype=torch.int32, device="cuda"))
    bounds = oq.shard_bounds(250, 3)
    os_, ls_ = [], []
    for r in range(3):
        a, b = bounds[r], bounds[r + 1]
        shard = CompactKVPool(1, b - a, S, H, D, sc)
        t0, t1 = a * S, min(b * S, n)
        p = torch.arange(t1 - t0, device="cuda")
        shard.write_kv(0, K[t0:t1].contiguous(), V[t0:t1].contiguous(), p, p + t0)
        btr = torch.arange(b - a, dtype=torch.int32, device="cuda").unsqueeze(0)
        o, lse = fused.decode(shard, 0, q, btr, torch.tensor([t1 - t0], dtype=torch.int32, device="cuda"),
                              page_begin=a)
        os_.append(o[0])
        ls_.append(lse[0])
    o_m, lse_m = fused.merge_partials(torch.stack(os_), torch.stack(ls_))
    full.check()
    # same math, different fp32 summation order (splits vs shards): ~1e-6 relative
    assert float((o_m - o_ref[0]).abs().max()) < 1e-4
    assert float((lse_m - lse_ref[0]).abs().max()) < 1e-4
    ro, rl = oatt.merge_partials(np16(torch.stack(os_)), np16(torch.stack(ls_)))
    np.testing.assert_allclose(np16(o_m), ro, atol=1e-6)


def test_decode_scale_and_group_one():
    """G = 1 (H == Hq, the reference's selected_attention shape) and a custom
    softmax scale."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    gpu, orc, bt, sl = _build([NUQ4], [700], seed=80)
    q = _query(1, 1, 81)
    o, _ = fused.decode(gpu, 0, q, bt, sl, softmax_scale=0.05)
    gpu.check()
    K, V = orc.dequant_sequence(0, np16(bt[0]), 700)
    ro, _ = oatt.decode_attention(np16(q[0]).astype(np.float64), K, V, scale=0.05)
    assert np.abs(np16(o[0]) - ro).max() < TOL


@pytest.mark.parametrize("k,n_splits", [(None, 7), (0, 5), (3, 37), (100000, 11), (None, 160)])
def test_decode_slice_counts_match_lists(k, n_splits):
    """The decode balanced by the threshold's per-slice counts (HX_SEL_SLICES)
    gives every CTA the same pages, in the same order, as the balanced lists
    (HX_SEL_LIST): bit-identical outputs, within TOL of the oracle. Ragged
    sequences (one shorter than the sinks), k = 0, k past every page, more
    splits than selected pages, a clustered selection (a planted block)."""
    from kvquant import fused
    from kvquant.synthetic import NUQ2
    lens = [40, 3 * 16 * 1024 + 9, 20000, 16 * 700]
    gpu, orc, bt, sl = _build([NUQ2], lens, seed=60, B=len(lens), shuffle=True)
    q = _query(len(lens), 7, 61)
    st = gpu.layers[0].stats  # (H, NB, 2, D): plant high-bound pages in one block of sequence 1
    rows = bt[1, 1000:1060].long()
    st[:, rows, 1] = 30.0
    kw = dict(top_k=k) if k is not None else dict(top_frac=(1, 4))
    sel = fused.quest_select(gpu, 0, q, bt, sl, sink_pages=4, lists=True, **kw)
    assert sel.slice_off is not None and sel.lists is not None
    o_s, lse_s = fused.decode(gpu, 0, q, bt, sl, sel, n_splits=n_splits)
    o_l, lse_l = fused.decode(gpu, 0, q, bt, sl, dataclasses.replace(sel, slice_off=None), n_splits=n_splits)
    gpu.check()
    np.testing.assert_array_equal(np16(o_s).view(np.uint32), np16(o_l).view(np.uint32))
    np.testing.assert_array_equal(np16(lse_s).view(np.uint32), np16(lse_l).view(np.uint32))
    # the slice counts themselves: selected non-sink pages of each slice
    off = np16(sel.slice_off)
    lists, counts = np16(sel.lists), np16(sel.counts)
    nsl = off.shape[1] - 1
    for b, n_tok in enumerate(lens):
        n = -(-n_tok // 16)
        sinks = min(4, n)
        per = -(-(n - sinks) // nsl) if n > sinks else 1
        for h in range(4):
            row = b * 4 + h
            pages = lists[row, :counts[row]]
            rest = pages[pages >= sinks]
            want = np.bincount(np.minimum((rest - sinks) // per, nsl - 1), minlength=nsl)
            np.testing.assert_array_equal(np.diff(off[row]), want)
    pages = [[lists[b * 4 + h, :counts[b * 4 + h]] for h in range(4)] for b in range(len(lens))]
    ro, _ = _oracle_out(orc, 0, q, bt, sl, pages)
    assert np.abs(np16(o_s) - ro).max() < TOL


@pytest.mark.parametrize("case", ["config3", "ragged", "ties", "edges"])
def test_fused_selection_decode_equals_two_kernel_path(case):
    """hx_decode_attn_select (each CTA finds its row's threshold) against
    quest_select + decode: the same thresholds' selections, the same slice
    offsets and the same outputs, bit for bit; the histogram is left zero."""
    import hxlib
    from kvquant import fused
    from kvquant.synthetic import NUQ2, NUQ4
    if case == "config3":
        gpu, orc, bt, sl = _build([NUQ4], [16384], seed=130)
        kw = dict(top_frac=(1, 4), sink_pages=4)
    elif case == "ragged":
        gpu, orc, bt, sl = _build([NUQ2], [1, 16, 777, 5000, 2048 + 5], seed=131, B=5, shuffle=True, pages_extra=3)
        kw = dict(top_frac=(1, 4), sink_pages=4)
    elif case == "ties":     # all-equal page statistics: ties everywhere
        gpu, orc, bt, sl = _build([NUQ4], [4000], seed=132)
        gpu.layers[0].stats.zero_()
        kw = dict(top_k=300, sink_pages=4)
    else:                    # k = 0 and k beyond the pages
        gpu, orc, bt, sl = _build([NUQ4], [3000, 500], seed=133, B=2)
        kw = dict(top_k=0, sink_pages=2)
    B = bt.shape[0]
    q = _query(B, 7, 134)
    ns = 6
    for kw2 in ([kw] if case != "edges" else [kw, dict(top_k=10 ** 6, sink_pages=2)]):
        sel = fused.quest_select(gpu, 0, q, bt, sl, **kw2)
        o_ref, l_ref = fused.decode(gpu, 0, q, bt, sl, sel, n_splits=ns)
        H = gpu.num_kv_heads
        C = int(hxlib.lib().hx_quest_slices(bt.shape[1]))
        th = torch.empty((B * H,), dtype=torch.int64, device="cuda")
        so = torch.empty((B * H, C + 1), dtype=torch.int32, device="cuda")
        o, l_ = fused.quest_decode(gpu, 0, q, bt, sl, n_splits=ns, thresh_out=th, slice_out=so, **kw2)
        gpu.check()
        np.testing.assert_array_equal(np16(so), np16(sel.slice_off))
        lists, counts = fused.selected_lists(sel)
        sel2 = fused.Selection(sel.scores, th, sel.seq_lens, sel.page_size, sel.max_pages, sel.sink_pages)
        lists2, counts2 = fused.selected_lists(sel2)
        np.testing.assert_array_equal(np16(counts2), np16(counts))
        np.testing.assert_array_equal(np16(lists2), np16(lists))
        np.testing.assert_array_equal(np16(o), np16(o_ref))
        np.testing.assert_array_equal(np16(l_), np16(l_ref))
        hist = hxlib.scratch("cuda", "quest_hist", 4)
        assert int(hist.view(torch.int32)[:B * H * 2 * 4096].abs().sum()) == 0
