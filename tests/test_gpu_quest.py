"""GPU parity: Kernel B (Quest scores and exact top-K with sinks) and the
quest API. Scores and selected page indices must be bit-exact against the
oracle's pinned arithmetic."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np16
from oracle import quest as oq

pytestmark = pytest.mark.gpu


def _pool_with_stats(P, H, D, seed):
    """A one-layer pool whose fp16 stats are written directly (config 2:
    per-page min / max of fp16 N(0,1) keys)."""
    from kvquant.compact_pool import CompactKVPool
    from kvquant.synthetic import NUQ4, make_scales
    sc = make_scales([NUQ4], H, D, t_cal=64, seed=seed)
    pool = CompactKVPool(1, P, 16, H, D, sc)
    g = torch.Generator(device="cuda").manual_seed(seed)
    K = torch.randn((P, 16, H, D), generator=g, device="cuda").to(torch.float16)
    kmin, kmax = K.amin(dim=1), K.amax(dim=1)                   # (P, H, D)
    st = pool.layers[0].stats                                    # (H, P, 2, D)
    st[:, :, 0] = kmin.permute(1, 0, 2)
    st[:, :, 1] = kmax.permute(1, 0, 2)
    return pool, np16(kmin), np16(kmax)


@pytest.mark.parametrize("gqa", ["sum", "mean"])
def test_config2_scores_and_selection_bit_exact(gqa):
    """Config 2: 8192 pages, H=4, D=128, 28 query heads (G=7), k = 25% + 4 sinks."""
    from kvquant.fused import quest_select, selected_lists
    P, H, D, G = 8192, 4, 128, 7
    pool, kmin, kmax = _pool_with_stats(P, H, D, seed=2)
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn((1, H * G, D), generator=g, device="cuda").to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").unsqueeze(0)
    sl = torch.tensor([P * 16], dtype=torch.int32, device="cuda")
    sel = quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, gqa=gqa)
    lists, counts = selected_lists(sel)
    pool.check()
    qp, qn = oq.group_terms(np16(q[0]), G, gqa)
    ref = oq.page_scores(qp, qn, kmin, kmax)                     # (P, H)
    np.testing.assert_array_equal(np16(sel.scores[0]).T.view(np.uint32), ref.view(np.uint32))
    for h in range(H):
        want = oq.select_pages(ref[:, h], P // 4, 4)
        assert int(counts[0, h]) == len(want) == 2052
        np.testing.assert_array_equal(np16(lists[0, h, :len(want)]), want)


@pytest.mark.parametrize("P,k,sinks", [(1, 5, 4), (5, 1, 4), (40, 100, 2), (40, 0, 3), (300, 17, 0),
                                       (70000, 17500, 4)])
def test_selection_edge_sizes(P, k, sinks):
    """Fewer pages than sinks, k >= remaining pages, k = 0, no sinks, and a
    1M-token-sized page count."""
    from kvquant.fused import quest_select, selected_lists
    H, D = 4, 128
    pool, kmin, kmax = _pool_with_stats(P, H, D, seed=P)
    q = torch.randn((1, H, D), device="cuda").to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").unsqueeze(0)
    sl = torch.tensor([P * 16 - 3], dtype=torch.int32, device="cuda")
    sel = quest_select(pool, 0, q, bt, sl, top_k=k, sink_pages=sinks, lists=True)
    lists, counts = selected_lists(sel)
    pool.check()
    qp, qn = oq.group_terms(np16(q[0]), 1, "sum")
    ref = oq.page_scores(qp, qn, kmin, kmax)
    for h in range(H):
        want = oq.select_pages(ref[:, h], k, sinks)
        assert int(counts[0, h]) == len(want)
        np.testing.assert_array_equal(np16(lists[0, h, :len(want)]), want)
        # the chunked lists the decode balances over (hx_quest_lists)
        assert int(sel.counts[h]) == len(want)
        np.testing.assert_array_equal(np16(sel.lists[h, :len(want)]), want)


def test_selection_ties_go_to_lower_page():
    """All-equal scores: the lowest non-sink pages win (pinned tie rule)."""
    from kvquant.fused import quest_select, selected_lists
    P, H, D = 3000, 4, 128
    pool, _, _ = _pool_with_stats(P, H, D, seed=9)
    pool.layers[0].stats.zero_()
    q = torch.randn((1, H, D), device="cuda").to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").unsqueeze(0)
    sl = torch.tensor([P * 16], dtype=torch.int32, device="cuda")
    sel = quest_select(pool, 0, q, bt, sl, top_k=700, sink_pages=4)
    lists, counts = selected_lists(sel)
    pool.check()
    for h in range(H):
        assert int(counts[0, h]) == 704
        np.testing.assert_array_equal(np16(lists[0, h, :704]), np.arange(704))


def test_batched_selection_with_block_tables_and_union():
    from kvquant.fused import quest_select, selected_lists
    P, H, D = 600, 4, 128
    pool, kmin, kmax = _pool_with_stats(P, H, D, seed=11)
    g = torch.Generator(device="cuda").manual_seed(12)
    perm = torch.randperm(P, generator=g, device="cuda").to(torch.int32)
    bt = torch.stack([perm[:300], perm[300:]])                   # two sequences
    sl = torch.tensor([300 * 16, 250 * 16 - 7], dtype=torch.int32, device="cuda")
    q = torch.randn((2, H * 7, D), generator=g, device="cuda").to(torch.float16)
    sel = quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, lists=True)
    lists, counts = selected_lists(sel)
    ulists, ucounts = selected_lists(sel, union=True)
    pool.check()
    for b in range(2):
        n = (int(sl[b]) + 15) // 16
        phys = np16(bt[b, :n]).astype(np.int64)
        qp, qn = oq.group_terms(np16(q[b]), 7, "sum")
        ref = oq.page_scores(qp, qn, kmin[phys], kmax[phys])
        union = set()
        for h in range(H):
            want = oq.select_pages(ref[:, h], n // 4, 4)
            union |= set(want.tolist())
            np.testing.assert_array_equal(np16(lists[b, h, :int(counts[b, h])]), want)
            assert int(sel.counts[b * H + h]) == len(want)
            np.testing.assert_array_equal(np16(sel.lists[b * H + h, :len(want)]), want)
        np.testing.assert_array_equal(np16(ulists[b, :int(ucounts[b])]), sorted(union))


def test_quest_api_matches_reference_fixture(golden):
    import quest
    g = golden("quest_spec.npz")
    K = torch.from_numpy(g["K"]).cuda()
    kmin, kmax = quest.compute_page_stats(K)
    np.testing.assert_array_equal(np16(kmin), g["kmin"])
    np.testing.assert_array_equal(np16(kmax), g["kmax"])
    q = torch.from_numpy(g["q"]).cuda()
    bound = quest.page_upper_bound(q, kmin, kmax)
    np.testing.assert_allclose(np16(bound), g["bound"], rtol=1e-5, atol=1e-5)
    b = torch.from_numpy(g["bound"]).cuda()
    np.testing.assert_array_equal(np16(quest.topk_pages_with_sinks(b, 5, 2)), g["topk_k5_s2"])
    np.testing.assert_array_equal(np16(quest.topk_pages_with_sinks(b[:4], 10, 1)), g["topk_small"])
    sel = torch.from_numpy(g["topk_k5_s2"]).cuda()
    out = quest.selected_attention(q, K, torch.from_numpy(g["V"]).cuda(), sel)
    np.testing.assert_allclose(np16(out), g["attention"], atol=1e-5)
    # fp16 stats through the Triton-compatible alias (fp16 bound)
    from quest.triton_kernels import page_upper_bound_triton
    b16 = page_upper_bound_triton(torch.from_numpy(g["q16"]).cuda(), torch.from_numpy(g["kmin16"]).cuda(),
                                  torch.from_numpy(g["kmax16"]).cuda())
    assert np.abs(np16(b16).astype(np.float32) - g["bound_triton16"].astype(np.float32)).max() <= 0.0625


def test_select_top_blocks_for_layer_planted_block_and_sinks():
    """The reference's selector tests (test_quest_selector.py:41-95)."""
    from kvquant.quest_selector import select_top_blocks_for_layer
    from kvquant.compact_pool import CompactKVPool
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    H, D, BS, NB, Tc = 2, 8, 4, 6, 32
    kp = torch.linspace(-1.5, 1.5, 16, dtype=torch.float16, device="cuda").reshape(1, 1, -1).expand(H, D, 16)
    vp = torch.linspace(-1.5, 1.5, 4, dtype=torch.float16, device="cuda").reshape(1, 1, -1).expand(H, Tc, 4)
    sc = KVScales([PerChannelScale(kp.contiguous(), torch.full((H, D), 2.0, dtype=torch.float16, device="cuda"),
                                   torch.full((H, D), -2.0, dtype=torch.float16, device="cuda"), 4)],
                  [PerTokenScale(vp.contiguous(), torch.full((H, Tc), 2.0, dtype=torch.float16, device="cuda"),
                                 torch.full((H, Tc), -2.0, dtype=torch.float16, device="cuda"), 2)])
    pool = CompactKVPool(1, NB, BS, H, D, sc)
    key = torch.zeros((5 * BS, H, D), dtype=torch.float16, device="cuda")
    key[3 * BS:4 * BS] = 1.0
    s = torch.arange(5 * BS, device="cuda")
    pool.write_kv(0, key, torch.zeros_like(key), s, s)
    q = torch.ones((H, D), dtype=torch.float16, device="cuda")
    used = torch.arange(5, device="cuda")
    ids, fp = select_top_blocks_for_layer(pool, 0, q, used, BS, top_k=1, sink_blocks=0)
    assert ids.tolist() == [3] and fp.tolist() == [12]
    pool2 = CompactKVPool(1, NB, BS, H, D, sc)
    z = torch.zeros((5 * BS, H, D), dtype=torch.float16, device="cuda")
    pool2.write_kv(0, z, z, s, s)
    ids, _ = select_top_blocks_for_layer(pool2, 0, q, used, BS, top_k=1, sink_blocks=2)
    assert {0, 1} <= set(ids.tolist())
    pool.check()


@pytest.mark.parametrize("P", [2000, 20000])   # one CTA per row; one CTA per 1024 pages
@pytest.mark.parametrize("case", ["wide", "anchor_low", "anchor_high", "dup_wide", "negative"])
def test_threshold_anchored_bins_wide_ranges(case, P):
    """The histogram bins are centred on the first non-sink page's score and
    clamp beyond 16 octaves; scores far from it (or a boundary inside a
    clamped end bin) must still give the exact top-k."""
    import quest
    H, sinks, k = 3, 4, P // 4 + 3
    rng = np.random.default_rng({"wide": 1, "anchor_low": 2, "anchor_high": 3, "dup_wide": 4, "negative": 5}[case])
    if case == "wide":         # log-uniform over 200 octaves, both signs
        b = np.sign(rng.standard_normal((P, H))) * np.exp2(rng.uniform(-100, 100, (P, H)))
    elif case == "anchor_low":  # every other score far above the anchor: top end bin
        b = rng.uniform(1.0, 2.0, (P, H))
        b[sinks] = 1e-30
    elif case == "anchor_high":  # every other score far below the anchor: bottom end bin
        b = rng.uniform(1.0, 2.0, (P, H))
        b[sinks] = 1e30
    elif case == "dup_wide":    # few distinct values spread wide, many ties
        b = np.exp2(rng.integers(-60, 60, (P, H)).astype(np.float64))
    else:                       # all negative, narrow
        b = -rng.uniform(3.0, 3.001, (P, H))
    b = b.astype(np.float32)
    got = np16(quest.topk_pages_with_sinks(torch.from_numpy(b).cuda(), k, sinks))
    np.testing.assert_array_equal(got, oq.topk_pages_with_sinks(b, k, sinks))
