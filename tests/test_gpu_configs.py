"""GPU parity at the benchmark configurations' own sizes (BASELINE configs 3
and 4), against the oracle: packed codes, outlier entries and page stats
bit-exact, Quest selections bit-exact, decode outputs within 2e-3 max-abs of
float64 dequantise-then-attend."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import gpu_codes, gpu_outlier_array, make_pools, np16
from oracle import attention as oatt
from oracle import quest as oq

pytestmark = pytest.mark.gpu

TOL = 2e-3
H, D, S, G = 4, 128, 16, 7


def _write_chunked(gpu, orc, layer, K, V, slots, pos, chunk=4096):
    """One GPU call for the whole batch; the oracle in chunks (its nearest-pole
    search holds (tokens, H, D, levels) floats)."""
    gpu.write_kv(layer, K, V, slots, pos)
    k, v, s, p = np16(K), np16(V), np16(slots), np16(pos)
    for a in range(0, k.shape[0], chunk):
        orc.write_kv(layer, k[a:a + chunk], v[a:a + chunk], s[a:a + chunk], p[a:a + chunk])


def _assert_pool_equal(gpu, orc, layer=0):
    for a, b in zip(gpu_codes(gpu, layer), orc.codes[layer]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(np16(gpu.layers[layer].stats).view(np.uint16), orc.stats[layer].view(np.uint16))
    np.testing.assert_array_equal(gpu_outlier_array(gpu, layer), orc.outlier_array(layer))


def _oracle_selection(orc, layer, q, used_pages, k, sinks=4):
    kmin = orc.stats[layer][:, used_pages, 0].transpose(1, 0, 2)
    kmax = orc.stats[layer][:, used_pages, 1].transpose(1, 0, 2)
    qp, qn = oq.group_terms(q, G, "sum")
    sc = oq.page_scores(qp, qn, kmin, kmax)
    return [oq.select_pages(sc[:, h], k, sinks) for h in range(H)]


def test_config3_128k_dense_and_quest():
    """Config 3: one nuq4 layer at 128K context (8192 pages), batch 1, G = 7:
    the pool bit-exact, the Quest 25% + 4 sinks selection bit-exact, and the
    fused decode within 2e-3 both dense and over the selection."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    T = 128 * 1024
    n = T // S
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=300)
    gpu, orc = make_pools(sc, n, S, H, D, outlier_frac=0.03)
    K, V = make_kv(T, H, D, seed=301, chan_seed=300)
    pos = torch.arange(T, device="cuda")
    _write_chunked(gpu, orc, 0, K, V, pos, pos)
    gpu.check()
    _assert_pool_equal(gpu, orc)

    g = torch.Generator(device="cuda").manual_seed(302)
    q = torch.randn((1, H * G, D), generator=g, device="cuda").to(torch.float16)
    bt = torch.arange(n, dtype=torch.int32, device="cuda").unsqueeze(0)
    sl = torch.tensor([T], dtype=torch.int32, device="cuda")
    sel = fused.quest_select(gpu, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, lists=True)
    o_q, _ = fused.decode(gpu, 0, q, bt, sl, sel)
    o_d, _ = fused.decode(gpu, 0, q, bt, sl)
    lists, counts = fused.selected_lists(sel)
    gpu.check()

    q0 = np16(q[0])
    pages = _oracle_selection(orc, 0, q0, np.arange(n), n // 4)
    for h in range(H):
        np.testing.assert_array_equal(np16(lists[0, h, :int(counts[0, h])]), pages[h])
    Kd, Vd = orc.dequant_sequence(0, np.arange(n), T)
    qd = q0.astype(np.float64)
    ro_d, _ = oatt.decode_attention(qd, Kd, Vd)
    ro_q, _ = oatt.decode_attention(qd, Kd, Vd, oatt.page_mask_to_token_mask(pages, T, S))
    assert np.abs(np16(o_d[0]) - ro_d).max() < TOL
    assert np.abs(np16(o_q[0]) - ro_q).max() < TOL


def test_config4_batched_append_then_decode():
    """Config 4 at B = 8: sequences of 24K tokens on shuffled block tables
    receive an 8K-token chunk each in one append call (65,536 tokens), then one
    decode token each is appended and attended with Quest 25% + 4 sinks and
    densely. Pool, selections and outputs against the oracle."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    B, pre, chunk = 8, 24 * 1024, 8 * 1024
    ctx = pre + chunk + 1
    npg = -(-ctx // S)
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=400)
    NB = B * npg + 11
    gpu, orc = make_pools(sc, NB, S, H, D, outlier_frac=0.03)
    rng = np.random.default_rng(401)
    perm = rng.permutation(NB)
    bt_np = perm[:B * npg].reshape(B, npg).astype(np.int32)
    bt = torch.from_numpy(bt_np).cuda()
    K, V = make_kv(B * ctx, H, D, seed=402, chan_seed=400)
    K, V = K.view(B, ctx, H, D), V.view(B, ctx, H, D)

    def slots_of(b, p):
        return bt[b, p // S].to(torch.int64) * S + p % S

    for b in range(B):                                   # the existing context, one prefill per sequence
        p = torch.arange(pre, device="cuda")
        _write_chunked(gpu, orc, 0, K[b, :pre].contiguous(), V[b, :pre].contiguous(), slots_of(b, p), p)
    # the step: every sequence's 8K chunk in one call, then one decode token each
    p = torch.arange(pre, pre + chunk, device="cuda")
    ks = torch.cat([K[b, pre:pre + chunk] for b in range(B)]).contiguous()
    vs = torch.cat([V[b, pre:pre + chunk] for b in range(B)]).contiguous()
    sl_ = torch.cat([slots_of(b, p) for b in range(B)])
    _write_chunked(gpu, orc, 0, ks, vs, sl_, p.repeat(B))
    last = torch.full((B,), ctx - 1, device="cuda")
    s1 = torch.stack([slots_of(b, last[b]) for b in range(B)])
    _write_chunked(gpu, orc, 0, K[:, ctx - 1].contiguous(), V[:, ctx - 1].contiguous(), s1, last)
    gpu.check()
    _assert_pool_equal(gpu, orc)

    g = torch.Generator(device="cuda").manual_seed(403)
    q = torch.randn((B, H * G, D), generator=g, device="cuda").to(torch.float16)
    sl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    sel = fused.quest_select(gpu, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, lists=True)
    o_q, _ = fused.decode(gpu, 0, q, bt, sl, sel)
    o_d, _ = fused.decode(gpu, 0, q, bt, sl)
    lists, counts = fused.selected_lists(sel)
    gpu.check()
    for b in range(B):
        qb = np16(q[b])
        pages = _oracle_selection(orc, 0, qb, bt_np[b], npg // 4)
        for h in range(H):
            np.testing.assert_array_equal(np16(lists[b, h, :int(counts[b, h])]), pages[h])
        Kd, Vd = orc.dequant_sequence(0, bt_np[b], ctx)
        qd = qb.astype(np.float64)
        ro_d, _ = oatt.decode_attention(qd, Kd, Vd)
        ro_q, _ = oatt.decode_attention(qd, Kd, Vd, oatt.page_mask_to_token_mask(pages, ctx, S))
        assert np.abs(np16(o_d[b]) - ro_d).max() < TOL, b
        assert np.abs(np16(o_q[b]) - ro_q).max() < TOL, b
