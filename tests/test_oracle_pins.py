"""Pin the CPU oracle to the reference before trusting it.

Two sources: the literal known answers of the reference's own CPU tests
(src/kvquant/tests/test_nuq_roundtrip.py, src/quest/tests/test_reference.py),
and the fixtures tests/golden/make_golden.py recorded by running the
reference's torch spec and its Triton kernels (interpreter) on seeded inputs.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import nuq as onuq
from oracle import packing as opack
from oracle import quest as oq
from oracle.pool import LayerScalesNP, OraclePool


# --- known answers from the reference's CPU tests -------------------------------

def test_kat_round_to_nearest_pole():
    # test_nuq_roundtrip.py:25-31
    values = np.array([0.1, 0.4, -0.6, 1.2], np.float32)
    poles = np.broadcast_to(np.array([-1.0, -0.5, 0.0, 0.5, 1.0], np.float32), (4, 5))
    out = onuq.round_to_nearest_pole(values, poles)
    np.testing.assert_array_equal(out, [0.0, 0.5, -0.5, 1.0])


def test_kat_band_outliers():
    # test_nuq_roundtrip.py:34-39
    values = np.array([[-2.0, -0.4, 0.1, 0.7, 3.5]], np.float32)
    mask = onuq.find_outliers(values, np.array([[1.0]]), np.array([[-1.0]]))
    assert mask.tolist() == [[True, False, False, False, True]]


def test_kat_first_few_fp16():
    # test_nuq_roundtrip.py:42-48
    values = np.zeros((5, 4), np.float32)
    mask = onuq.find_outliers(values, np.full((5, 4), 1.0), np.full((5, 4), -1.0),
                              first_few_fp16=2, seq_dim=0)
    assert mask[:2].all() and not mask[2:].any()


def test_kat_outliers_preserved():
    # test_nuq_roundtrip.py:65-75
    values = np.array([-5.0, -0.3, 0.0, 0.4, 7.0], np.float32)
    poles = np.broadcast_to(np.array([-0.5, 0.0, 0.5], np.float32), (5, 3))
    out, mask = onuq.quantize_nuq(values, poles, np.full(5, 1.0), np.full(5, -1.0))
    assert out[0] == -5.0 and out[-1] == 7.0
    assert mask.tolist() == [True, False, False, False, True]


def test_kat_no_outlier_roundtrip_error():
    # test_nuq_roundtrip.py:51-62
    values = np.linspace(-1, 1, 256).astype(np.float32)
    poles = np.broadcast_to(np.array([-1.0, -0.33, 0.33, 1.0], np.float32), (256, 4))
    out, mask = onuq.quantize_nuq(values, poles, np.full(256, 100.0), np.full(256, -100.0))
    assert mask.sum() == 0
    assert np.abs(out - values).max() < 0.34


def test_kat_page_stats_and_bound():
    # test_reference.py:34-63: stats are the slot-axis min/max; the bound is
    # an upper bound of the true per-page max of q.k
    rng = np.random.default_rng(1)
    K = rng.standard_normal((8, 16, 4, 32)).astype(np.float32)
    q = rng.standard_normal((4, 32)).astype(np.float32)
    kmin, kmax = oq.compute_page_stats(K)
    assert kmin[1, 0, 3] == K[1, :, 0, 3].min() and kmax[1, 0, 3] == K[1, :, 0, 3].max()
    qp, qn = oq.group_terms(q, 1, "sum")
    bound = oq.page_scores(qp, qn, kmin, kmax)
    true_max = np.einsum("pthd,hd->pth", K, q).max(axis=1)
    assert (bound - true_max >= -1e-4).all()


def test_kat_topk_sinks_sorted_and_clipped():
    # test_reference.py:66-92
    rng = np.random.default_rng(2)
    bound = rng.standard_normal((16, 4)).astype(np.float32)
    bound[0, :] = -100.0
    sel = oq.topk_pages_with_sinks(bound, k=4, sink_pages=2)
    assert sel.shape == (6, 4)
    for h in range(4):
        assert {0, 1} <= set(sel[:, h].tolist())
        assert (np.diff(sel[:, h]) >= 0).all()
    assert oq.topk_pages_with_sinks(rng.standard_normal((3, 2)), k=10, sink_pages=1).shape == (3, 2)


def test_kat_all_pages_equals_dense_and_low_page_excluded():
    # test_reference.py:95-139
    rng = np.random.default_rng(3)
    K = rng.standard_normal((32, 2, 16))
    V = rng.standard_normal((32, 2, 16))
    q = rng.standard_normal((2, 16))
    o, _ = oatt.decode_attention(q, K, V)
    for h in range(2):
        s = K[:, h] @ q[h] / math.sqrt(16)
        p = np.exp(s - s.max())
        np.testing.assert_allclose(o[h], p @ V[:, h] / p.sum(), atol=1e-12)
    Kz = np.zeros((16, 1, 8))
    Vz = np.zeros((16, 1, 8))
    Kz[8, 0, 0] = 1.0
    Vz[8, 0, 0] = 5.0
    qz = np.zeros((1, 8))
    qz[0, 0] = 1.0
    mask = oatt.page_mask_to_token_mask([[0]], 16, 4)
    o, _ = oatt.decode_attention(qz, Kz, Vz, mask)
    assert o[0, 0] < 1.0


# --- fixtures recorded from the reference --------------------------------------

def test_pin_nuq_spec(golden):
    g = golden("nuq_spec.npz")
    out = onuq.round_to_nearest_pole(g["values"], g["poles"])
    np.testing.assert_array_equal(out, g["round_to_nearest_pole"])
    np.testing.assert_array_equal(onuq.find_outliers(g["values"], g["upper"], g["lower"]),
                                  g["find_outliers"])
    np.testing.assert_array_equal(
        onuq.find_outliers(g["values"], g["upper"], g["lower"], first_few_fp16=3, seq_dim=0),
        g["find_outliers_first3"])
    rec, mask = onuq.quantize_nuq(g["values"], g["poles"], g["upper"], g["lower"])
    np.testing.assert_array_equal(rec, g["quantize_recon"])
    np.testing.assert_array_equal(mask, g["quantize_mask"])
    np.testing.assert_array_equal(onuq.nearest_codes(g["values"], g["poles"]), g["codes"])
    deq = onuq.dequantize_nuq(g["codes"], np.where(mask, g["values"], 0), mask, g["poles"])
    np.testing.assert_array_equal(deq, g["dequantize"])


@pytest.mark.parametrize("name", ["k16", "k4", "v16", "v4"])
def test_pin_triton_dense(golden, name):
    g = golden("triton_dense.npz")
    v, p, up, lo = (g[f"{name}_{k}"] for k in ("values", "poles", "upper", "lower"))
    if name.startswith("k"):
        codes, outv, outm = onuq.pack_keys_per_channel(v, p, up, lo)
        rec = onuq.unpack_keys_per_channel(codes, outv, outm, p)
    else:
        codes, outv, outm = onuq.pack_values_per_token(v, p, up, lo)
        rec = onuq.unpack_values_per_token(codes, outv, outm, p)
    np.testing.assert_array_equal(codes, g[f"{name}_codes"])
    np.testing.assert_array_equal(outm, g[f"{name}_outm"])
    np.testing.assert_array_equal(outv.view(np.uint16), g[f"{name}_outv"].view(np.uint16))
    np.testing.assert_array_equal(rec.view(np.uint16), g[f"{name}_recon"].view(np.uint16))


def _pool_from_fixture(g):
    NB, BS, H, D, Lk, Lv, Tc = (int(x) for x in g["meta"])
    sc = LayerScalesNP(g["k_poles"], g["k_upper"], g["k_lower"],
                       g["v_poles"], g["v_upper"], g["v_lower"])
    pool = OraclePool(1, NB, BS, H, D, [sc])
    pool.write_kv(0, g["key"], g["value"], g["slots"], g["abs_pos"])
    return pool, (NB, BS, H, D)


def test_pin_triton_pool_codes_outliers_stats(golden):
    g = golden("triton_pool.npz")
    pool, (NB, BS, H, D) = _pool_from_fixture(g)
    written = np.zeros((NB, BS), bool)
    for s in g["slots"]:
        if s >= 0:
            written[s // BS, s % BS] = True
    for kv, bits in ((0, pool.scales[0].bits_k), (1, pool.scales[0].bits_v)):
        name = "k" if kv == 0 else "v"
        ref_codes = g[f"{name}_codes"]                 # (NB, BS, H, D) one byte per code
        ref_m = g[f"{name}_outm"].astype(bool)
        ref_v = g[f"{name}_outv"]
        packed = pool.codes[0][kv]                      # (H, NB, BS, D*bits/8)
        for b in range(NB):
            for s in range(BS):
                if not written[b, s]:
                    continue
                for h in range(H):
                    np.testing.assert_array_equal(opack.unpack_codes(packed[h, b, s], bits),
                                                  ref_codes[b, s, h])
        for h in range(H):
            for b in range(NB):
                want = sorted((s, d, int(ref_v[b, s, h, d].view(np.uint16)))
                              for s in range(BS) if written[b, s]
                              for d in np.nonzero(ref_m[b, s, h])[0])
                assert pool.outlier_entries(0, h, b, kv) == want
    st = pool.stats[0]
    used = written.any(axis=1)
    for h in range(H):
        for b in range(NB):
            if used[b]:
                np.testing.assert_array_equal(st[h, b, 0].astype(np.float32), g["k_min"][b, h])
                np.testing.assert_array_equal(st[h, b, 1].astype(np.float32), g["k_max"][b, h])


def test_pin_triton_pool_staging(golden):
    g = golden("triton_pool.npz")
    pool, (NB, BS, H, D) = _pool_from_fixture(g)
    sk, sv = pool.unpack_to_staging(0, g["block_ids"], g["first_pos"])
    written = np.zeros((NB, BS), bool)
    for s in g["slots"]:
        if s >= 0:
            written[s // BS, s % BS] = True
    for i, b in enumerate(g["block_ids"]):
        rows = written[b]
        np.testing.assert_array_equal(sk[i, rows].view(np.uint16), g["staging_k"][i, rows].view(np.uint16))
        np.testing.assert_array_equal(sv[i, rows].view(np.uint16), g["staging_v"][i, rows].view(np.uint16))


def test_pin_quest_spec(golden):
    g = golden("quest_spec.npz")
    kmin, kmax = oq.compute_page_stats(g["K"])
    np.testing.assert_array_equal(kmin, g["kmin"])
    np.testing.assert_array_equal(kmax, g["kmax"])
    qp, qn = oq.group_terms(g["q"], 1, "sum")
    bound = oq.page_scores(qp, qn, kmin, kmax)
    # same formula, different float32 summation order than torch's .sum()
    np.testing.assert_allclose(bound, g["bound"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(oq.topk_pages_with_sinks(g["bound"], 5, 2), g["topk_k5_s2"])
    np.testing.assert_array_equal(oq.topk_pages_with_sinks(g["bound"][:4], 10, 1), g["topk_small"])
    # selected_attention (H == H_v, fp32) vs the float64 restatement
    P, S, H, D = g["K"].shape
    sel = g["topk_k5_s2"]
    mask = oatt.page_mask_to_token_mask([sel[:, h] for h in range(H)], P * S, S)
    o, _ = oatt.decode_attention(g["q"], g["K"].reshape(P * S, H, D), g["V"].reshape(P * S, H, D), mask)
    np.testing.assert_allclose(o, g["attention"], atol=2e-5)
    # Triton bound: fp32 accumulate, fp16 store (quest/triton_kernels.py:57)
    qp16, qn16 = oq.group_terms(g["q16"], 1, "sum")
    b16 = oq.page_scores(qp16, qn16, g["kmin16"], g["kmax16"]).astype(np.float16)
    assert np.abs(b16.astype(np.float32) - g["bound_triton16"].astype(np.float32)).max() <= 0.0625


def test_packing_roundtrip():
    rng = np.random.default_rng(5)
    for bits in (2, 4):
        c = rng.integers(0, 1 << bits, size=(7, 3, 128), dtype=np.uint8)
        p = opack.pack_codes(c, bits)
        assert p.shape == (7, 3, 128 * bits // 8)
        np.testing.assert_array_equal(opack.unpack_codes(p, bits), c)
    # pinned bit order
    assert opack.pack_codes(np.array([1, 2], np.uint8), 4).tolist() == [0x21]
    assert opack.pack_codes(np.array([1, 2, 3, 0], np.uint8), 2).tolist() == [0b00111001]


def test_merge_partials_matches_unsharded():
    rng = np.random.default_rng(6)
    K = rng.standard_normal((96, 2, 16))
    V = rng.standard_normal((96, 2, 16))
    q = rng.standard_normal((4, 16))
    o_ref, lse_ref = oatt.decode_attention(q, K, V)
    parts = [oatt.decode_attention(q, K[a:b], V[a:b]) for a, b in ((0, 40), (40, 41), (41, 96))]
    o, lse = oatt.merge_partials([p[0] for p in parts], [p[1] for p in parts])
    np.testing.assert_allclose(o, o_ref, atol=1e-12)
    np.testing.assert_allclose(lse, lse_ref, atol=1e-12)
