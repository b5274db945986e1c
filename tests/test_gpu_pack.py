"""GPU parity: Kernel A (pack-on-write), staging unpack, dense pack / unpack,
the torch-spec nuq API. Integer and byte outputs must be bit-exact against the
oracle and the reference fixtures."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import gpu_codes, gpu_outlier_sets, make_pools, np16, oracle_outlier_sets, write_both

pytestmark = pytest.mark.gpu


def _t(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("name", ["k16", "k4", "v16", "v4"])
def test_dense_pack_unpack_matches_reference_fixture(golden, name):
    from kvquant import batched
    g = golden("triton_dense.npz")
    v, p, up, lo = (_t(g[f"{name}_{k}"]) for k in ("values", "poles", "upper", "lower"))
    if name.startswith("k"):
        c, ov, om = batched.pack_keys_per_channel_batched(v, p, up, lo)
        rec = batched.unpack_keys_per_channel_batched(c, ov, om, p)
    else:
        c, ov, om = batched.pack_values_per_token_batched(v, p, up, lo)
        rec = batched.unpack_values_per_token_batched(c, ov, om, p)
    np.testing.assert_array_equal(np16(c), g[f"{name}_codes"])
    np.testing.assert_array_equal(np16(om), g[f"{name}_outm"])
    np.testing.assert_array_equal(np16(ov).view(np.uint16), g[f"{name}_outv"].view(np.uint16))
    np.testing.assert_array_equal(np16(rec).view(np.uint16), g[f"{name}_recon"].view(np.uint16))


def test_per_head_pack_equals_batched(golden):
    from kvquant import batched
    g = golden("triton_dense.npz")
    v, p, up, lo = (_t(g[f"k16_{k}"]) for k in ("values", "poles", "upper", "lower"))
    c, ov, om = batched.pack_keys_per_channel_batched(v, p, up, lo)
    for h in range(v.shape[1]):
        c1, ov1, om1 = batched.pack_keys_per_channel(v[:, h].contiguous(), p[h], up[h], lo[h])
        assert torch.equal(c1, c[:, h]) and torch.equal(om1, om[:, h]) and torch.equal(ov1, ov[:, h])


def _fixture_pool(g):
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    NB, BS, H, D, Lk, Lv, Tc = (int(x) for x in g["meta"])
    sc = KVScales([PerChannelScale(_t(g["k_poles"]), _t(g["k_upper"]), _t(g["k_lower"]), 4)],
                  [PerTokenScale(_t(g["v_poles"]), _t(g["v_upper"]), _t(g["v_lower"]), 2)])
    gpu, orc = make_pools(sc, NB, BS, H, D)
    write_both(gpu, orc, 0, _t(g["key"]), _t(g["value"]), _t(g["slots"]), _t(g["abs_pos"]))
    gpu.check()
    return gpu, orc, (NB, BS, H, D)


def test_pool_write_matches_reference_pool_fixture(golden):
    g = golden("triton_pool.npz")
    gpu, orc, (NB, BS, H, D) = _fixture_pool(g)
    written = np.zeros((NB, BS), bool)
    for s in g["slots"]:
        if s >= 0:
            written[s // BS, s % BS] = True
    kc = np16(gpu.k_codes)[0]
    vc = np16(gpu.v_codes)[0]
    np.testing.assert_array_equal(kc[written], g["k_codes"][written])
    np.testing.assert_array_equal(vc[written], g["v_codes"][written])
    km, vm = np16(gpu.k_outm)[0], np16(gpu.v_outm)[0]
    np.testing.assert_array_equal(km[written], g["k_outm"][written])
    np.testing.assert_array_equal(vm[written], g["v_outm"][written])
    np.testing.assert_array_equal(np16(gpu.k_outv)[0][written].view(np.uint16),
                                  g["k_outv"][written].view(np.uint16))
    used = written.any(axis=1)
    np.testing.assert_array_equal(np16(gpu.k_min)[0][used], g["k_min"][used])
    np.testing.assert_array_equal(np16(gpu.k_max)[0][used], g["k_max"][used])
    # and the packed bytes / sparse lists equal the oracle's
    for a, b in zip(gpu_codes(gpu, 0), orc.codes[0]):
        np.testing.assert_array_equal(a, b)
    assert gpu_outlier_sets(gpu, 0) == oracle_outlier_sets(orc, 0)


def test_unpack_to_staging_matches_reference_fixture(golden):
    g = golden("triton_pool.npz")
    gpu, orc, (NB, BS, H, D) = _fixture_pool(g)
    ids, fp = _t(g["block_ids"]), _t(g["first_pos"])
    sk = torch.empty((len(ids), BS, H, D), dtype=torch.float16, device="cuda")
    sv = torch.empty_like(sk)
    gpu.unpack_to_staging(0, ids, fp, sk, sv)
    gpu.check()
    written = np.zeros((NB, BS), bool)
    for s in g["slots"]:
        if s >= 0:
            written[s // BS, s % BS] = True
    for i, b in enumerate(g["block_ids"]):
        rows = written[b]
        np.testing.assert_array_equal(np16(sk)[i, rows].view(np.uint16), g["staging_k"][i, rows].view(np.uint16))
        np.testing.assert_array_equal(np16(sv)[i, rows].view(np.uint16), g["staging_v"][i, rows].view(np.uint16))
    ok, ov = orc.unpack_to_staging(0, g["block_ids"], g["first_pos"])
    np.testing.assert_array_equal(np16(sk).view(np.uint16), ok.view(np.uint16))
    np.testing.assert_array_equal(np16(sv).view(np.uint16), ov.view(np.uint16))


@pytest.mark.parametrize("layout", ["nuq4", "nuq2", "k4v2"])
def test_pool_config1_bit_exact(layout):
    """Config 1 shapes (T=4096, H=4, D=128, 1% outliers x10): packed codes,
    outlier lists and page stats bit-exact against the oracle."""
    from kvquant.synthetic import NUQ2, NUQ4, make_kv, make_scales
    lay = {"nuq4": [NUQ4], "nuq2": [NUQ2], "k4v2": [NUQ4]}[layout]
    T, H, D, S = 4096, 4, 128, 16
    sc = make_scales(lay, H, D, t_cal=4096, seed=0)
    if layout == "k4v2":  # 16-level K with 4-level V, as the reference's own tests mix
        sc2 = make_scales([NUQ2], H, D, t_cal=4096, seed=0)
        sc.per_layer_values[0] = sc2.per_layer_values[0]
    K, V = make_kv(T, H, D, seed=0, outlier_frac=lay[0][1])
    gpu, orc = make_pools(sc, T // S, S, H, D)
    slots = torch.arange(T, device="cuda")
    write_both(gpu, orc, 0, K, V, slots, slots)
    gpu.check()
    for a, b in zip(gpu_codes(gpu, 0), orc.codes[0]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(np16(gpu.layers[0].stats).view(np.uint16), orc.stats[0].view(np.uint16))
    gs, os_ = gpu_outlier_sets(gpu, 0), oracle_outlier_sets(orc, 0)
    assert gs.keys() == os_.keys()
    assert gs == os_
    n_out = sum(len(v) for v in gs.values())
    assert 0.005 * T * H * D * 2 < n_out < 0.1 * T * H * D * 2


def _adversarial_codebooks(L):
    """Codebook rows (fp16) that stress the bisection path of the pack kernel:
    regular, tiny gaps, duplicates, unsorted, subnormal, huge spread, a
    non-finite pole, all equal."""
    from kvquant.synthetic import codebook
    z = codebook(L, "cpu").numpy().astype(np.float64)
    rng = np.random.default_rng(L)
    rows = [z, z * 1e-3, np.repeat(z[::2], 2)[:L], rng.permutation(z),
            np.arange(L) * 6e-8 - 6e-8 * (L // 2), np.sign(z) * np.abs(z) ** 4 * 6e4 / np.abs(z).max() ** 4,
            np.where(np.arange(L) == L - 1, np.inf, z), np.full(L, 0.5)]
    if L == 4:
        rows[5] = np.array([-6e4, -1e-3, 1e-3, 6e4])
        rows[6] = np.array([-1.0, 0.0, np.nan, 1.0])
    return np.stack([np.asarray(r, np.float64).astype(np.float16) for r in rows])  # (8, L)


@pytest.mark.parametrize("levels", [16, 4])
def test_pool_codes_exhaustive_fp16_adversarial_codebooks(levels):
    """Every fp16 bit pattern (finite, subnormal, +-inf, NaN) through the pool
    pack under eight kinds of codebook, for K (per-channel rows) and V
    (per-token rows): codes, outlier lists and page stats bit-exact against
    the reference's fp32 scan (oracle)."""
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    H, D, S, T = 4, 128, 16, 1024
    books = _adversarial_codebooks(levels)                       # (8, L)
    # K: channel (h, d) uses book (h * D + d) % 8; its 64 channels share x patterns
    kidx = (np.arange(H * D) % 8).reshape(H, D)
    k_poles = books[kidx]                                        # (H, D, L)
    jj = (np.arange(H * D) // 8).reshape(H, D)                   # index among its book's channels
    kbits = (np.arange(T)[:, None, None] * 64 + jj[None]).astype(np.uint16)   # (T, H, D)
    # V: token row (h, t) uses book t % 8; rows of one book cover every pattern
    v_poles = books[np.broadcast_to(np.arange(T) % 8, (H, T))]   # (H, T, L)
    vbits = ((((np.arange(T) // 8)[:, None, None] * H + np.arange(H)[None, :, None]) * D)
             + np.arange(D)[None, None, :]).astype(np.uint16)
    big = np.float16(65504.0)
    sc = KVScales([PerChannelScale(torch.from_numpy(k_poles).cuda(), torch.full((H, D), big).cuda(),
                                   torch.full((H, D), -big).cuda())],
                  [PerTokenScale(torch.from_numpy(v_poles.copy()).cuda(), torch.full((H, T), big).cuda(),
                                 torch.full((H, T), -big).cuda())])
    K = torch.from_numpy(kbits.view(np.float16)).cuda()
    V = torch.from_numpy(vbits.view(np.float16)).cuda()
    gpu, orc = make_pools(sc, T // S, S, H, D, outlier_frac=0.05)
    slots = torch.arange(T, device="cuda")
    write_both(gpu, orc, 0, K, V, slots, slots)
    gpu.check()
    for a, b in zip(gpu_codes(gpu, 0), orc.codes[0]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(np16(gpu.layers[0].stats).view(np.uint16), orc.stats[0].view(np.uint16))
    assert gpu_outlier_sets(gpu, 0) == oracle_outlier_sets(orc, 0)


@pytest.mark.parametrize("layout", ["nuq4", "nuq2"])
def test_pool_slots_in_any_order(layout):
    """Tokens of a page need not be contiguous in the input: slots [5, 3, 4,
    20] (two runs on page 0), then a whole 64-page prefill in a random slot
    order (each page written by many runs in one call). Same bytes as the
    oracle, which writes the tokens one by one."""
    from kvquant.synthetic import NUQ2, NUQ4, make_kv, make_scales
    lay = {"nuq4": [NUQ4], "nuq2": [NUQ2]}[layout]
    H, D, S = 4, 128, 16
    sc = make_scales(lay, H, D, t_cal=512, seed=11)
    # pages grown by many small runs double their lists repeatedly: room for that
    gpu, orc = make_pools(sc, 70, S, H, D, outlier_frac=1.0)
    K, V = make_kv(1024 + 4, H, D, seed=12, outlier_frac=lay[0][1] * 4, chan_seed=11)
    s = torch.tensor([5, 3, 4, 20], device="cuda")
    write_both(gpu, orc, 0, K[:4].contiguous(), V[:4].contiguous(), s, s)
    g = torch.Generator(device="cuda").manual_seed(13)
    perm = torch.randperm(1024, generator=g, device="cuda") + 5 * S
    write_both(gpu, orc, 0, K[4:].contiguous(), V[4:].contiguous(), perm, perm)
    gpu.check()
    for a, b in zip(gpu_codes(gpu, 0), orc.codes[0]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(np16(gpu.layers[0].stats).view(np.uint16), orc.stats[0].view(np.uint16))
    assert gpu_outlier_sets(gpu, 0) == oracle_outlier_sets(orc, 0)
    # a record's last word: rows (bits 0-7) | this launch's run count (8-30) | lock (31)
    last = np16(gpu.layers[0].dir)[..., 3].view(np.uint32)      # (H, NB, 2)
    assert (last & np.uint32(0xFFFFFF00) == 0).all()             # run counts back to 0, locks released


def test_pool_incremental_appends_and_overwrite():
    """Decode-style one-token appends, a chunk straddling pages, skipped (-1)
    slots, an overwrite of a written slot, a sequence starting mid-page, and
    positions past t_cal (V tail clamp)."""
    from kvquant.synthetic import NUQ2, make_kv, make_scales
    H, D, S = 4, 128, 16
    sc = make_scales([NUQ2], H, D, t_cal=48, seed=3)
    gpu, orc = make_pools(sc, 12, S, H, D)
    K, V = make_kv(200, H, D, seed=4, outlier_frac=0.05, chan_seed=3)
    # prefill 37 tokens from slot 5, then 20 single-token appends
    slots = torch.arange(5, 42, device="cuda")
    write_both(gpu, orc, 0, K[:37].contiguous(), V[:37].contiguous(), slots, slots)
    for i in range(20):
        s = torch.tensor([42 + i], device="cuda")
        write_both(gpu, orc, 0, K[37 + i:38 + i].contiguous(), V[37 + i:38 + i].contiguous(), s, s)
    # a batch with padding and two sequences in other pages
    sl = torch.tensor([-1, 128, 129, 130, -1, 160, 161], device="cuda")
    write_both(gpu, orc, 0, K[60:67].contiguous(), V[60:67].contiguous(), sl, sl + 1000)
    # overwrite slots 44..46 (already written) with new data
    s = torch.arange(44, 47, device="cuda")
    write_both(gpu, orc, 0, K[100:103].contiguous(), V[100:103].contiguous(), s, s)
    gpu.check()
    for a, b in zip(gpu_codes(gpu, 0), orc.codes[0]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(np16(gpu.layers[0].stats).view(np.uint16), orc.stats[0].view(np.uint16))
    assert gpu_outlier_sets(gpu, 0) == oracle_outlier_sets(orc, 0)
    # staging unpack of every written page equals the oracle
    ids = torch.tensor([0, 1, 2, 3, 8, 10], device="cuda")
    fp = ids * S
    sk = torch.empty((6, S, H, D), dtype=torch.float16, device="cuda")
    sv = torch.empty_like(sk)
    gpu.unpack_to_staging(0, ids, fp, sk, sv)
    ok, ov = orc.unpack_to_staging(0, np16(ids), np16(fp))
    np.testing.assert_array_equal(np16(sk).view(np.uint16), ok.view(np.uint16))
    np.testing.assert_array_equal(np16(sv).view(np.uint16), ov.view(np.uint16))


def test_pool_reset_pages_empties_lists_and_stats():
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S = 4, 128, 16
    sc = make_scales([NUQ4], H, D, t_cal=64, seed=5)
    gpu, _ = make_pools(sc, 4, S, H, D)
    K, V = make_kv(64, H, D, seed=6, outlier_frac=0.05, chan_seed=5)
    s = torch.arange(64, device="cuda")
    gpu.write_kv(0, K, V, s, s)
    gpu.reset_pages(0, torch.tensor([1, 2], device="cuda"))
    gpu.check()
    st = np16(gpu.layers[0].stats)
    assert np.isposinf(st[:, 1:3, 0].astype(np.float32)).all() and np.isneginf(st[:, 1:3, 1].astype(np.float32)).all()
    assert (np16(gpu.layers[0].dir)[:, 1:3, :, 2] == 0).all()


def test_arena_exhaustion_is_flagged():
    import hxlib
    from kvquant.synthetic import NUQ2, make_kv, make_scales
    H, D, S = 4, 128, 16
    sc = make_scales([NUQ2], H, D, t_cal=64, seed=7)
    gpu, _ = make_pools(sc, 8, S, H, D, outlier_capacity=64)
    K, V = make_kv(128, H, D, seed=8, outlier_frac=0.2)
    s = torch.arange(128, device="cuda")
    gpu.write_kv(0, K, V, s, s)
    with pytest.raises(hxlib.HelixError, match="arena"):
        gpu.check()


def test_nuq_spec_api_matches_reference_fixture(golden):
    import kvquant
    g = golden("nuq_spec.npz")
    v, p, up, lo = (_t(g[k]) for k in ("values", "poles", "upper", "lower"))
    np.testing.assert_array_equal(np16(kvquant.round_to_nearest_pole(v, p)), g["round_to_nearest_pole"])
    np.testing.assert_array_equal(np16(kvquant.find_outliers(v, up, lo)), g["find_outliers"])
    np.testing.assert_array_equal(np16(kvquant.find_outliers(v, up, lo, first_few_fp16=3, seq_dim=0)),
                                  g["find_outliers_first3"])
    rec, mask = kvquant.quantize_nuq(v, p, up, lo)
    np.testing.assert_array_equal(np16(rec), g["quantize_recon"])
    np.testing.assert_array_equal(np16(mask), g["quantize_mask"])
    deq = kvquant.dequantize_nuq(_t(g["codes"]), torch.where(mask, v, torch.zeros_like(v)), mask, p)
    np.testing.assert_array_equal(np16(deq), g["dequantize"])


def test_cpu_tensors_are_rejected():
    import hxlib
    import kvquant
    x = torch.randn(4, 8)
    with pytest.raises(hxlib.HelixError):
        kvquant.quantize_nuq(x, torch.randn(4, 8, 4), torch.ones(4, 8), -torch.ones(4, 8))
