"""CPU tests: the C ABI library loads and exports every declared symbol, the
host-side logic (scales file format, shard plan, synthetic inputs, argument
checks) and the split-KV exchange across two gloo ranks."""
from __future__ import annotations

import ctypes
import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "helix_kv.h").read_text()
    return re.findall(r"HX_API\s+[\w\s\*]+?\b(hx_\w+)\s*\(", text)


def test_header_declares_the_entry_points():
    names = _declared()
    assert len(names) == len(set(names)) >= 17
    for n in ("hx_pack_append", "hx_quest_scores", "hx_quest_threshold", "hx_decode_attn", "hx_merge_partials"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import hxlib
    lib = ctypes.CDLL(str(hxlib.LIB_PATH))
    for n in _declared():
        assert hasattr(lib, n), f"{n} declared in helix_kv.h but not exported"
    assert set(hxlib._SIGS) == set(_declared())


def test_host_only_entry_points():
    import hxlib
    assert "sm_100a" in hxlib.version()
    n = hxlib.lib().hx_decode_scratch_bytes(2, 4, 10)
    assert n >= 2 * 4 * 10 * (8 * 128 + 16) * 4
    assert hxlib.lib().hx_decode_scratch_bytes(0, 4, 10) == 0
    # argument validation happens before any device work
    assert hxlib.lib().hx_merge_partials(None, None, None, 0, 1, 1, None, None, None) == hxlib.HX_ERR_ARG
    assert hxlib.lib().hx_pack_append(None, None, None, None, None, None, None, 1, None) == hxlib.HX_ERR_ARG


def test_cpu_tensors_raise_instead_of_falling_back():
    import hxlib
    with pytest.raises(hxlib.HelixError):
        hxlib.ptr(torch.zeros(3))


def test_scales_file_format_round_trip(tmp_path):
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    ks = PerChannelScale(torch.randn(2, 8, 16).half(), torch.ones(2, 8).half(), -torch.ones(2, 8).half(), 4)
    vs = PerTokenScale(torch.randn(2, 32, 4).half(), torch.ones(2, 32).half(), -torch.ones(2, 32).half(), 2)
    sc = KVScales([ks], [vs], first_few_fp16=3, num_bits=4)
    p = tmp_path / "s.pt"
    sc.save(str(p))
    d = torch.load(p, weights_only=True)   # the reference's dict layout (scales.py:105-130)
    assert set(d) == {"per_layer_keys", "per_layer_values", "first_few_fp16", "num_bits"}
    assert set(d["per_layer_keys"][0]) == {"poles", "upper_threshold", "lower_threshold", "num_bits"}
    back = KVScales.load(str(p))
    assert back.num_layers == 1 and back.first_few_fp16 == 3
    assert torch.equal(back.per_layer_values[0].poles, vs.poles)
    with pytest.raises(AssertionError):
        KVScales([ks, ks], [vs])


def test_shard_plan_covers_pages_once():
    from kvquant.splitkv import local_k, shard_plan
    for n in (1, 7, 65536, 65537):
        for w in (1, 2, 4, 8):
            sh = [shard_plan(n, w, r) for r in range(w)]
            assert sh[0].page_begin == 0 and sh[0].sink_pages == 4
            assert all(s.sink_pages == 0 for s in sh[1:])
            for a, b in zip(sh, sh[1:]):
                assert a.page_begin + a.n_pages == b.page_begin
            assert sh[-1].page_begin + sh[-1].n_pages == n
            assert sum(local_k(s) for s in sh) <= n // 4 + w


def test_synthetic_inputs_are_seeded_and_sorted():
    from kvquant.synthetic import NUQ2, NUQ4, codebook, make_kv, make_scales, mixed_layout
    z = codebook(16, "cpu")
    assert torch.all(z[1:] > z[:-1]) and abs(float(z.sum())) < 1e-5
    K1, V1 = make_kv(64, 2, 32, seed=5, device="cpu")
    K2, V2 = make_kv(64, 2, 32, seed=5, device="cpu")
    assert torch.equal(K1, K2) and torch.equal(V1, V2) and K1.dtype == torch.float16
    sc = make_scales([NUQ4, NUQ2], 2, 32, t_cal=64, seed=1, device="cpu")
    assert sc.per_layer_keys[0].poles.shape == (2, 32, 16) and sc.per_layer_values[1].poles.shape == (2, 64, 4)
    p = sc.per_layer_keys[0].poles.float()
    assert torch.all(p[..., 1:] >= p[..., :-1])
    lay = mixed_layout()
    assert len(lay) == 28 and lay[15] == NUQ2 and lay[16] == NUQ4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_worker(rank, world, port, q, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kvquant.splitkv import exchange_partials, shard_plan
        from oracle import attention as oatt
        rng = np.random.default_rng(0)
        K = rng.standard_normal((160, 2, 16))
        V = rng.standard_normal((160, 2, 16))
        sh = shard_plan(10, world, rank)
        a, b = sh.page_begin * 16, (sh.page_begin + sh.n_pages) * 16
        o, lse = oatt.decode_attention(q, K[a:b], V[a:b])
        O, L = exchange_partials(torch.tensor(o, dtype=torch.float32), torch.tensor(lse, dtype=torch.float32))
        om, lm = oatt.merge_partials(O.numpy(), L.numpy())
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.concatenate([om.ravel(), lm]))
    finally:
        dist.destroy_process_group()


def test_split_kv_exchange_two_gloo_ranks(tmp_path):
    """Each rank attends its shard; the all-gathered partials merge to the
    unsharded result on every rank."""
    from oracle import attention as oatt
    q = np.random.default_rng(1).standard_normal((4, 16))
    port = _free_port()
    mp.start_processes(_gloo_worker, args=(2, port, q, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    rng = np.random.default_rng(0)
    K = rng.standard_normal((160, 2, 16))
    V = rng.standard_normal((160, 2, 16))
    o_ref, lse_ref = oatt.decode_attention(q, K, V)
    for r in range(2):
        got = np.load(tmp_path / f"r{r}.npy")
        np.testing.assert_allclose(got[:64].reshape(4, 16), o_ref, atol=1e-5)
        np.testing.assert_allclose(got[64:], lse_ref, atol=1e-5)


def test_global_selection_shard_thresholds_match_one_gpu():
    """The rule hx_quest_localize applies: a single-GPU threshold restated per
    shard selects, with local page indices, exactly the single-GPU choice's
    pages on that shard (ties across shard edges, k = 0, k >= n, sinks
    spilling past the first shard)."""
    from oracle import quest as oq
    rng = np.random.default_rng(7)
    for trial in range(1500):
        R, n = int(rng.integers(1, 7)), int(rng.integers(1, 48))
        N = R * n
        s = (np.round(rng.standard_normal(N) * rng.choice([0.5, 2.0, 8.0])) / 4).astype(np.float32)
        if trial % 7 == 0:
            s[:] = 1.0
        k, sinks = int(rng.integers(0, N + 3)), int(rng.integers(0, 6))
        T = oq.threshold64(s, k, sinks)
        np.testing.assert_array_equal(oq.select_by_threshold(s, T, sinks), oq.select_pages(s, k, sinks))
        want = oq.global_selection_per_shard(s, R, k, sinks)
        b = oq.shard_bounds(N, R)
        for r in range(R):
            ls = oq.shard_sinks(sinks, b[r], b[r + 1] - b[r])
            got = oq.select_by_threshold(s[b[r]:b[r + 1]], oq.shard_threshold(T, b[r]), ls)
            np.testing.assert_array_equal(got, want[r])


def _gather_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kvquant.splitkv import gather_score_rows
        B, H, n = 2, 3, 5
        loc = torch.arange(B * H * n, dtype=torch.float32).view(B, H, n) + 1000 * rank
        gathered = torch.empty((world, B * H, n))
        glob = torch.empty((B, H, world * n))
        gather_score_rows(loc, gathered, glob)
        np.save(os.path.join(result_dir, f"g{rank}.npy"), glob.numpy())
    finally:
        dist.destroy_process_group()


def test_global_selection_score_gather_two_gloo_ranks(tmp_path):
    """The score gather of the global selection puts rank r's pages of every
    (b, h) row at global pages r*n .. r*n + n - 1, on every rank."""
    port = _free_port()
    mp.start_processes(_gather_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    B, H, n = 2, 3, 5
    base = np.arange(B * H * n, dtype=np.float32).reshape(B, H, n)
    want = np.concatenate([base, base + 1000], axis=2)
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"g{r}.npy"), want)


def test_slice_index_by_reciprocal_multiply_is_exact():
    """The fused selection (csrc/select.cuh, row_select) finds a page's slice
    as (x * m) >> 32 with m = ceil(2^32 / per) instead of x / per. That is the
    quotient for every non-sink offset x the kernel can meet (x < 16,384, the
    fused-selection row limit) and every slice width 2 <= per <= 16,384; width
    1 takes x itself. Checked exhaustively here."""
    x = np.arange(16384, dtype=np.uint64)
    for per in range(2, 16385):
        m = np.uint64(((1 << 32) + per - 1) // per)
        assert np.array_equal((x * m) >> np.uint64(32), x // np.uint64(per)), per
