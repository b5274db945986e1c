"""The allocation-free decode entry point, called through the C ABI.

hx_decode_attn_noalloc serves callers that cannot call cudaMalloc (an engine
that has reserved nearly all HBM for its own KV pool and allows no allocation
while decoding, or a foreign-language binding holding only raw device
pointers): it keeps its scratch in a fixed array inside the library. These
tests call it twice in a row and compare each result with hx_decode_attn on a
caller-provided scratch buffer, and check that an oversized request is
refused before any work runs. This file sorts last so a stop-at-first-failure
run has already run every other test.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the decode parity tolerance (max-abs on the normalised output)


def _setup():
    from kvquant import fused
    from kvquant.compact_pool import CompactKVPool
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S, n = 4, 128, 16, 3000
    sc = make_scales([NUQ4], H, D, t_cal=1024, seed=90)
    pool = CompactKVPool(1, 200, S, H, D, sc)
    K, V = make_kv(n, H, D, seed=91, chan_seed=90)
    pos = torch.arange(n, device="cuda")
    pool.write_kv(0, K, V, pos, pos)
    g = torch.Generator(device="cuda").manual_seed(92)
    q = torch.randn((1, H * 7, D), generator=g, device="cuda").to(torch.float16)
    bt = torch.arange(200, dtype=torch.int32, device="cuda").unsqueeze(0)
    sl = torch.tensor([n], dtype=torch.int32, device="cuda")
    sel = fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4)
    return pool, q, bt, sl, sel


def _call_noalloc(pool, q, bt, sl, sel, n_splits):
    import hxlib
    B, Hq, D = q.shape
    o = torch.full((B, Hq, D), float("nan"), dtype=torch.float32, device="cuda")
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device="cuda")
    st, _keep = pool.scales.device_layer(0, pool.device)
    rc = hxlib.lib().hx_decode_attn_noalloc(
        hxlib.stream(pool.device), ctypes.byref(pool.layers[0].struct), ctypes.byref(st),
        hxlib.ptr(q), B, Hq // pool.num_kv_heads, 1.0 / math.sqrt(D), hxlib.ptr(bt), bt.shape[1],
        hxlib.ptr(sl), 0, sel.max_pages, hxlib.SEL_THRESHOLD, hxlib.ptr(sel.scores), hxlib.ptr(sel.thresh),
        sel.sink_pages, None, 0, None, n_splits, hxlib.ptr(o), hxlib.ptr(lse), None,
        hxlib.ptr(hxlib.err_word(pool.device)))
    return rc, o, lse


def test_noalloc_decode_matches_scratch_decode_twice():
    import hxlib
    from kvquant import fused
    pool, q, bt, sl, sel = _setup()
    ns = 37
    o_ref, lse_ref = fused.decode(pool, 0, q, bt, sl, sel, n_splits=ns)
    for _ in range(2):
        rc, o, lse = _call_noalloc(pool, q, bt, sl, sel, ns)
        assert rc == hxlib.HX_OK
        pool.check()
        assert float((o - o_ref).abs().max()) < TOL
        assert float((lse - lse_ref).abs().max()) < TOL


def test_noalloc_decode_refuses_oversized_requests():
    import hxlib
    pool, q, bt, sl, sel = _setup()
    rc, o, _ = _call_noalloc(pool, q, bt, sl, sel, n_splits=1024 // pool.num_kv_heads + 1)
    assert rc == hxlib.HX_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.isnan(o).all()  # nothing ran
