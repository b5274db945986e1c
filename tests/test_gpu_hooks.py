"""The vLLM hooks end to end on the GPU, with a stand-in FlashAttentionImpl
(no vLLM engine): the compact-pool hook's cache update + decode against the
oracle's selection and attention, and the quantise-dequantise hook against
the oracle's reconstruction."""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from helpers import np16, oracle_scales
from oracle import attention as oatt
from oracle import quest as oq
from oracle.pool import OraclePool

pytestmark = pytest.mark.gpu

TOL = 2e-3


class FakeImpl:
    def __init__(self, scale):
        self.scale, self.sliding_window, self.alibi_slopes = scale, (-1, -1), None
        self.logits_soft_cap, self.sinks, self.sent = 0, None, []

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        self.sent.append((key.clone(), value.clone()))
        return output

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        pass


class FakeBackend:
    get_impl_cls = staticmethod(lambda: FakeImpl)


def test_compact_hook_decode_matches_oracle():
    from kvquant import compact_backend as cb
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S, n, G = 4, 128, 16, 3000, 7
    sc = make_scales([NUQ4], H, D, t_cal=1024, seed=70)
    backend = type("B", (FakeBackend,), {})
    n_pages = -(-n // S)
    cb.install_compact_backend("", num_layers=1, num_blocks=n_pages, block_size=S, num_kv_heads=H, head_size=D,
                               device="cuda", top_k_blocks_decode=n_pages // 4, sink_blocks=4, gqa="sum",
                               scales=sc, backend_cls=backend, impl_cls=FakeImpl)
    impl = backend.get_impl_cls()(scale=D ** -0.5)
    layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
    K, V = make_kv(n, H, D, seed=71, chan_seed=70)
    slots = torch.arange(n, device="cuda")
    for a in range(0, n, 1000):                       # a prefill in chunks, as vLLM updates the cache
        impl.do_kv_cache_update(layer, K[a:a + 1000], V[a:a + 1000], None, slots[a:a + 1000])
    cb.pool().check()
    g = torch.Generator(device="cuda").manual_seed(72)
    q = torch.randn((1, H * G, D), generator=g, device="cuda").to(torch.float16)
    meta = types.SimpleNamespace(max_query_len=1, num_actual_tokens=1, causal=True,
                                 block_table=torch.arange(n_pages, dtype=torch.int32, device="cuda").unsqueeze(0),
                                 seq_lens=torch.tensor([n], dtype=torch.int32, device="cuda"))
    out = torch.zeros((1, H * G, D), dtype=torch.float16, device="cuda")
    impl.forward(layer, q, K[:1], V[:1], None, meta, out)
    cb.pool().check()
    assert not impl.sent                              # served by the fused path, not FlashAttention
    orc = OraclePool(1, n_pages, S, H, D, oracle_scales(sc))
    orc.write_kv(0, np16(K), np16(V), np16(slots), np16(slots))
    kmin = orc.stats[0][:, :n_pages, 0].transpose(1, 0, 2)
    kmax = orc.stats[0][:, :n_pages, 1].transpose(1, 0, 2)
    qp, qn = oq.group_terms(np16(q[0]), G, "sum")
    ref = oq.page_scores(qp, qn, kmin, kmax)
    pages = [oq.select_pages(ref[:, h], n_pages // 4, 4) for h in range(H)]
    Kd, Vd = orc.dequant_sequence(0, np.arange(n_pages), n)
    o, _ = oatt.decode_attention(np16(q[0]).astype(np.float64), Kd, Vd,
                                 oatt.page_mask_to_token_mask(pages, n, S))
    # the hook writes vLLM's fp16 output: TOL plus half an fp16 ulp of the value
    err = np.abs(np16(out[0]).astype(np.float64) - o)
    assert (err <= TOL + np.abs(o) * 2.0 ** -11).all(), err.max()


def test_compact_hook_shuffled_block_table_matches_oracle():
    """vLLM hands out blocks from a free list (block 0 is its null block):
    two sequences on shuffled, non-identity block tables, contexts longer
    than t_cal. The hook packs V with abs_positions = slot (the reference
    hook) and the decode must read each page's V rows at its physical slot
    (reference: pack compact_pool.py:467 with compact_backend.py:157-167,
    unpack quest_selector.py:89 + compact_pool.py:370-372)."""
    from kvquant import compact_backend as cb
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S, G = 4, 128, 16, 7
    lens = [3000, 1200]
    t_cal, top_k = 256, 40
    sc = make_scales([NUQ4], H, D, t_cal=t_cal, seed=90)
    n_pages = [-(-n // S) for n in lens]
    NB = sum(n_pages) + 37
    backend = type("B", (FakeBackend,), {})
    cb.install_compact_backend("", num_layers=1, num_blocks=NB, block_size=S, num_kv_heads=H, head_size=D,
                               device="cuda", top_k_blocks_decode=top_k, sink_blocks=4, gqa="sum",
                               scales=sc, backend_cls=backend, impl_cls=FakeImpl)
    impl = backend.get_impl_cls()(scale=D ** -0.5)
    layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
    rng = np.random.default_rng(91)
    free = rng.permutation(np.arange(1, NB))              # block 0 is never handed out
    bt = np.zeros((2, max(n_pages)), np.int32)
    bt[0, :n_pages[0]] = free[:n_pages[0]]
    bt[1, :n_pages[1]] = free[n_pages[0]:n_pages[0] + n_pages[1]]
    assert not np.array_equal(bt[0, :n_pages[0]], np.arange(n_pages[0]))
    orc = OraclePool(1, NB, S, H, D, oracle_scales(sc))
    for b, n in enumerate(lens):
        K, V = make_kv(n, H, D, seed=92 + b, chan_seed=90)
        pos = np.arange(n)
        slots = torch.from_numpy(bt[b, pos // S].astype(np.int64) * S + pos % S).cuda()
        for a in range(0, n, 700):                        # chunked prefill, one cache update per chunk
            impl.do_kv_cache_update(layer, K[a:a + 700], V[a:a + 700], None, slots[a:a + 700])
        orc.write_kv(0, np16(K), np16(V), np16(slots), np16(slots))
    cb.pool().check()
    g = torch.Generator(device="cuda").manual_seed(93)
    q = torch.randn((2, H * G, D), generator=g, device="cuda").to(torch.float16)
    meta = types.SimpleNamespace(max_query_len=1, num_actual_tokens=2, causal=True,
                                 block_table=torch.from_numpy(bt).cuda(),
                                 seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"))
    out = torch.zeros((2, H * G, D), dtype=torch.float16, device="cuda")
    impl.forward(layer, q, q[:, :H], q[:, :H], None, meta, out)
    cb.pool().check()
    assert not impl.sent
    for b, n in enumerate(lens):
        used = bt[b, :n_pages[b]]
        kmin = orc.stats[0][:, used, 0].transpose(1, 0, 2)
        kmax = orc.stats[0][:, used, 1].transpose(1, 0, 2)
        qp, qn = oq.group_terms(np16(q[b]), G, "sum")
        ref = oq.page_scores(qp, qn, kmin, kmax)
        pages = [oq.select_pages(ref[:, h], top_k, 4) for h in range(H)]
        mask = oatt.page_mask_to_token_mask(pages, n, S)
        qd = np16(q[b]).astype(np.float64)
        Kd, Vd = orc.dequant_sequence(0, used, n, v_pos="physical")
        o, _ = oatt.decode_attention(qd, Kd, Vd, mask)
        # the case discriminates: the logical-position rule gives another answer
        _, Vl = orc.dequant_sequence(0, used, n, v_pos="logical")
        o_logical, _ = oatt.decode_attention(qd, Kd, Vl, mask)
        assert np.abs(o_logical - o).max() > 10 * TOL
        err = np.abs(np16(out[b]).astype(np.float64) - o)
        assert (err <= TOL + np.abs(o) * 2.0 ** -11).all(), (b, err.max())


def test_quantise_dequantise_hook_matches_oracle():
    from kvquant import vllm_backend as vb
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    from oracle.pool import quantize_k_rows, quantize_v_rows
    H, D = 4, 128
    sc = make_scales([NUQ4, NUQ4], H, D, t_cal=256, seed=80)
    backend = type("B", (FakeBackend,), {})
    vb.install_kvquant_backend("", device="cuda", scales=sc, backend_cls=backend, impl_cls=FakeImpl)
    impl = backend.get_impl_cls()(scale=1.0)
    K, V = make_kv(300, H, D, seed=81, chan_seed=1080)
    q = torch.zeros((300, 28, D), dtype=torch.float16, device="cuda")
    impl.forward(types.SimpleNamespace(layer_name="model.layers.1.self_attn.attn"), q, K, V, None,
                 types.SimpleNamespace(num_actual_tokens=280), q)
    kq, vq = impl.sent[0]
    ls = oracle_scales(sc)[1]
    _, km, krec = quantize_k_rows(np16(K[:280]), ls)
    vc, vm = quantize_v_rows(np16(V[:280]), np.arange(280), ls)
    np.testing.assert_array_equal(np16(kq[:280]).view(np.uint16), krec.astype(np.float16).view(np.uint16))
    pr = np.minimum(np.arange(280), ls.t_cal - 1)
    L = ls.v_poles.shape[-1]
    vpol = np.broadcast_to(ls.v_poles[:, pr].transpose(1, 0, 2)[:, :, None, :], (280, H, D, L))
    vrec = np.take_along_axis(vpol, vc[..., None].astype(np.int64), -1)[..., 0]
    vrec = np.where(vm, np16(V[:280]), vrec).astype(np.float16)
    np.testing.assert_array_equal(np16(vq[:280]).view(np.uint16), vrec.view(np.uint16))
    assert torch.equal(kq[280:], K[280:]) and torch.equal(vq[280:], V[280:])


class FakeAttention:
    def get_kv_cache_spec(self, vllm_config):
        return None


def test_compact_hook_without_fp16_cache_mixed_batch():
    """fp16_cache=False: a mixed batch of a 40-token prefill chunk (its
    sequence's earlier 260 tokens already in the pool) and one decode token
    of another sequence, both served from the pool by the chunked-prefill
    kernel; shuffled blocks, V rows by physical slot (the hook's rule)."""
    from kvquant import compact_backend as cb
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    H, D, S, G = 4, 128, 16, 7
    lens, chunk = [300, 150], [40, 1]
    sc = make_scales([NUQ4], H, D, t_cal=1024, seed=90)
    backend = type("B", (FakeBackend,), {})
    NB = 40
    cb.install_compact_backend("", num_layers=1, num_blocks=NB, block_size=S, num_kv_heads=H, head_size=D,
                               device="cuda", top_k_blocks_decode=0, scales=sc, backend_cls=backend,
                               impl_cls=FakeImpl, fp16_cache=False, attention_cls=FakeAttention)
    try:
        impl = backend.get_impl_cls()(scale=D ** -0.5)
        layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")
        g = torch.Generator(device="cuda").manual_seed(91)
        perm = torch.randperm(NB, generator=g, device="cuda").to(torch.int32)
        bt = torch.stack([perm[:20], perm[20:40]])                       # 20 blocks per sequence
        orc = OraclePool(1, NB, S, H, D, oracle_scales(sc))
        KV = [make_kv(n, H, D, seed=92 + b, chan_seed=90) for b, n in enumerate(lens)]
        for b, n in enumerate(lens):                                     # the earlier tokens, then the chunks
            pos = torch.arange(n, device="cuda")
            slots = bt[b, pos // S].to(torch.int64) * S + pos % S
            for a, e in ((0, n - chunk[b]), (n - chunk[b], n)):
                impl.do_kv_cache_update(layer, KV[b][0][a:e], KV[b][1][a:e], None, slots[a:e])
            orc.write_kv(0, np16(KV[b][0]), np16(KV[b][1]), np16(slots), np16(slots))
        cb.pool().check()
        q = torch.randn((sum(chunk), H * G, D), generator=g, device="cuda").to(torch.float16)
        meta = types.SimpleNamespace(max_query_len=40, num_actual_tokens=41, causal=True,
                                     query_start_loc=torch.tensor([0, 40, 41], dtype=torch.int32, device="cuda"),
                                     block_table=bt, seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"))
        out = torch.zeros((44, H * G, D), dtype=torch.float16, device="cuda")   # padded past 41 tokens
        impl.forward(layer, torch.cat([q, q[:3]]), None, None, None, meta, out)
        cb.pool().check()
        assert not impl.sent and torch.all(out[41:] == 0)
        rows = [(0, i, lens[0] - chunk[0] + i) for i in range(chunk[0])] + [(1, 40, lens[1] - 1)]
        for b, r, pos in rows:
            Kd, Vd = orc.dequant_sequence(0, np16(bt[b]), lens[b], v_pos="physical")
            o, _ = oatt.decode_attention(np16(q[r]).astype(np.float64), Kd[:pos + 1], Vd[:pos + 1])
            err = np.abs(np16(out[r]).astype(np.float64) - o)
            assert (err <= TOL + np.abs(o) * 2.0 ** -11).all(), err.max()
    finally:
        cb._FP16_CACHE = True
