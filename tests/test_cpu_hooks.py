"""The vLLM hooks' routing, on the CPU with stand-in base classes (the
reference's hooks subclass vLLM's FlashAttentionImpl; compact_backend.py
and vllm_backend.py). The CUDA work is replaced by recorders here; the GPU
file tests the same hooks end to end."""
from __future__ import annotations

import types

import pytest
import torch


class FakeImpl:
    """Stands in for FlashAttentionImpl: records what reaches it."""
    def __init__(self, scale=0.125, sliding_window=(-1, -1), alibi_slopes=None, logits_soft_cap=0, sinks=None):
        self.scale, self.sliding_window = scale, sliding_window
        self.alibi_slopes, self.logits_soft_cap, self.sinks = alibi_slopes, logits_soft_cap, sinks
        self.calls = []

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        self.calls.append(("forward", key.clone()))
        return output

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        self.calls.append(("update", slot_mapping.clone()))


class FakeBackend:
    @staticmethod
    def get_impl_cls():
        return FakeImpl


class FakePool:
    num_layers = 4

    def __init__(self):
        self.writes = []

    def write_kv(self, layer, key, value, slots, pos):
        self.writes.append((layer, key.dtype, value.dtype, slots.tolist(), pos.tolist()))


def _meta(B, max_q, Hmax=6):
    return types.SimpleNamespace(max_query_len=max_q, num_actual_tokens=B, causal=True,
                                 block_table=torch.arange(B * Hmax, dtype=torch.int32).reshape(B, Hmax),
                                 seq_lens=torch.full((B,), 80, dtype=torch.int32))


def _layer(i):
    return types.SimpleNamespace(layer_name=f"model.layers.{i}.self_attn.attn")


@pytest.fixture
def compact(monkeypatch):
    from kvquant import compact_backend as cb
    calls = []

    def quest_select(pool, li, q, bt, sl, **kw):
        calls.append(("select", li, tuple(q.shape), kw))
        return "sel"

    def decode(pool, li, q, bt, sl, sel=None, **kw):
        calls.append(("decode", li, sel, kw))
        return torch.full(q.shape, 0.5), torch.zeros(q.shape[:2])

    monkeypatch.setattr(cb, "fused", types.SimpleNamespace(quest_select=quest_select, decode=decode))
    pool = FakePool()
    monkeypatch.setattr(cb, "_POOL", pool)
    monkeypatch.setattr(cb, "_TOP_K", 8)
    monkeypatch.setattr(cb, "_SINK_BLOCKS", 4)
    monkeypatch.setattr(cb, "_GQA", "mean")
    return cb, pool, calls


def test_compact_decode_goes_to_the_fused_path(compact):
    cb, pool, calls = compact
    impl = cb.make_impl_cls(FakeImpl)()
    B, Hq, D = 3, 28, 128
    q = torch.randn(B + 2, Hq, D)          # rows past num_actual_tokens are padding
    out = torch.zeros(B + 2, Hq, D, dtype=torch.float16)
    k = torch.randn(B + 2, 4, D)
    r = impl.forward(_layer(2), q, k, k, None, _meta(B, 1), out)
    assert r is out
    assert not impl.calls                   # FlashAttention not used
    assert calls[0][0] == "select" and calls[0][1] == 2 and calls[0][2] == (B, Hq, D)
    assert calls[0][3] == {"top_k": 8, "sink_pages": 4, "gqa": "mean"}
    assert calls[1][0] == "decode" and calls[1][2] == "sel" and calls[1][3]["softmax_scale"] == 0.125
    # V is packed with abs_positions = slot, so it is read back by physical slot
    assert calls[1][3]["v_pos"] == "physical"
    assert torch.all(out[:B] == 0.5) and torch.all(out[B:] == 0)


def test_compact_passthrough_cases(compact):
    cb, pool, calls = compact
    q = torch.randn(4, 28, 128)
    out = torch.zeros_like(q)
    impl = cb.make_impl_cls(FakeImpl)()
    impl.forward(_layer(0), q, q, q, None, _meta(4, 7), out)           # prefill
    impl.forward(_layer(0), q, q, q, None, None, out)                  # profiling run
    impl.forward(_layer(9), q, q, q, None, _meta(4, 1), out)           # layer past the pool
    windowed = cb.make_impl_cls(FakeImpl)
    w = windowed(sliding_window=(511, 0))
    w.forward(_layer(0), q, q, q, None, _meta(4, 1), out)              # sliding window
    s = windowed(alibi_slopes=[0.1])
    s.forward(_layer(0), q, q, q, None, _meta(4, 1), out)              # ALiBi
    assert len(impl.calls) == 3 and len(w.calls) == 1 and len(s.calls) == 1
    assert not calls


def test_compact_top_k_zero_attends_every_block(compact, monkeypatch):
    cb, pool, calls = compact
    monkeypatch.setattr(cb, "_TOP_K", 0)
    q = torch.randn(2, 28, 128)
    impl = cb.make_impl_cls(FakeImpl)()
    impl.forward(_layer(1), q, q, q, None, _meta(2, 1), torch.zeros_like(q))
    assert [c[0] for c in calls] == ["decode"] and calls[0][2] is None


def test_compact_cache_update_mirrors_into_the_pool(compact):
    cb, pool, calls = compact
    impl = cb.make_impl_cls(FakeImpl)()
    key = torch.randn(5, 4, 128, dtype=torch.bfloat16)
    slots = torch.tensor([32, 33, 34, 35, 36])
    impl.do_kv_cache_update(_layer(3), key, key, None, slots)
    assert impl.calls[0][0] == "update"
    assert pool.writes == [(3, torch.float16, torch.float16, [32, 33, 34, 35, 36], [32, 33, 34, 35, 36])]


def test_layer_index_rules():
    from kvquant import compact_backend as cb
    cb._LAYER_INDEX.clear()
    assert cb.layer_index(_layer(17)) == 17
    assert cb.layer_index(types.SimpleNamespace(layer_name="decoder.attn_a")) == 0
    assert cb.layer_index(types.SimpleNamespace(layer_name="decoder.attn_b")) == 1
    assert cb.layer_index(types.SimpleNamespace(layer_name="decoder.attn_a")) == 0
    assert cb.layer_index(types.SimpleNamespace()) is None


def test_quantise_dequantise_hook_install_and_route(monkeypatch):
    from kvquant import vllm_backend as vb
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    H, D, L, Tc = 4, 128, 16, 64
    ks = PerChannelScale(torch.zeros(H, D, L, dtype=torch.float16), torch.ones(H, D, dtype=torch.float16),
                         -torch.ones(H, D, dtype=torch.float16), 4)
    vs = PerTokenScale(torch.zeros(H, Tc, L, dtype=torch.float16), torch.ones(H, Tc, dtype=torch.float16),
                       -torch.ones(H, Tc, dtype=torch.float16), 4)
    backend = type("Backend", (FakeBackend,), {})
    vb.install_kvquant_backend("", device="cpu", scales=KVScales([ks, ks], [vs, vs]), backend_cls=backend,
                               impl_cls=FakeImpl)
    cls = backend.get_impl_cls()
    assert cls.__name__ == "KVQuantAttentionImpl" and issubclass(cls, FakeImpl)
    seen = []

    def qd(k, v, kscale, vscale):
        seen.append(k.shape[0])
        return k + 1, v + 1
    monkeypatch.setattr(vb, "quant_dequant_kv", qd)
    impl = cls()
    key = torch.zeros(6, H, D)
    impl.forward(_layer(1), key, key, key, None, types.SimpleNamespace(num_actual_tokens=4), key)
    sent = impl.calls[0][1]
    assert seen == [4] and torch.all(sent[:4] == 1) and torch.all(sent[4:] == 0)
    impl.forward(_layer(7), key, key, key, None, types.SimpleNamespace(num_actual_tokens=4), key)
    assert torch.all(impl.calls[1][1] == 0)    # no scales for layer 7: unchanged


def test_hooks_subclass_the_installed_vllm_impl():
    """The hooks build on vLLM 0.22's FlashAttentionImpl, whose forward and
    do_kv_cache_update signatures they keep."""
    import inspect
    fa = pytest.importorskip("vllm.v1.attention.backends.flash_attn")
    from kvquant import compact_backend as cb
    from kvquant import vllm_backend as vb
    for mk in (cb.make_impl_cls, vb.make_impl_cls):
        cls = mk(fa.FlashAttentionImpl)
        assert issubclass(cls, fa.FlashAttentionImpl)
    base = inspect.signature(fa.FlashAttentionImpl.forward).parameters
    assert list(base)[:8] == ["self", "layer", "query", "key", "value", "kv_cache", "attn_metadata", "output"]
    assert list(inspect.signature(fa.FlashAttentionImpl.do_kv_cache_update).parameters) == \
        ["self", "layer", "key", "value", "kv_cache", "slot_mapping"]


class FakeAttention:
    """Stands in for vLLM's Attention layer: reports an fp16 cache spec."""
    def get_kv_cache_spec(self, vllm_config):
        fa = pytest.importorskip("vllm.v1.kv_cache_interface")
        return fa.FullAttentionSpec(block_size=16, num_kv_heads=4, head_size=128, dtype=torch.float16)


def test_no_fp16_cache_install_shrinks_vllm_cache(monkeypatch):
    """fp16_cache=False: the layer spec asks for one head of one channel (64
    bytes per block and layer instead of 32 KB) and the backend's shape is the
    matching placeholder; the impl never calls FlashAttention's cache update."""
    from kvquant import compact_backend as cb
    from kvquant.scales import KVScales, PerChannelScale, PerTokenScale
    H, D, L, Tc = 4, 128, 16, 64
    ks = PerChannelScale(torch.zeros(H, D, L, dtype=torch.float16), torch.ones(H, D, dtype=torch.float16),
                         -torch.ones(H, D, dtype=torch.float16), 4)
    vs = PerTokenScale(torch.zeros(H, Tc, L, dtype=torch.float16), torch.ones(H, Tc, dtype=torch.float16),
                       -torch.ones(H, Tc, dtype=torch.float16), 4)
    monkeypatch.setattr(cb, "CompactKVPool", lambda *a, **k: FakePool())
    backend = type("Backend", (FakeBackend,), {})
    attn = type("Attn", (FakeAttention,), {})
    full = FakeAttention().get_kv_cache_spec(None)
    cb.install_compact_backend("", num_layers=2, device="cpu", scales=KVScales([ks, ks], [vs, vs]),
                               backend_cls=backend, impl_cls=FakeImpl, fp16_cache=False, attention_cls=attn)
    try:
        spec = attn().get_kv_cache_spec(None)
        assert full.page_size_bytes == 2 * 16 * 4 * 128 * 2
        assert spec.page_size_bytes == 2 * 16 * 1 * 1 * 2 and spec.block_size == 16
        assert backend.get_kv_cache_shape(100, 16, 1, 1) == (2, 100, 16, 1, 1)
        # installing again keeps one level of wrapping
        cb.install_compact_backend("", num_layers=2, device="cpu", scales=KVScales([ks, ks], [vs, vs]),
                                   backend_cls=backend, impl_cls=FakeImpl, fp16_cache=False, attention_cls=attn)
        assert attn().get_kv_cache_spec(None).page_size_bytes == 64
        impl = backend.get_impl_cls()()
        key = torch.randn(3, 4, 128)
        impl.do_kv_cache_update(_layer(1), key, key, None, torch.tensor([5, 6, 7]))
        assert not impl.calls and cb.pool().writes[0][0] == 1 and cb.pool().writes[0][3] == [5, 6, 7]
    finally:
        monkeypatch.setattr(cb, "_FP16_CACHE", True)


def test_no_fp16_cache_prefill_reads_the_pool(compact, monkeypatch):
    """Prefill and mixed batches go to the chunked-prefill kernel with vLLM's
    query_start_loc / seq_lens / block_table; a profiling run is a no-op and
    options the kernels lack raise instead of falling back."""
    cb, pool, calls = compact
    monkeypatch.setattr(cb, "_FP16_CACHE", False)
    seen = []

    def prefill(pool_, li, q, qs, bt, sl, **kw):
        seen.append((li, tuple(q.shape), qs.tolist(), tuple(bt.shape), sl.tolist(), kw["max_query_len"],
                     kw["v_pos"], kw["softmax_scale"]))
        return torch.full(q.shape, 0.25, dtype=torch.float16), None

    monkeypatch.setattr(cb.fused, "prefill", prefill, raising=False)
    impl = cb.make_impl_cls(FakeImpl)()
    q = torch.randn(9, 28, 128)
    out = torch.zeros(9, 28, 128, dtype=torch.float16)
    meta = types.SimpleNamespace(max_query_len=5, num_actual_tokens=7, causal=True,
                                 query_start_loc=torch.tensor([0, 5, 6, 7], dtype=torch.int32),
                                 block_table=torch.zeros((3, 6), dtype=torch.int32),
                                 seq_lens=torch.tensor([40, 17, 90], dtype=torch.int32))
    impl.forward(_layer(2), q, q, q, None, meta, out)
    assert seen == [(2, (7, 28, 128), [0, 5, 6, 7], (3, 6), [40, 17, 90], 5, "physical", 0.125)]
    assert torch.all(out[:7] == 0.25) and torch.all(out[7:] == 0) and not impl.calls
    assert impl.forward(_layer(2), q, q, q, None, None, out) is out      # profiling run
    w = cb.make_impl_cls(FakeImpl)(sliding_window=(511, 0))
    with pytest.raises(NotImplementedError):
        w.forward(_layer(2), q, q, q, None, meta, out)
    impl.forward(_layer(2), q, q, q, None, _meta(3, 1), out)            # decode: the Quest path
    assert [c[0] for c in calls] == ["select", "decode"]
