"""vLLM hook for the compact pool: pack on cache update, fused Quest decode.

Same entry point and behaviour as the reference's Phase 1B hook
(src/kvquant/compact_backend.py:70-300): ``install_compact_backend`` loads
the scales, allocates a shadow ``CompactKVPool`` and points vLLM's
``FlashAttentionBackend.get_impl_cls`` at ``KVQuantCompactImpl``, whose

  do_kv_cache_update  keeps vLLM's fp16 cache (prefill reads it) and also
                      packs the step's K/V into the compact pool (Kernel A);
  forward             on decode steps (max_query_len == 1) scores the pool's
                      pages, keeps each sequence's sinks + top-k per KV head
                      (Kernel B) and attends over the packed pages directly
                      (Kernel C); it writes ``output`` and returns it.

Where the reference unpacks the selected blocks into an fp16 staging buffer
and calls FlashAttention on it, one batch at a time and batch 1 only
(compact_backend.py:194-299), the fused decode reads the packed pages,
handles any batch of decode tokens in one call and never materialises fp16
K/V. Prefill, profiling runs and attention features the fused kernel does
not implement (sliding window, ALiBi, logits soft cap, attention sinks,
cross attention) go to FlashAttention unchanged.

With ``fp16_cache=False`` vLLM keeps no fp16 cache at all (the reference's
planned custom backend, src/kvquant/PHASE_1B_DESIGN.md:81-88): each decoder
layer's KV-cache spec asks for one KV head of one channel, so vLLM budgets
64 bytes per block and layer instead of the fp16 page, the backend's
``get_kv_cache_shape`` returns the matching (2, blocks, block_size, 1, 1)
placeholder, and the impl never touches ``kv_cache``: the cache update
packs into the compact pool only, decode steps run as above, and prefill or
mixed batches run the chunked-prefill kernel over the pool (every query
token attends causally to its sequence's packed tokens). vLLM must then be
given at most the pool's block count (``num_gpu_blocks_override``); the
kernels flag any block id past it.

The base classes are vLLM's (``vllm.v1.attention.backends.flash_attn``);
``backend_cls`` / ``impl_cls`` may be passed to install against other
classes with the same interface (the tests do).
"""
from __future__ import annotations

import re

import torch

from . import fused
from .compact_pool import CompactKVPool
from .scales import KVScales

# module state, set by install_compact_backend (the reference keeps the same
# globals: vLLM builds the impl objects itself and passes no extra arguments)
_POOL: CompactKVPool | None = None
_SCALES: KVScales | None = None
_TOP_K: int = 0            # decode top-k blocks per KV head; 0 = attend to every block
_SINK_BLOCKS: int = 4
_GQA: str = "mean"         # how the group's queries bound a page (the reference hook: mean)
_LAYER_INDEX: dict[str, int] = {}
_IMPL_CLS = None
_FP16_CACHE: bool = True   # False: vLLM keeps no fp16 cache; prefill reads the pool


def layer_index(layer) -> int | None:
    """Transformer layer of a vLLM Attention module: N from a layer_name like
    ``model.layers.N.self_attn.attn``, else first-seen order of the names
    (compact_backend.py:127-134)."""
    name = getattr(layer, "layer_name", "") or ""
    m = re.search(r"layers?\.(\d+)\.", name)
    if m:
        return int(m.group(1))
    if not name:
        return None
    if name not in _LAYER_INDEX:
        _LAYER_INDEX[name] = len(_LAYER_INDEX)
    return _LAYER_INDEX[name]


def _unsupported(impl) -> bool:
    """Attention options the fused decode does not implement."""
    window = getattr(impl, "sliding_window", None)
    if window is not None and tuple(window) not in ((-1, -1), (-1, 0)):
        return True
    return (getattr(impl, "alibi_slopes", None) is not None
            or bool(getattr(impl, "logits_soft_cap", None))
            or getattr(impl, "sinks", None) is not None)


def make_impl_cls(base):
    """The compact-pool impl as a subclass of ``base`` (a FlashAttentionImpl)."""

    class KVQuantCompactImpl(base):
        can_return_lse_for_decode: bool = True

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            if _FP16_CACHE:
                super().do_kv_cache_update(layer, key, value, kv_cache, slot_mapping)
            pool = _POOL
            idx = layer_index(layer)
            n = int(slot_mapping.shape[0])
            if pool is None or idx is None or idx >= pool.num_layers or n == 0:
                return
            slots = slot_mapping[:n].to(torch.int64)
            # a token's absolute position is taken as its slot, as the
            # reference hook does (compact_backend.py:157-167); the decode
            # reads V back with the same rule (v_pos="physical"), so a page's
            # V scale rows follow its pool block wherever vLLM put it
            pool.write_kv(idx, key[:n].to(torch.float16), value[:n].to(torch.float16), slots, slots)

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            pool = _POOL
            idx = layer_index(layer)
            passthrough = (pool is None or attn_metadata is None or idx is None or idx >= pool.num_layers
                           or output_scale is not None or output_block_scale is not None
                           or getattr(attn_metadata, "max_query_len", 0) != 1
                           or getattr(attn_metadata, "block_table", None) is None
                           or getattr(attn_metadata, "seq_lens", None) is None
                           or getattr(attn_metadata, "causal", True) is False
                           or _unsupported(self))
            if passthrough and not _FP16_CACHE:
                # no fp16 cache to fall back on: prefill and mixed batches read
                # the pool; what the kernels do not implement is an error
                if attn_metadata is None:
                    return output                 # profiling run: nothing cached yet
                if (pool is None or idx is None or idx >= pool.num_layers or _unsupported(self)
                        or output_scale is not None or output_block_scale is not None
                        or getattr(attn_metadata, "causal", True) is False):
                    raise NotImplementedError("the compact-pool backend without an fp16 cache supports causal "
                                              "decoder attention of the pool's layers only")
                if getattr(attn_metadata, "max_query_len", 0) != 1:
                    return prefill_into(pool, idx, query, attn_metadata, output, scale=float(self.scale))
            elif passthrough:
                return super().forward(layer, query, key, value, kv_cache, attn_metadata, output,
                                       output_scale, output_block_scale)
            return decode_into(pool, idx, query, attn_metadata, output, scale=float(self.scale))

    KVQuantCompactImpl.__name__ = "KVQuantCompactImpl"
    KVQuantCompactImpl.__qualname__ = "KVQuantCompactImpl"
    return KVQuantCompactImpl


def decode_into(pool: CompactKVPool, idx: int, query: torch.Tensor, attn_metadata, output: torch.Tensor,
                scale: float) -> torch.Tensor:
    """One decode token per sequence: Quest selection + fused decode over
    the pool, written into ``output[:num_actual_tokens]``."""
    n = int(getattr(attn_metadata, "num_actual_tokens", query.shape[0]))
    B = n  # one token per sequence; rows past n are padding
    if attn_metadata.block_table.shape[0] < B:
        raise ValueError(f"decode expects one token per sequence: {n} tokens, "
                         f"{attn_metadata.block_table.shape[0]} block-table rows")
    bt = attn_metadata.block_table[:B]
    Hq, D = query.shape[-2], query.shape[-1]
    q = query[:n].reshape(B, Hq, D)
    seq_lens = attn_metadata.seq_lens[:B]
    if _TOP_K > 0:
        sel = fused.quest_select(pool, idx, q, bt, seq_lens, top_k=_TOP_K, sink_pages=_SINK_BLOCKS, gqa=_GQA)
        o, _ = fused.decode(pool, idx, q, bt, seq_lens, sel, softmax_scale=scale, v_pos="physical")
    else:
        o, _ = fused.decode(pool, idx, q, bt, seq_lens, softmax_scale=scale, v_pos="physical")
    out = output[:n].view(B, Hq, D)
    out.copy_(o.to(out.dtype))
    return output


def prefill_into(pool: CompactKVPool, idx: int, query: torch.Tensor, attn_metadata, output: torch.Tensor,
                 scale: float) -> torch.Tensor:
    """Every query token of the batch (prefill chunks and decode tokens alike)
    attends causally to its sequence's tokens in the pool; written into
    ``output[:num_actual_tokens]``."""
    n = int(getattr(attn_metadata, "num_actual_tokens", query.shape[0]))
    qsl = attn_metadata.query_start_loc
    B = int(qsl.shape[0]) - 1
    Hq, D = query.shape[-2], query.shape[-1]
    out = output[:n].view(n, Hq, D)
    o16, _ = fused.prefill(pool, idx, query[:n].reshape(n, Hq, D), qsl, attn_metadata.block_table[:B],
                           attn_metadata.seq_lens[:B], max_query_len=int(attn_metadata.max_query_len),
                           softmax_scale=scale, v_pos="physical",
                           out=out if out.dtype == torch.float16 and out.is_contiguous() else None)
    if o16.data_ptr() != out.data_ptr():
        out.copy_(o16.to(out.dtype))
    return output


def tiny_kv_cache_spec(spec):
    """A decoder layer's vLLM KV-cache spec reduced to one KV head of one
    channel: vLLM then budgets 2 * block_size * dtype bytes per block and
    layer, and keeps no fp16 K/V (the compact pool holds them)."""
    import dataclasses
    kw = {"num_kv_heads": 1, "head_size": 1}
    if hasattr(spec, "head_size_v"):
        kw["head_size_v"] = 1
    return dataclasses.replace(spec, **kw)


def tiny_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int = 1, head_size: int = 1,
                        cache_dtype_str: str = "auto") -> tuple[int, ...]:
    """FlashAttentionBackend.get_kv_cache_shape's layout at one head of one
    channel: the placeholder vLLM allocates in place of the fp16 cache."""
    return (2, num_blocks, block_size, 1, 1)


def install_compact_backend(scales_path: str, *, num_layers: int = 28, num_blocks: int = 16_384,
                            block_size: int = 16, num_kv_heads: int = 4, head_size: int = 128,
                            device: str = "cuda:0", top_k_blocks_decode: int = 0, sink_blocks: int = 4,
                            gqa: str = "mean", scales: KVScales | None = None, backend_cls=None,
                            impl_cls=None, fp16_cache: bool = True, attention_cls=None) -> None:
    """Allocate the compact pool and route vLLM's FlashAttention backend to
    ``KVQuantCompactImpl`` (compact_backend.py:70-119). Call before building
    the vLLM engine. ``top_k_blocks_decode`` = 0 attends to every block;
    ``scales`` (already loaded) takes the place of ``scales_path``.
    ``fp16_cache=False`` also removes vLLM's fp16 cache: ``attention_cls``
    (vLLM's Attention layer by default) reports the tiny KV-cache spec and
    ``backend_cls`` the tiny shape; prefill then reads the compact pool."""
    global _POOL, _SCALES, _TOP_K, _SINK_BLOCKS, _GQA, _IMPL_CLS, _FP16_CACHE
    if backend_cls is None or impl_cls is None:
        from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend, FlashAttentionImpl
        backend_cls = backend_cls or FlashAttentionBackend
        impl_cls = impl_cls or FlashAttentionImpl
    if not fp16_cache and attention_cls is None:
        from vllm.model_executor.layers.attention.attention import Attention
        attention_cls = Attention
    sc = scales if scales is not None else KVScales.load(scales_path, map_location=device)
    sc = sc.to(device)
    if sc.num_layers != num_layers:
        raise ValueError(f"scales have {sc.num_layers} layers, expected {num_layers}")
    if gqa not in ("mean", "sum"):
        raise ValueError("gqa must be 'mean' or 'sum'")
    _SCALES = sc
    _POOL = CompactKVPool(num_layers, num_blocks, block_size, num_kv_heads, head_size, sc, device=device)
    _TOP_K = int(top_k_blocks_decode)
    _SINK_BLOCKS = int(sink_blocks)
    _GQA = gqa
    _LAYER_INDEX.clear()
    _IMPL_CLS = make_impl_cls(impl_cls)
    _FP16_CACHE = bool(fp16_cache)
    backend_cls.get_impl_cls = staticmethod(lambda: _IMPL_CLS)
    if not fp16_cache:
        backend_cls.get_kv_cache_shape = staticmethod(tiny_kv_cache_shape)
        base_spec = getattr(attention_cls, "_hx_base_kv_cache_spec", attention_cls.get_kv_cache_spec)

        def get_kv_cache_spec(self, vllm_config):
            spec = base_spec(self, vllm_config)
            return tiny_kv_cache_spec(spec) if spec is not None else None

        attention_cls._hx_base_kv_cache_spec = base_spec
        attention_cls.get_kv_cache_spec = get_kv_cache_spec


def pool() -> CompactKVPool | None:
    """The installed compact pool (None before install_compact_backend)."""
    return _POOL
