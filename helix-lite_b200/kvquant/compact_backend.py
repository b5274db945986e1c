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
            if passthrough:
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


def install_compact_backend(scales_path: str, *, num_layers: int = 28, num_blocks: int = 16_384,
                            block_size: int = 16, num_kv_heads: int = 4, head_size: int = 128,
                            device: str = "cuda:0", top_k_blocks_decode: int = 0, sink_blocks: int = 4,
                            gqa: str = "mean", scales: KVScales | None = None, backend_cls=None,
                            impl_cls=None) -> None:
    """Allocate the compact pool and route vLLM's FlashAttention backend to
    ``KVQuantCompactImpl`` (compact_backend.py:70-119). Call before building
    the vLLM engine. ``top_k_blocks_decode`` = 0 attends to every block;
    ``scales`` (already loaded) takes the place of ``scales_path``."""
    global _POOL, _SCALES, _TOP_K, _SINK_BLOCKS, _GQA, _IMPL_CLS
    if backend_cls is None or impl_cls is None:
        from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend, FlashAttentionImpl
        backend_cls = backend_cls or FlashAttentionBackend
        impl_cls = impl_cls or FlashAttentionImpl
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
    backend_cls.get_impl_cls = staticmethod(lambda: _IMPL_CLS)


def pool() -> CompactKVPool | None:
    """The installed compact pool (None before install_compact_backend)."""
    return _POOL
