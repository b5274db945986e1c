"""vLLM hook, quantise-dequantise mode (the reference's Phase 1A,
src/kvquant/vllm_backend.py:60-230).

``install_kvquant_backend(scales_path, device)`` loads the scales and points
vLLM's ``FlashAttentionBackend.get_impl_cls`` at ``KVQuantAttentionImpl``,
which replaces the step's K and V (the first ``num_actual_tokens`` rows) by
their nuq reconstruction before FlashAttention caches and attends to them:
K with its per-channel scales, V with its per-token scales at row
min(position, t_cal - 1) (vllm_backend.py:112-162). The pack and unpack are
this library's batched CUDA kernels (``kvquant.batched``). vLLM's fp16 cache
layout is unchanged; ``kvquant.compact_backend`` is the packed-pool mode.
"""
from __future__ import annotations

import re

import torch

from .batched import (pack_keys_per_channel_batched, pack_values_per_token_batched,
                      unpack_keys_per_channel_batched, unpack_values_per_token_batched)
from .scales import KVScales, PerChannelScale, PerTokenScale

_SCALES: KVScales | None = None
_LAYER_INDEX: dict[str, int] = {}
_IMPL_CLS = None


def layer_index(layer) -> int | None:
    """N from ``...layers.N....`` in layer_name, else first-seen order."""
    name = getattr(layer, "layer_name", "") or ""
    if not name:
        return None
    m = re.search(r"layers?\.(\d+)\.", name)
    if m:
        return int(m.group(1))
    if name not in _LAYER_INDEX:
        _LAYER_INDEX[name] = len(_LAYER_INDEX)
    return _LAYER_INDEX[name]


def quant_dequant_kv(key: torch.Tensor, value: torch.Tensor, k_scale: PerChannelScale, v_scale: PerTokenScale):
    """nuq reconstruction of (T, H, D) key and value, in their dtype. Token t
    uses V scale row min(t, t_cal - 1) (positions counted from the step's
    first token, as the reference wrapper does)."""
    if key.numel() == 0:
        return key, value
    T = key.shape[0]
    k16 = key.to(torch.float16).contiguous()
    v16 = value.to(torch.float16).contiguous()
    kc, kov, kom = pack_keys_per_channel_batched(k16, k_scale.poles, k_scale.upper_threshold,
                                                 k_scale.lower_threshold)
    kq = unpack_keys_per_channel_batched(kc, kov, kom, k_scale.poles)
    rows = torch.arange(T, device=value.device).clamp_(max=v_scale.poles.shape[1] - 1)
    vp = v_scale.poles.index_select(1, rows).contiguous()
    vu = v_scale.upper_threshold.index_select(1, rows).contiguous()
    vl = v_scale.lower_threshold.index_select(1, rows).contiguous()
    vc, vov, vom = pack_values_per_token_batched(v16, vp, vu, vl)
    vq = unpack_values_per_token_batched(vc, vov, vom, vp)
    return kq.to(key.dtype), vq.to(value.dtype)


def make_impl_cls(base):
    """The quantise-dequantise impl as a subclass of ``base``."""

    class KVQuantAttentionImpl(base):
        can_return_lse_for_decode: bool = True

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            sc = _SCALES
            idx = layer_index(layer)
            n = int(getattr(attn_metadata, "num_actual_tokens", 0)) if attn_metadata is not None else 0
            if sc is not None and idx is not None and idx < sc.num_layers and n > 0 and key.numel() > 0:
                with torch.no_grad():
                    kq, vq = quant_dequant_kv(key[:n], value[:n], sc.per_layer_keys[idx], sc.per_layer_values[idx])
                    if key.shape[0] > n:
                        key = torch.cat([kq, key[n:]], dim=0)
                        value = torch.cat([vq, value[n:]], dim=0)
                    else:
                        key, value = kq, vq
            return super().forward(layer, query, key, value, kv_cache, attn_metadata, output,
                                   output_scale, output_block_scale)

    KVQuantAttentionImpl.__name__ = "KVQuantAttentionImpl"
    KVQuantAttentionImpl.__qualname__ = "KVQuantAttentionImpl"
    return KVQuantAttentionImpl


def install_kvquant_backend(scales_path: str, device: str = "cuda:0", *, scales: KVScales | None = None,
                            backend_cls=None, impl_cls=None) -> None:
    """Load the scales and route vLLM's FlashAttention backend to
    ``KVQuantAttentionImpl``; call before building the vLLM engine."""
    global _SCALES, _IMPL_CLS
    if backend_cls is None or impl_cls is None:
        from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend, FlashAttentionImpl
        backend_cls = backend_cls or FlashAttentionBackend
        impl_cls = impl_cls or FlashAttentionImpl
    sc = scales if scales is not None else KVScales.load(scales_path, map_location=device)
    _SCALES = sc.to(device)
    _LAYER_INDEX.clear()
    _IMPL_CLS = make_impl_cls(impl_cls)
    backend_cls.get_impl_cls = staticmethod(lambda: _IMPL_CLS)
