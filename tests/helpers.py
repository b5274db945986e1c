"""Shared test helpers: build matching GPU and oracle pools, read device state."""
from __future__ import annotations

import numpy as np
import torch

from oracle.pool import LayerScalesNP, OraclePool


def np16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def oracle_scales(kvscales):
    out = []
    for ks, vs in zip(kvscales.per_layer_keys, kvscales.per_layer_values):
        out.append(LayerScalesNP(np16(ks.poles.half()), np16(ks.upper_threshold.half()),
                                 np16(ks.lower_threshold.half()), np16(vs.poles.half()),
                                 np16(vs.upper_threshold.half()), np16(vs.lower_threshold.half())))
    return out


def make_pools(kvscales, num_blocks, block_size, H, D, device="cuda", **kw):
    from kvquant.compact_pool import CompactKVPool
    gpu = CompactKVPool(kvscales.num_layers, num_blocks, block_size, H, D, kvscales, device=device, **kw)
    orc = OraclePool(kvscales.num_layers, num_blocks, block_size, H, D, oracle_scales(kvscales))
    return gpu, orc


def write_both(gpu, orc, layer, key, value, slots, pos):
    gpu.write_kv(layer, key, value, slots, pos)
    orc.write_kv(layer, np16(key), np16(value), np16(slots), np16(pos))


def gpu_codes(gpu, layer):
    """(K rows (H, NB, S, RBk), V rows (H, NB, S, RBv)) as numpy."""
    lay = gpu.layers[layer]
    S, D = gpu.block_size, gpu.head_size
    rbk, rbv = D * lay.bits_k // 8, D * lay.bits_v // 8
    c = np16(lay.codes)
    H, NB, _ = c.shape
    return c[:, :, :S * rbk].reshape(H, NB, S, rbk), c[:, :, S * rbk:].reshape(H, NB, S, rbv)


def gpu_outlier_array(gpu, layer):
    """Every outlier entry of the GPU pool as rows (h, page, kv, slot, d,
    fp16 bits), sorted; the order inside a page list is not part of the format."""
    lay = gpu.layers[layer]
    d = np16(lay.dir).astype(np.int64)                        # (H, NB, 2, 4)
    arena = np16(lay.arena).astype(np.int64) & 0xFFFFFFFF
    off, cnt = d[..., 0].reshape(-1), d[..., 2].reshape(-1)
    if cnt.sum() == 0:
        return np.zeros((0, 6), np.int64)
    rec = np.repeat(np.arange(off.size), cnt)
    start = np.repeat(np.cumsum(cnt) - cnt, cnt)
    e = arena[np.repeat(off, cnt) + np.arange(cnt.sum()) - start]
    H, NB = d.shape[:2]
    h, rest = np.divmod(rec, NB * 2)
    b, kv = np.divmod(rest, 2)
    a = np.stack([h, b, kv, (e >> 24) & 31, (e >> 16) & 255, e & 0xFFFF], axis=1)
    return a[np.lexsort(a.T[::-1])]


def _sets(a):
    out = {}
    for h, b, kv, s, d, bits in a.tolist():
        out.setdefault((h, b, kv), []).append((s, d, bits))
    return {k: sorted(v) for k, v in out.items()}


def gpu_outlier_sets(gpu, layer):
    """{(h, page, kv): sorted [(slot, d, bits)]} for every non-empty list."""
    return _sets(gpu_outlier_array(gpu, layer))


def oracle_outlier_sets(orc, layer):
    return _sets(orc.outlier_array(layer))
