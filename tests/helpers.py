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


def gpu_outlier_sets(gpu, layer):
    """{(h, page, kv): sorted [(slot, d, bits)]} for every non-empty list."""
    lay = gpu.layers[layer]
    d = np16(lay.dir).astype(np.int64)
    arena = np16(lay.arena).astype(np.int64) & 0xFFFFFFFF
    out = {}
    H, NB = d.shape[:2]
    for h in range(H):
        for b in range(NB):
            for kv in range(2):
                off, _cap, cnt, _rows = d[h, b, kv]
                if cnt:
                    e = arena[off:off + cnt]
                    out[(h, b, kv)] = sorted(zip(((e >> 24) & 31).tolist(), ((e >> 16) & 255).tolist(),
                                                 (e & 0xFFFF).tolist()))
    return out


def oracle_outlier_sets(orc, layer):
    out = {}
    for (h, pg, kv, s), (d, v) in orc.rows[layer].items():
        if d.size:
            out.setdefault((h, pg, kv), []).extend(
                (s, int(dd), int(bb)) for dd, bb in zip(d, v.view(np.uint16)))
    return {k: sorted(v) for k, v in out.items()}
