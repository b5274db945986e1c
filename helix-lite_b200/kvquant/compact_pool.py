"""Compact paged KV pool (src/kvquant/compact_pool.py:398-537), B200 layout.

Constructor, ``write_kv`` and ``unpack_to_staging`` keep the reference's
signatures. Storage is the packed format of include/helix_kv.h rather than
one byte per code plus dense fp16 outliers (compact_pool.py:426-441):

  codes   (H, NB, seg) uint8 per layer; a (head, page) segment is the page's
          K code rows then its V code rows, 4 bits per code for up to 16
          levels, 2 bits for up to 4
  stats   (H, NB, 2, D) fp16: running min / max of reconstructed K per page
          (exact in fp16; the reference keeps fp32 only for sm_86 atomics)
  dir     (H, NB, 2, 4) int32: {offset, capacity, count, rows} of the page's
          sparse outlier list (K, V) in the layer's arena
  arena   int32 outlier entries: fp16 value | channel << 16 | slot << 24;
          sized by ``outlier_capacity`` entries or ``outlier_frac`` (one
          fraction, or one per layer) of the layer's K and V elements

Head-major, page-contiguous segments let the decode kernel move a page with
one bulk copy. Debug accessors (``k_codes``, ``k_outv``, ``k_outm``,
``k_min`` ...) rebuild the reference's dense tensors on demand.
"""
from __future__ import annotations

import math

import torch

import hxlib
from hxlib import PoolLayer, call, ptr, stream

from .scales import KVScales


def code_bits(levels: int) -> int:
    if levels <= 4:
        return 2
    if levels <= 16:
        return 4
    raise ValueError(f"at most 16 levels per code are supported, got {levels}")


class _Layer:
    def __init__(self, NB, S, H, D, bk, bv, arena_entries, device):
        self.seg = S * D * (bk + bv) // 8
        self.bits_k, self.bits_v = bk, bv
        self.codes = torch.zeros((H, NB, self.seg), dtype=torch.uint8, device=device)
        self.stats = torch.empty((H, NB, 2, D), dtype=torch.float16, device=device)
        self.dir = torch.zeros((H, NB, 2, 4), dtype=torch.int32, device=device)
        self.arena = torch.zeros((max(int(arena_entries), 1024),), dtype=torch.int32, device=device)
        self.arena_top = torch.zeros((1,), dtype=torch.int32, device=device)
        self.struct = PoolLayer(self.codes.data_ptr(), self.stats.data_ptr(), self.dir.data_ptr(),
                                self.arena.data_ptr(), self.arena_top.data_ptr(), self.arena.numel(),
                                NB, S, H, D, bk, bv)


class CompactKVPool:
    """A paged KV cache of packed nuq codes and sparse fp16 outliers."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                 head_size: int, scales: KVScales, device: str = "cuda:0",
                 outlier_capacity: int | None = None, outlier_frac=0.125):
        self.num_layers, self.num_blocks, self.block_size = num_layers, num_blocks, block_size
        self.num_kv_heads, self.head_size = num_kv_heads, head_size
        self.scales = scales
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise hxlib.HelixError("CompactKVPool lives on a CUDA device (no CPU fallback)")
        if block_size > 32 or head_size % 8 or head_size > 256:
            raise ValueError("block_size <= 32 and head_size a multiple of 8 up to 256 are supported")
        self._k_levels = [int(s.poles.shape[-1]) for s in scales.per_layer_keys]
        self._v_levels = [int(s.poles.shape[-1]) for s in scales.per_layer_values]
        elems = num_blocks * block_size * num_kv_heads * head_size * 2
        fracs = list(outlier_frac) if isinstance(outlier_frac, (list, tuple)) else [outlier_frac] * num_layers
        self.layers = []
        with torch.cuda.device(self.device):
            for i in range(num_layers):
                cap = outlier_capacity if outlier_capacity is not None else int(math.ceil(elems * fracs[i])) + 4096
                lay = _Layer(num_blocks, block_size, num_kv_heads, head_size, code_bits(self._k_levels[i]),
                             code_bits(self._v_levels[i]), cap, self.device)
                call("hx_pool_init", stream(self.device), ctypes_ref(lay.struct))
                self.layers.append(lay)

    # -- write side (compact_pool.py:447-489) --
    def write_kv(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor,
                 slot_mapping: torch.Tensor, abs_positions: torch.Tensor) -> None:
        assert layer_idx < self.num_layers
        assert key.is_contiguous(), "key must be contiguous (T, H, D)"
        assert value.is_contiguous()
        T = key.shape[0]
        if T == 0:
            return
        assert key.shape == (T, self.num_kv_heads, self.head_size) and value.shape == key.shape
        hxlib.require_cuda(key, value, slot_mapping, abs_positions)
        k = key if key.dtype == torch.float16 else key.to(torch.float16)
        v = value if value.dtype == torch.float16 else value.to(torch.float16)
        sm = slot_mapping.to(torch.int64).contiguous()
        ap = abs_positions.to(torch.int64).contiguous()
        st, _keep = self.scales.device_layer(layer_idx, self.device)
        lay = self.layers[layer_idx]
        with torch.cuda.device(self.device):
            call("hx_pack_append", stream(self.device), ctypes_ref(lay.struct), ctypes_ref(st), ptr(k), ptr(v),
                 ptr(sm), ptr(ap), T, ptr(hxlib.err_word(self.device)))

    # -- read side (compact_pool.py:492-537) --
    def unpack_to_staging(self, layer_idx: int, block_id_list: torch.Tensor, block_first_position: torch.Tensor,
                          staging_k: torch.Tensor, staging_v: torch.Tensor) -> None:
        assert layer_idx < self.num_layers
        NK = block_id_list.shape[0]
        shape = (NK, self.block_size, self.num_kv_heads, self.head_size)
        assert tuple(staging_k.shape) == shape, f"staging_k shape {tuple(staging_k.shape)} != {shape}"
        assert staging_v.shape == staging_k.shape
        assert staging_k.dtype == torch.float16 and staging_v.dtype == torch.float16
        assert staging_k.is_contiguous() and staging_v.is_contiguous()
        if NK == 0:
            return
        ids = block_id_list.to(torch.int64).contiguous()
        fp = block_first_position.to(torch.int64).contiguous()
        st, _keep = self.scales.device_layer(layer_idx, self.device)
        with torch.cuda.device(self.device):
            call("hx_unpack_pages", stream(self.device), ctypes_ref(self.layers[layer_idx].struct),
                 ctypes_ref(st), ptr(ids), ptr(fp), NK, ptr(staging_k), ptr(staging_v),
                 ptr(hxlib.err_word(self.device)))

    def reset_pages(self, layer_idx: int, pages: torch.Tensor) -> None:
        """Empty pages (stats and outlier lists) before they are reused."""
        p = pages.to(device=self.device, dtype=torch.int32).contiguous()
        with torch.cuda.device(self.device):
            call("hx_pool_reset_pages", stream(self.device), ctypes_ref(self.layers[layer_idx].struct), ptr(p),
                 p.numel(), ptr(hxlib.err_word(self.device)))

    def check(self) -> None:
        """Synchronise and raise if a kernel flagged a device error."""
        hxlib.check_device_errors(self.device)

    # -- debug views in the reference's dense layout --------------------------
    def _codes_dense(self, kv: int) -> torch.Tensor:
        out = []
        S, H, D = self.block_size, self.num_kv_heads, self.head_size
        for lay in self.layers:
            bits = lay.bits_k if kv == 0 else lay.bits_v
            rb_k = D * lay.bits_k // 8
            rb = D * bits // 8
            base = 0 if kv == 0 else S * rb_k
            rows = lay.codes[:, :, base:base + S * rb].reshape(H, self.num_blocks, S, rb)
            per = 8 // bits
            shifts = torch.arange(per, device=self.device, dtype=torch.uint8) * bits
            c = (rows.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
            out.append(c.reshape(H, self.num_blocks, S, D).permute(1, 2, 0, 3))
        return torch.stack(out).contiguous()

    def _outliers_dense(self, kv: int):
        S, H, D, NB = self.block_size, self.num_kv_heads, self.head_size, self.num_blocks
        vals = torch.zeros((self.num_layers, NB, S, H, D), dtype=torch.float16, device=self.device)
        mask = torch.zeros((self.num_layers, NB, S, H, D), dtype=torch.uint8, device=self.device)
        for li, lay in enumerate(self.layers):
            d = lay.dir[:, :, kv].to(torch.int64)        # (H, NB, 4)
            off, cnt = d[..., 0], d[..., 2]
            tot = int(cnt.sum().item())
            if tot == 0:
                continue
            hh, bb = torch.nonzero(cnt > 0, as_tuple=True)
            for h, b in zip(hh.tolist(), bb.tolist()):
                e = lay.arena[int(off[h, b]):int(off[h, b]) + int(cnt[h, b])].to(torch.int64) & 0xFFFFFFFF
                v16 = (e & 0xFFFF).to(torch.int16).view(torch.float16)
                ch = (e >> 16) & 0xFF
                sl = (e >> 24) & 0x1F
                vals[li, b, sl, h, ch] = v16
                mask[li, b, sl, h, ch] = 1
        return vals, mask

    @property
    def k_codes(self):
        return self._codes_dense(0)

    @property
    def v_codes(self):
        return self._codes_dense(1)

    @property
    def k_outv(self):
        return self._outliers_dense(0)[0]

    @property
    def k_outm(self):
        return self._outliers_dense(0)[1]

    @property
    def v_outv(self):
        return self._outliers_dense(1)[0]

    @property
    def v_outm(self):
        return self._outliers_dense(1)[1]

    @property
    def k_min(self):
        return torch.stack([lay.stats[:, :, 0].permute(1, 0, 2).float() for lay in self.layers])

    @property
    def k_max(self):
        return torch.stack([lay.stats[:, :, 1].permute(1, 0, 2).float() for lay in self.layers])

    def outlier_entries(self, layer_idx: int, head: int, page: int, kv: int):
        """Sorted (slot, channel, fp16 bits) of one page list (parity tests)."""
        lay = self.layers[layer_idx]
        off, _cap, cnt, _rows = (int(x) for x in lay.dir[head, page, kv].tolist())
        e = lay.arena[off:off + cnt].to(torch.int64).cpu() & 0xFFFFFFFF
        return sorted(((int(x) >> 24) & 31, (int(x) >> 16) & 255, int(x) & 0xFFFF) for x in e.tolist())

    def arena_used(self, layer_idx: int) -> int:
        return int(self.layers[layer_idx].arena_top.item())

    # -- sizes --
    def segment_bytes(self, layer_idx: int) -> int:
        return self.layers[layer_idx].seg


def ctypes_ref(s):
    import ctypes
    return ctypes.byref(s)
