"""Compact paged KV pool restated in numpy (test infrastructure only).

Follows src/kvquant/compact_pool.py:
  * ``write_kv``           :447-489 (K kernel :222-287, V kernel :161-218)
  * V tail clamp           :467 (``pos = min(abs_pos, T_cal - 1)``)
  * skip negative slots    :245-247
  * K page stats           :285-287 (running min / max of the reconstructed K)
  * ``unpack_to_staging``  :492-537 (K :293-340, V :344-395, V clamp :372)

The storage format is the build's (the reference stores dense 1-byte codes
plus dense fp16 outlier values and masks, :426-432):
  * codes   [layer] per (head, page) one segment: K rows (S, D*bk/8) then
            V rows (S, D*bv/8), rows packed by ``oracle.packing``; bk / bv
            are 2 (up to 4 levels) or 4 (up to 16 levels)
  * stats   [layer] (H, NB, 2, D) fp16: [.,.,0] running min, [.,.,1] running
            max of reconstructed K; +inf / -inf until the page is written
  * outliers: for every (head, page, K|V, slot) the ascending channel list
            with the original fp16 values. Writing a slot replaces its list,
            exactly as the dense store overwrites a slot.
"""
from __future__ import annotations

import numpy as np

from .nuq import band_outliers, nearest_codes
from .packing import pack_codes, unpack_codes


class LayerScalesNP:
    """Host copy of one layer's scales (shapes of src/kvquant/scales.py:14-70)."""

    def __init__(self, k_poles, k_upper, k_lower, v_poles, v_upper, v_lower):
        self.k_poles = np.asarray(k_poles, dtype=np.float16)   # (H, D, Lk)
        self.k_upper = np.asarray(k_upper, dtype=np.float16)   # (H, D)
        self.k_lower = np.asarray(k_lower, dtype=np.float16)
        self.v_poles = np.asarray(v_poles, dtype=np.float16)   # (H, Tc, Lv)
        self.v_upper = np.asarray(v_upper, dtype=np.float16)   # (H, Tc)
        self.v_lower = np.asarray(v_lower, dtype=np.float16)

    @property
    def t_cal(self) -> int:
        return self.v_poles.shape[1]

    @property
    def bits_k(self) -> int:
        return code_bits(self.k_poles.shape[-1])

    @property
    def bits_v(self) -> int:
        return code_bits(self.v_poles.shape[-1])


def code_bits(levels: int) -> int:
    """Packed width of a code: 2 bits up to 4 levels, 4 bits up to 16."""
    if levels <= 4:
        return 2
    if levels <= 16:
        return 4
    raise ValueError(f"at most 16 levels are supported, got {levels}")


def quantize_k_rows(x, sc: LayerScalesNP):
    """K rows x (N, H, D) fp16 -> codes (N, H, D), mask, recon fp16.

    The reconstruction of a non-outlier is its pole; when no level is closer
    than +inf (x NaN or infinite) the reference's scan keeps its initial pole
    0.0 (compact_pool.py:260-268), and so does this.
    """
    codes = nearest_codes(x, sc.k_poles[None])
    mask = band_outliers(x, sc.k_upper[None], sc.k_lower[None])
    pole = np.take_along_axis(np.broadcast_to(sc.k_poles[None], x.shape + (sc.k_poles.shape[-1],)),
                              codes[..., None].astype(np.int64), axis=-1)[..., 0]
    d = np.abs(x.astype(np.float32)[..., None] - sc.k_poles[None].astype(np.float32))
    none_closer = ~(d < np.float32(np.inf)).any(axis=-1)
    pole = np.where(none_closer, np.float16(0.0), pole)
    recon = np.where(mask, x, pole).astype(np.float16)
    return codes, mask, recon


def quantize_v_rows(x, pos, sc: LayerScalesNP):
    """V rows x (N, H, D) fp16 at absolute positions pos (N,)."""
    p = np.minimum(np.asarray(pos, dtype=np.int64), sc.t_cal - 1)
    poles = np.transpose(sc.v_poles[:, p], (1, 0, 2))        # (N, H, L)
    codes = nearest_codes(x, poles[:, :, None, :])
    up = np.transpose(sc.v_upper[:, p])[:, :, None]           # (N, H, 1)
    lo = np.transpose(sc.v_lower[:, p])[:, :, None]
    mask = band_outliers(x, up, lo)
    return codes, mask


class OraclePool:
    """The pool's contents, written and read the reference's way.

    Outliers are kept densely per slot (``outm`` / ``outv``: (H, NB, S, D) per
    layer and K|V, allocated on first write), which is the reference's own
    storage (compact_pool.py:426-432); ``outlier_entries`` / ``outlier_array``
    list them in the build's sparse form for comparison.
    """

    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_size, scales):
        self.L, self.NB, self.S = num_layers, num_blocks, block_size
        self.H, self.D = num_kv_heads, head_size
        self.scales = list(scales)
        self.codes, self.stats = [], []
        self.outm = [[None, None] for _ in self.scales]
        self.outv = [[None, None] for _ in self.scales]
        for sc in self.scales:
            self.codes.append((np.zeros((self.H, self.NB, self.S, self.D * sc.bits_k // 8), np.uint8),
                               np.zeros((self.H, self.NB, self.S, self.D * sc.bits_v // 8), np.uint8)))
            st = np.empty((self.H, self.NB, 2, self.D), np.float16)
            st[:, :, 0] = np.float16(np.inf)
            st[:, :, 1] = np.float16(-np.inf)
            self.stats.append(st)

    def _outliers(self, layer, kv):
        if self.outm[layer][kv] is None:
            shape = (self.H, self.NB, self.S, self.D)
            self.outm[layer][kv] = np.zeros(shape, bool)
            self.outv[layer][kv] = np.zeros(shape, np.float16)
        return self.outm[layer][kv], self.outv[layer][kv]

    # -- write side (compact_pool.py:447-489) --
    def write_kv(self, layer, key, value, slot_mapping, abs_positions):
        """Tokens are written in input order: a slot written twice keeps the
        later token, and its outlier row is replaced, as the dense store does."""
        sc = self.scales[layer]
        key = np.asarray(key, np.float16)
        value = np.asarray(value, np.float16)
        slots = np.asarray(slot_mapping, np.int64)
        pos = np.asarray(abs_positions, np.int64)
        keep = slots >= 0
        if not keep.any():
            return
        key, value, slots, pos = key[keep], value[keep], slots[keep], pos[keep]
        kc, km, krec = quantize_k_rows(key, sc)
        vc, vm = quantize_v_rows(value, pos, sc)
        kp = pack_codes(kc, sc.bits_k)
        vp = pack_codes(vc, sc.bits_v)
        pages, t = slots // self.S, slots % self.S
        codes, stats = self.codes[layer], self.stats[layer]
        # numpy assigns repeated indices in order, so the last token of a slot wins
        codes[0][:, pages, t] = kp.transpose(1, 0, 2)
        codes[1][:, pages, t] = vp.transpose(1, 0, 2)
        for h in range(self.H):
            np.minimum.at(stats[h, :, 0], pages, krec[:, h])
            np.maximum.at(stats[h, :, 1], pages, krec[:, h])
        for kv, (m, x) in enumerate(((km, key), (vm, value))):
            om, ov = self._outliers(layer, kv)
            om[:, pages, t] = m.transpose(1, 0, 2)
            ov[:, pages, t] = np.where(m, x, np.float16(0)).transpose(1, 0, 2)

    # -- canonical outlier listing, the form parity tests compare --
    def outlier_entries(self, layer, h, page, kv):
        """Sorted (slot, d, fp16 bits) tuples of one page segment."""
        if self.outm[layer][kv] is None:
            return []
        m = self.outm[layer][kv][h, page]
        s, d = np.nonzero(m)
        bits = self.outv[layer][kv][h, page][s, d].view(np.uint16)
        return sorted(zip(s.tolist(), d.tolist(), bits.tolist()))

    def outlier_array(self, layer):
        """Every outlier as rows (h, page, kv, slot, d, fp16 bits), sorted."""
        parts = []
        for kv in range(2):
            if self.outm[layer][kv] is None:
                continue
            h, b, s, d = np.nonzero(self.outm[layer][kv])
            bits = self.outv[layer][kv][h, b, s, d].view(np.uint16).astype(np.int64)
            parts.append(np.stack([h, b, np.full_like(h, kv), s, d, bits], axis=1))
        if not parts:
            return np.zeros((0, 6), np.int64)
        a = np.concatenate(parts).astype(np.int64)
        return a[np.lexsort(a.T[::-1])]

    # -- dequantise (compact_pool.py:293-395) --
    def dequant_pages(self, layer, pages, first_pos):
        """(K, V) fp16 (H, P, S, D) of pool pages ``pages`` whose slot 0 sits
        at absolute position ``first_pos`` (V tail clamp, compact_pool.py:370-372)."""
        sc = self.scales[layer]
        pages = np.asarray(pages, np.int64)
        first_pos = np.asarray(first_pos, np.int64)
        kc = unpack_codes(self.codes[layer][0][:, pages], sc.bits_k)                # (H, P, S, D)
        vc = unpack_codes(self.codes[layer][1][:, pages], sc.bits_v)
        k = np.take_along_axis(sc.k_poles[:, None, None, :, :], kc[..., None].astype(np.intp), axis=-1)[..., 0]
        p = np.minimum(first_pos[:, None] + np.arange(self.S)[None], sc.t_cal - 1)  # (P, S)
        vpol = sc.v_poles[:, p]                                                    # (H, P, S, L)
        v = np.take_along_axis(vpol[:, :, :, None, :], vc[..., None].astype(np.intp), axis=-1)[..., 0]
        k, v = k.astype(np.float16), v.astype(np.float16)
        for kv, arr in ((0, k), (1, v)):
            if self.outm[layer][kv] is not None:
                m = self.outm[layer][kv][:, pages]
                arr[m] = self.outv[layer][kv][:, pages][m]
        return k, v

    def dequant_page(self, layer, h, page, first_pos):
        """(K, V) fp16 arrays (S, D) of one page for head h."""
        k, v = self.dequant_pages(layer, [page], [first_pos])
        return k[h, 0], v[h, 0]

    def unpack_to_staging(self, layer, block_ids, first_pos):
        """(NK, S, H, D) fp16 staging for K and V (compact_pool.py:492-537)."""
        k, v = self.dequant_pages(layer, block_ids, first_pos)
        return k.transpose(1, 2, 0, 3).copy(), v.transpose(1, 2, 0, 3).copy()

    def dequant_sequence(self, layer, block_table, n_tokens, page_offset=0, v_pos="logical", chunk=1024):
        """Dequantised (n_tokens, H, D) K and V of one sequence.

        Logical page j lives in pool page ``block_table[j]`` and starts at
        absolute position ``(page_offset + j) * S``; with v_pos="physical" its
        V rows are those of ``(page_offset + block_table[j]) * S``, the
        reference's rule (a slot is its position: compact_backend.py:157-167,
        unpack from ``block_id * BS``: quest_selector.py:89,
        compact_pool.py:370-372).
        """
        n_pages = -(-n_tokens // self.S)
        bt = np.asarray(block_table, np.int64)[:n_pages]
        first = (bt if v_pos == "physical" else np.arange(n_pages)) + page_offset
        K = np.zeros((n_pages * self.S, self.H, self.D), np.float16)
        V = np.zeros_like(K)
        for a in range(0, n_pages, chunk):
            b = min(a + chunk, n_pages)
            k, v = self.dequant_pages(layer, bt[a:b], first[a:b] * self.S)
            K[a * self.S:b * self.S] = k.transpose(1, 2, 0, 3).reshape(-1, self.H, self.D)
            V[a * self.S:b * self.S] = v.transpose(1, 2, 0, 3).reshape(-1, self.H, self.D)
        return K[:n_tokens], V[:n_tokens]


def dequant_packed_pages(k_rows, v_rows, dir_h, arena, pages, first_pos, k_poles_h, v_poles_h, bits_k, bits_v):
    """Decode pages of one head straight from the packed pool format.

    ``k_rows`` / ``v_rows`` (NB, S, RB) uint8 code rows of head h, ``dir_h``
    (NB, 2, 4) directory records {offset, capacity, count, rows}, ``arena``
    the layer's entries (fp16 value | channel << 16 | slot << 24), ``pages``
    the pool pages to decode with the absolute position of their slot 0 in
    ``first_pos``; poles of head h: K (D, Lk), V (t_cal, Lv). Returns K, V
    (m, S, D) fp16 (compact_pool.py:293-395, V rows clamped at t_cal - 1).
    """
    pages = np.asarray(pages, np.int64)
    first_pos = np.asarray(first_pos, np.int64)
    kc = unpack_codes(k_rows[pages], bits_k).astype(np.intp)                     # (m, S, D)
    vc = unpack_codes(v_rows[pages], bits_v).astype(np.intp)
    m, S, D = kc.shape
    K = np.take_along_axis(np.asarray(k_poles_h)[None, None], kc[..., None], axis=-1)[..., 0]
    t_cal = v_poles_h.shape[0]
    pos = np.minimum(first_pos[:, None] + np.arange(S)[None], t_cal - 1)         # (m, S)
    V = np.take_along_axis(np.asarray(v_poles_h)[pos][:, :, None, :], vc[..., None], axis=-1)[..., 0]
    K, V = K.astype(np.float16), V.astype(np.float16)
    arena = np.asarray(arena).astype(np.int64) & 0xFFFFFFFF
    for kv, arr in ((0, K), (1, V)):
        rec = np.asarray(dir_h)[pages, kv].astype(np.int64)                      # (m, 4)
        off, cnt = rec[:, 0], rec[:, 2]
        tot = int(cnt.sum())
        if tot == 0:
            continue
        which = np.repeat(np.arange(m), cnt)
        start = np.repeat(np.cumsum(cnt) - cnt, cnt)
        e = arena[np.repeat(off, cnt) + np.arange(tot) - start]
        slot, ch = (e >> 24) & 31, (e >> 16) & 255
        arr[which, slot, ch] = (e & 0xFFFF).astype(np.uint16).view(np.float16)
    return K, V
