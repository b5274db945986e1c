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
    """K rows x (N, H, D) fp16 -> codes (N, H, D), mask, recon fp16."""
    codes = nearest_codes(x, sc.k_poles[None])
    mask = band_outliers(x, sc.k_upper[None], sc.k_lower[None])
    pole = np.take_along_axis(np.broadcast_to(sc.k_poles[None], x.shape + (sc.k_poles.shape[-1],)),
                              codes[..., None].astype(np.int64), axis=-1)[..., 0]
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
    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_size, scales):
        self.L, self.NB, self.S = num_layers, num_blocks, block_size
        self.H, self.D = num_kv_heads, head_size
        self.scales = list(scales)
        self.codes, self.stats, self.rows = [], [], []
        for sc in self.scales:
            self.codes.append((np.zeros((self.H, self.NB, self.S, self.D * sc.bits_k // 8), np.uint8),
                               np.zeros((self.H, self.NB, self.S, self.D * sc.bits_v // 8), np.uint8)))
            st = np.empty((self.H, self.NB, 2, self.D), np.float16)
            st[:, :, 0] = np.float16(np.inf)
            st[:, :, 1] = np.float16(-np.inf)
            self.stats.append(st)
            # rows[(h, page, kv, slot)] = (d_idx uint8 array, values fp16 array)
            self.rows.append({})

    # -- write side (compact_pool.py:447-489) --
    def write_kv(self, layer, key, value, slot_mapping, abs_positions):
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
        codes, stats, rows = self.codes[layer], self.stats[layer], self.rows[layer]
        for i in range(slots.shape[0]):
            pg, s = pages[i], t[i]
            for h in range(self.H):
                codes[0][h, pg, s] = kp[i, h]
                codes[1][h, pg, s] = vp[i, h]
                stats[h, pg, 0] = np.minimum(stats[h, pg, 0], krec[i, h])
                stats[h, pg, 1] = np.maximum(stats[h, pg, 1], krec[i, h])
                for kv, (m, x) in enumerate(((km, key), (vm, value))):
                    d = np.nonzero(m[i, h])[0].astype(np.uint8)
                    rows[(h, int(pg), kv, int(s))] = (d, x[i, h, d].astype(np.float16))

    # -- canonical outlier listing, the form parity tests compare --
    def outlier_entries(self, layer, h, page, kv):
        """Sorted (slot, d, fp16 bits) tuples of one page segment."""
        out = []
        for (hh, pg, k, s), (d, v) in self.rows[layer].items():
            if hh == h and pg == page and k == kv:
                bits = v.view(np.uint16)
                out.extend((s, int(dd), int(bb)) for dd, bb in zip(d, bits))
        return sorted(out)

    # -- dequantise (compact_pool.py:293-395) --
    def dequant_page(self, layer, h, page, first_pos):
        """(K, V) fp16 arrays (S, D) of one page for head h.

        ``first_pos`` is the absolute position of slot 0 (V tail clamp,
        compact_pool.py:370-372).
        """
        sc = self.scales[layer]
        kc = unpack_codes(self.codes[layer][0][h, page], sc.bits_k).astype(np.int64)   # (S, D)
        vc = unpack_codes(self.codes[layer][1][h, page], sc.bits_v).astype(np.int64)
        k = np.take_along_axis(np.broadcast_to(sc.k_poles[h][None], (self.S, self.D, sc.k_poles.shape[-1])),
                               kc[..., None], axis=-1)[..., 0].astype(np.float16)
        p = np.minimum(first_pos + np.arange(self.S), sc.t_cal - 1)
        vpol = sc.v_poles[h, p]                                                     # (S, L)
        v = np.take_along_axis(vpol[:, None, :].repeat(self.D, 1), vc[..., None], axis=-1)[..., 0]
        v = v.astype(np.float16)
        for s in range(self.S):
            for kv, arr in ((0, k), (1, v)):
                r = self.rows[layer].get((h, int(page), kv, s))
                if r is not None and r[0].size:
                    arr[s, r[0].astype(np.int64)] = r[1]
        return k, v

    def unpack_to_staging(self, layer, block_ids, first_pos):
        """(NK, S, H, D) fp16 staging for K and V (compact_pool.py:492-537)."""
        nk = len(block_ids)
        sk = np.zeros((nk, self.S, self.H, self.D), np.float16)
        sv = np.zeros_like(sk)
        for i, (b, fp) in enumerate(zip(block_ids, first_pos)):
            for h in range(self.H):
                k, v = self.dequant_page(layer, h, int(b), int(fp))
                sk[i, :, h] = k
                sv[i, :, h] = v
        return sk, sv

    def dequant_sequence(self, layer, block_table, n_tokens, page_offset=0, v_pos="logical"):
        """Dequantised (n_tokens, H, D) K and V of one sequence.

        Logical page j lives in pool page ``block_table[j]`` and starts at
        absolute position ``(page_offset + j) * S``; with v_pos="physical" its
        V rows are those of ``(page_offset + block_table[j]) * S``, the
        reference's rule (a slot is its position: compact_backend.py:157-167,
        unpack from ``block_id * BS``: quest_selector.py:89,
        compact_pool.py:370-372).
        """
        n_pages = -(-n_tokens // self.S)
        K = np.zeros((n_pages * self.S, self.H, self.D), np.float16)
        V = np.zeros_like(K)
        for j in range(n_pages):
            for h in range(self.H):
                first = int(block_table[j]) if v_pos == "physical" else j
                k, v = self.dequant_page(layer, h, int(block_table[j]), (page_offset + first) * self.S)
                K[j * self.S:(j + 1) * self.S, h] = k
                V[j * self.S:(j + 1) * self.S, h] = v
        return K[:n_tokens], V[:n_tokens]
