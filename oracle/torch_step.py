"""The reference's own torch path for one layer, on the host CPU.

TEST INFRASTRUCTURE ONLY: ``bench.py`` times this as its CPU baseline (the
``cpu_baseline`` field and the ``--impl reference`` arm). It restates, in
torch on every host core and with no per-page Python loop, what the reference
computes for the path (xFuzzitx/helix-lite):

write (pack-on-write, ``CompactKVPool.write_kv``, src/kvquant/compact_pool.py:447-489)
  * outliers: the band test ``x > upper | x < lower`` (nuq.py:72;
    compact_pool.py:254-256), K per channel, V per token at row
    ``min(pos, t_cal - 1)`` (compact_pool.py:190-201, :467);
  * codes: ``argmin |x - pole|`` over the levels in fp32 (round_to_nearest_pole,
    nuq.py:22-38, as the pool's Triton kernels evaluate it,
    compact_pool.py:258-268);
  * storage: the reference pool's dense layout, one uint8 code, one fp16
    outlier value and one mask byte per element (compact_pool.py:426-432);
  * K page stats: fp32 running min / max of the reconstruction
    ``where(outlier, x, pole)`` (compact_pool.py:270, :285-287).

decode (``KVQuantCompactImpl.forward`` with Quest, src/kvquant/compact_backend.py:225-299)
  * ``page_upper_bound`` (src/quest/reference.py:59-93) with the GQA group
    terms Qp = sum_g max(q_g, 0), Qn = sum_g min(q_g, 0) of each KV head's
    query group (the sum of the group's per-head bounds);
  * ``topk_pages_with_sinks`` (reference.py:96-133): sinks masked to -inf,
    ``torch.topk``, sinks prepended, indices sorted;
  * dequantisation of the selected pages (``dequantize_nuq`` nuq.py:135-156,
    ``unpack_to_staging`` compact_pool.py:492-537, V rows clamped at t_cal);
  * ``selected_attention`` (reference.py:136-168) generalised to grouped
    queries, fp32 scores and softmax, scale 1/sqrt(D).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class RefLayer:
    """One layer of the reference pool (dense layout) plus its scales."""
    k_codes: torch.Tensor   # (T, H, D) uint8
    k_outv: torch.Tensor    # (T, H, D) fp16, 0 where not an outlier
    k_outm: torch.Tensor    # (T, H, D) bool
    v_codes: torch.Tensor
    v_outv: torch.Tensor
    v_outm: torch.Tensor
    k_min: torch.Tensor     # (P, H, D) fp32
    k_max: torch.Tensor
    k_poles: torch.Tensor   # (H, D, Lk) fp32
    v_poles: torch.Tensor   # (H, t_cal, Lv) fp32
    page: int

    @property
    def tokens(self) -> int:
        return self.k_codes.shape[0]

    def dense_bytes(self) -> int:
        """Bytes of the reference's storage of this layer (codes, outlier values, masks, fp32 stats)."""
        n = self.k_codes.numel() + self.v_codes.numel()
        return n * (1 + 2 + 1) + 2 * self.k_min.numel() * 4


def _nearest(x: torch.Tensor, poles: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 |x - pole| argmin (first level on ties) and the chosen pole."""
    diff = (x.unsqueeze(-1) - poles).abs()
    idx = diff.argmin(dim=-1, keepdim=True)
    return idx.squeeze(-1).to(torch.uint8), torch.gather(poles.expand_as(diff), -1, idx).squeeze(-1)


def write_layer(K: torch.Tensor, V: torch.Tensor, pos: torch.Tensor, k_poles, k_upper, k_lower, v_poles,
                v_upper, v_lower, page: int = 16, chunk: int = 8192) -> RefLayer:
    """Quantise one layer's K, V (T, H, D) at absolute positions ``pos`` into
    the reference's dense pool layout; T a multiple of ``page`` (slot t = t)."""
    T, H, D = K.shape
    kp, ku, kl = k_poles.float(), k_upper.float(), k_lower.float()
    vp, vu, vl = v_poles.float(), v_upper.float(), v_lower.float()
    t_cal = vp.shape[1]
    out = {n: torch.empty((T, H, D), dtype=dt) for n, dt in
           (("k_codes", torch.uint8), ("k_outv", torch.float16), ("k_outm", torch.bool),
            ("v_codes", torch.uint8), ("v_outv", torch.float16), ("v_outm", torch.bool))}
    P = T // page
    k_min = torch.empty((P, H, D), dtype=torch.float32)
    k_max = torch.empty((P, H, D), dtype=torch.float32)
    hidx = torch.arange(H).unsqueeze(0)
    for a in range(0, T, chunk):
        b = min(a + chunk, T)
        x = K[a:b].float()
        m = (x > ku) | (x < kl)
        c, pole = _nearest(x, kp)
        rec = torch.where(m, x, pole)
        out["k_codes"][a:b], out["k_outm"][a:b] = c, m
        out["k_outv"][a:b] = torch.where(m, x, torch.zeros_like(x)).half()
        r = rec.view(-1, page, H, D)
        k_min[a // page:b // page] = r.amin(dim=1)
        k_max[a // page:b // page] = r.amax(dim=1)
        rows = pos[a:b].clamp(min=0, max=t_cal - 1)
        x = V[a:b].float()
        up = vu[hidx, rows.unsqueeze(1)].unsqueeze(-1)          # (n, H, 1)
        lo = vl[hidx, rows.unsqueeze(1)].unsqueeze(-1)
        m = (x > up) | (x < lo)
        c, _ = _nearest(x, vp[hidx, rows.unsqueeze(1)].unsqueeze(2))   # poles (n, H, 1, L)
        out["v_codes"][a:b], out["v_outm"][a:b] = c, m
        out["v_outv"][a:b] = torch.where(m, x, torch.zeros_like(x)).half()
    return RefLayer(**out, k_min=k_min, k_max=k_max, k_poles=kp, v_poles=vp, page=page)


def topk_pages_with_sinks(bound: torch.Tensor, k: int, sink_pages: int) -> torch.Tensor:
    """reference.py:96-133: (P, H) bounds -> (sinks + k_eff, H) sorted page indices."""
    P, H = bound.shape
    sink_pages = max(0, min(sink_pages, P))
    k_eff = max(0, min(k, P - sink_pages))
    sink_idx = torch.arange(sink_pages).unsqueeze(1).expand(-1, H)
    if k_eff == 0:
        return sink_idx
    masked = bound.clone()
    masked[:sink_pages] = float("-inf")
    top = torch.topk(masked, k=k_eff, dim=0)
    return torch.cat([sink_idx, top.indices], dim=0).sort(dim=0).values


def decode_layer(layer: RefLayer, q: torch.Tensor, k_pages: int, sink_pages: int = 4, chunk: int = 65536):
    """One decode token: q (Hq, D). Returns (o (Hq, D) fp32, selected (k, H))."""
    P, H, D = layer.k_min.shape
    Hq = q.shape[0]
    G = Hq // H
    S = layer.page
    qf = q.float().view(H, G, D)
    qp, qn = qf.clamp(min=0).sum(1), qf.clamp(max=0).sum(1)                       # (H, D)
    bound = (qp.unsqueeze(0) * layer.k_max).sum(-1) + (qn.unsqueeze(0) * layer.k_min).sum(-1)
    sel = topk_pages_with_sinks(bound, k_pages, sink_pages)                        # (k, H)
    t_cal = layer.v_poles.shape[1]
    scale = 1.0 / math.sqrt(D)
    o = torch.empty((H, G, D), dtype=torch.float32)
    for h in range(H):   # each KV head attends its own selection (reference.py:157-167)
        tok = (sel[:, h].unsqueeze(1) * S + torch.arange(S)).reshape(-1)         # (N,)
        kpol = layer.k_poles[h]                                                    # (D, Lk)
        scores, vals = [], []
        for a in range(0, tok.numel(), chunk):
            t = tok[a:a + chunk]
            kc = layer.k_codes[t, h].long()                                        # (n, D)
            Kd = torch.gather(kpol.expand(t.numel(), -1, -1), -1, kc.unsqueeze(-1)).squeeze(-1)
            Kd = torch.where(layer.k_outm[t, h], layer.k_outv[t, h].float(), Kd)
            scores.append(qf[h] @ Kd.t() * scale)                                   # (G, n)
            vrow = layer.v_poles[h, t.clamp(max=t_cal - 1)]                         # (n, Lv)
            vc = layer.v_codes[t, h].long()
            Vd = torch.gather(vrow.unsqueeze(1).expand(-1, D, -1), -1, vc.unsqueeze(-1)).squeeze(-1)
            vals.append(torch.where(layer.v_outm[t, h], layer.v_outv[t, h].float(), Vd))
        p = torch.softmax(torch.cat(scores, dim=1), dim=1)                          # (G, N)
        o[h] = p @ torch.cat(vals, dim=0)
    return o.view(Hq, D), sel


def decode_bytes(layer: RefLayer, sel: torch.Tensor, Hq: int) -> int:
    """Bytes this path reads for one decode of the layer in the reference
    layout: fp32 stats of every page, and code + outlier value + mask (4 B)
    per element of the selected pages, V rows of selected tokens below t_cal
    (fp32 poles), q and o."""
    P, H, D = layer.k_min.shape
    S = layer.page
    n_sel = sel.numel()
    t_cal = layer.v_poles.shape[1]
    vrows = int(((sel * S) < t_cal).sum()) * S
    return (2 * layer.k_min.numel() * 4 + n_sel * S * D * 2 * 4 + vrows * layer.v_poles.shape[-1] * 4
            + Hq * D * (2 + 4))
