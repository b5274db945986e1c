#!/usr/bin/env python
"""Benchmark of the long-context KV hot path (headline).

One step = a full 28-layer decode step at 1M context served from the compact
pool: per layer, Quest page scores over every page (fp16 K min / max), the
exact top-25% + 4 sinks threshold, and the fused-dequant split-KV decode
(layers 0-15 nuq2 with 5% outliers, 16-27 nuq4 with 1%); 4 KV / 28 query
heads, head_dim 128, 16-token pages. With N ranks the sequence's pages are
split N ways (split-KV): each rank selects and attends its shard and one
NCCL all-gather of (o, lse) per layer feeds the merge.

  value     effective KV GB/s: algorithmic bytes of the step (stats scanned +
            selected code segments + their outlier entries and directory
            records + V level rows + q / o) / device step time, all ranks;
            the step replays as a CUDA graph with inputs resident in HBM
  e2e       the same bytes / wall time per step with the 28 queries copied
            from pinned host memory into the step's input buffer and the
            outputs read back to host every step (the captured step)
  parity    once, outside the timed region: two layers' selections against
            the oracle (bit-exact) and their decode outputs against float64
            dequantise-then-attend (within 2e-3)
  configs   at N = 1, BASELINE configs 1-4 measured each with its own
            roofline (pack, Quest at 128K, decode at 128K, batched append +
            decode)
  cpu_baseline  the reference's torch path (oracle/torch_step.py) on all host
            cores: two whole layers of the same workload at full context

``--impl reference`` times that torch path alone (rank 0; the other ranks exit).

Usage: python bench.py [--gpus N --steps K --warmup W --impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "helix-lite_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-step µs & effective KV GB/s (vs HBM peak) @128K/1M ctx; pack GB/s"
H, G, D, S = 4, 7, 128, 16
TOL = 2e-3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ctx", type=int, default=1 << 20, help="context tokens (multiple of 16)")
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--cut", type=int, default=16, help="layers below cut are nuq2")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1-4 measurements")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="split-KV exchange: peer-memory merge kernel, or NCCL all-gather + merge")
    ap.add_argument("--profile", action="store_true", help="setup + warmup + steps only (for ncu)")
    ap.add_argument("--no-fused-select", action="store_true",
                    help="keep the threshold kernel between scores and decode for small shards too")
    ap.add_argument("--splits", type=int, default=0,
                    help="decode splits per (sequence, KV head); 0 = about one CTA per SM")
    ap.add_argument("--decode-cores", choices=["tensor", "cuda"], default="tensor",
                    help="decode QK / PV on the tensor cores (mma.sync) or as FFMA on the CUDA cores (comparison)")
    ap.add_argument("--select", choices=["shard", "global"], default="shard",
                    help="N > 1: top-K per shard (the default), or the single-GPU top-K over every shard's pages")
    return ap.parse_args()


def workload(args, world):
    """The workload both arms run (identical dicts)."""
    return {"workload": f"config5: {args.layers}-layer mixed nuq2/nuq4 decode step at {args.ctx} ctx, "
                        f"Quest 25%+4 sinks, split-KV over {world} GPU(s)",
            "context_tokens": args.ctx, "layers": args.layers, "nuq2_layers": min(args.cut, args.layers),
            "kv_heads": H, "q_heads": H * G, "head_dim": D, "page": S, "batch": 1,
            "l2": "inputs larger than L2 (stats + selected codes per step >> 126 MB)"}


def read_traffic(kernel):
    """dram bytes per launch of `kernel` from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) == 2 and parts[0] == kernel and not line.startswith("#"):
            return int(parts[1])
    return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def roofline(bytes_, ms, peak, src, kernel, traffic=None):
    ach = bytes_ / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": kernel, "achieved": round(ach, 1), "peak": peak, "peak_source": src,
            "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": traffic,
            "algorithmic_bytes_per_launch": int(bytes_), "avg_launch_ms": round(ms, 5)}


def step_layer_bytes(n_pages, sel_pages, entries, vrows, seg, levels_v, hq=H * G):
    """Algorithmic bytes of one layer of the decode step (both arms):
    scores: every page-head's fp16 {min, max} (512 B) read, its fp32 score
    written; threshold: the scores read; decode: per selected page-head its
    code segment, two 16-byte directory records and 4 B per outlier entry,
    per-token V level rows below t_cal, the scores scanned; q in, o / lse out."""
    stats = n_pages * H * (2 * D * 2 + 4)
    thr = n_pages * H * 4
    dec = sel_pages * (seg + 32) + 4 * entries + vrows * S * levels_v * 2 + n_pages * H * 4
    qo = hq * D * 2 + hq * (D + 1) * 4
    return {"stats": stats, "threshold": thr, "decode": dec + qo}


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML reads only)

class ClockSampler:
    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            pr = torch.cuda.get_device_properties(index)
            try:
                bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass

    def _run(self):
        nv = self.nv
        bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
                r = fn(self.h)
                for name, bit in bits.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.05)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# the synthetic workload (seeded; both arms build the same tensors)

def layer_seed(layer):
    return 1234 + 1000 * layer


CHUNK = 1 << 16


def layer_scales_all(args, device):
    from kvquant.synthetic import make_scales, mixed_layout
    layout = mixed_layout(args.layers, args.cut)
    return layout, make_scales(layout, H, D, t_cal=4096, seed=1234, device=device, calib_tokens=4096)


def layer_chunk(li, lay, c, device, cs):
    """K, V of global tokens [c * CHUNK, (c + 1) * CHUNK) of layer li."""
    from kvquant.synthetic import make_kv
    return make_kv(CHUNK, H, D, seed=layer_seed(li) + 7 * c + 1, outlier_frac=lay[1], device=device, chan_scale=cs)


def queries(args, device):
    import torch
    g = torch.Generator(device=device).manual_seed(99)
    return torch.randn((args.layers, 1, H * G, D), generator=g, device=device).to(torch.float16)


def build_world(args, rank, world, device):
    import torch
    from kvquant import fused
    from kvquant.compact_pool import CompactKVPool
    from kvquant.splitkv import local_k, shard_plan
    from kvquant.synthetic import NUQ2, channel_scales

    n_pages = args.ctx // S
    shard = shard_plan(n_pages, world, rank)
    layout, scales = layer_scales_all(args, device)
    fracs = [0.10 if lay is NUQ2 else 0.03 for lay in layout]
    pool = CompactKVPool(args.layers, shard.n_pages, S, H, D, scales, device=device, outlier_frac=fracs)

    # fill: global chunks of 64K tokens so a token's data does not depend on N
    t0g, t1g = shard.page_begin * S, (shard.page_begin + shard.n_pages) * S
    pack_ms, pack_tokens = 0.0, 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for li, lay in enumerate(layout):
        cs = channel_scales(H, D, layer_seed(li), device)
        for c in range(t0g // CHUNK, (t1g + CHUNK - 1) // CHUNK):
            a, b = max(c * CHUNK, t0g), min((c + 1) * CHUNK, t1g)
            K, V = layer_chunk(li, lay, c, device, cs)
            K, V = K[a - c * CHUNK:b - c * CHUNK].contiguous(), V[a - c * CHUNK:b - c * CHUNK].contiguous()
            pos = torch.arange(a, b, device=device)
            ev0.record()
            pool.write_kv(li, K, V, pos - t0g, pos)
            ev1.record()
            ev1.synchronize()
            pack_ms += ev0.elapsed_time(ev1)
            pack_tokens += b - a
    pool.check()

    qs = queries(args, device)
    bt = torch.arange(shard.n_pages, dtype=torch.int32, device=device).unsqueeze(0)
    sl = torch.tensor([shard.n_pages * S], dtype=torch.int32, device=device)
    kk = local_k(shard)
    ns = args.splits if args.splits > 0 else fused.default_splits(1, H, shard.n_pages)
    gsel = None
    if args.select == "global" and world > 1:
        from kvquant.splitkv import GlobalSelect
        if n_pages % world:
            raise SystemExit("--select global needs the pages split evenly over the GPUs")
        gsel = GlobalSelect(1, H, shard.n_pages, world, device, sink_pages=4, top_frac=(1, 4))
        gsel.set_lengths(torch.tensor([args.ctx], dtype=torch.int32))

    # algorithmic bytes: selection is fixed per layer (fixed queries)
    per_layer = []
    for li in range(args.layers):
        if gsel is not None:
            sel = gsel.select(pool, li, qs[li], bt, sl, shard)
        else:
            sel = fused.quest_select(pool, li, qs[li], bt, sl, top_k=kk, sink_pages=shard.sink_pages)
        lists, counts = fused.selected_lists(sel)
        lay = pool.layers[li]
        dirc = lay.dir[:, :, :, 2].to(torch.int64)                 # (H, NB, 2)
        ent = npages = vrows = 0
        for h in range(H):
            c = int(counts[0, h])
            pg = lists[0, h, :c].long()
            npages += c
            ent += int(dirc[h, pg].sum())
            vrows += int(((shard.page_begin + pg) * S < 4096).sum())
        levels_v = int(scales.per_layer_values[li].poles.shape[-1])
        b = step_layer_bytes(shard.n_pages, npages, ent, vrows, lay.seg, levels_v)
        b.update(pages=npages, entries=ent)
        per_layer.append(b)
    pack_bytes = 0
    for li in range(args.layers):
        lay = pool.layers[li]
        pack_bytes += shard.n_pages * S * H * D * 2 * 2                  # fp16 K, V read
        pack_bytes += shard.n_pages * H * lay.seg                        # codes written
        pack_bytes += shard.n_pages * H * 2 * D * 2 * 2                  # stats read + written
        pack_bytes += 4 * int(lay.dir[:, :, :, 2].to(torch.int64).sum())  # outlier entries written
    return dict(pool=pool, shard=shard, qs=qs, bt=bt, sl=sl, k=kk, ns=ns, per_layer=per_layer, gsel=gsel,
                cores=args.decode_cores, fused_select=not args.no_fused_select,
                pack=dict(ms=pack_ms, tokens=pack_tokens, bytes=pack_bytes), scales=scales, layout=layout)


def make_step(W, world, group, timing=None):
    """The decode step over all layers; `timing` records events around each kernel group."""
    import torch
    import hxlib
    from kvquant import fused
    from kvquant.splitkv import Exchange

    pool, qs, bt, sl, shard = W["pool"], W["qs"], W["bt"], W["sl"], W["shard"]
    L = qs.shape[0]
    dev = pool.device
    scores = [torch.empty((1, H, shard.n_pages), dtype=torch.float32, device=dev) for _ in range(L)]
    thresh = [torch.empty((H,), dtype=torch.int64, device=dev) for _ in range(L)]
    nsl = int(hxlib.lib().hx_quest_slices(shard.n_pages))
    slices = [torch.empty((H, nsl + 1), dtype=torch.int32, device=dev) for _ in range(L)]
    o_loc = torch.empty((L, 1, H * G, D), dtype=torch.float32, device=dev)
    lse_loc = torch.empty((L, 1, H * G), dtype=torch.float32, device=dev)
    o_out = torch.empty((L, H * G, D), dtype=torch.float32, device=dev)
    pex = W.get("pex")
    ex = Exchange(H * G, D, world, dev, group) if world > 1 and pex is None else None

    # rows of at most FUSED_MAX_PAGES pages (N >= 4 at 1M): the decode's CTAs
    # find the threshold themselves, no threshold kernel between scores and decode
    fused_sel = W.get("gsel") is None and shard.n_pages <= fused.FUSED_MAX_PAGES and W.get("fused_select", True)
    hist = hxlib.scratch(dev, "quest_hist", H * 2 * 4096 * 4)

    def step(q_in=None):
        q_all = qs if q_in is None else q_in
        for li in range(L):
            if timing is not None:
                timing["ev"][li][0].record()
            if fused_sel:
                fused.page_scores(pool, li, q_all[li], bt, sl, shard.n_pages, shard.sink_pages, scores[li], hist)
                if timing is not None:
                    timing["ev"][li][1].record()
                if world == 1:
                    o_dst, lse_dst = o_out[li].view(1, H * G, D), lse_loc[li]
                elif pex is not None:
                    o_dst, lse_dst = pex.o_view(li).view(1, H * G, D), pex.lse_view(li).view(1, H * G)
                else:
                    o_dst, lse_dst = o_loc[li], lse_loc[li]
                fused.decode_select(pool, li, q_all[li], bt, sl, scores[li], top_k=W["k"],
                                    sink_pages=shard.sink_pages, page_begin=shard.page_begin, n_splits=W["ns"],
                                    o=o_dst, lse=lse_dst, cores=W.get("cores", "tensor"))
                if timing is not None:
                    timing["ev"][li][2].record()
                if world > 1:
                    if pex is not None:
                        pex.merge(li, o_out[li])
                    else:
                        ex.merge(o_loc[li].view(H * G, D), lse_loc[li].view(H * G), o_out[li])
                continue
            if W.get("gsel") is not None:
                sel = W["gsel"].select(pool, li, q_all[li], bt, sl, shard)
            else:
                sel = fused.quest_select(pool, li, q_all[li], bt, sl, top_k=W["k"], sink_pages=shard.sink_pages,
                                         scores=scores[li], thresh=thresh[li], slice_out=slices[li])
            if timing is not None:
                timing["ev"][li][1].record()
            # one GPU: the decode writes the layer's output in place; several:
            # its partials, into the exchange's row for the layer
            if world == 1:
                o_dst, lse_dst = o_out[li].view(1, H * G, D), lse_loc[li]
            elif pex is not None:
                o_dst, lse_dst = pex.o_view(li).view(1, H * G, D), pex.lse_view(li).view(1, H * G)
            else:
                o_dst, lse_dst = o_loc[li], lse_loc[li]
            fused.decode(pool, li, q_all[li], bt, sl, sel, page_begin=shard.page_begin, n_splits=W["ns"],
                         o=o_dst, lse=lse_dst, cores=W.get("cores", "tensor"))
            if timing is not None:
                timing["ev"][li][2].record()
            if world > 1:
                if pex is not None:
                    pex.merge(li, o_out[li])
                else:
                    ex.merge(o_loc[li].view(H * G, D), lse_loc[li].view(H * G), o_out[li])
        return o_out

    return step


# ---------------------------------------------------------------------------
# parity of the step (outside every timed region)

def check_parity(W, args, world, rank, group):
    """Two layers (the first nuq2 and the first nuq4 layer): each rank's
    selection against the oracle's pinned scores and top-K on its own pages
    (bit-exact), and the decode output against float64 dequantise-then-attend
    over the oracle's decode of the pool bytes (within 2e-3); with N > 1 each
    rank's exact partial (o, lse) is gathered and merged by the oracle, and the
    page recall of the sharded selection against one global top-K is given."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from kvquant import fused
    from oracle import attention as oatt
    from oracle import quest as oq
    from oracle.pool import dequant_packed_pages

    pool, shard, qs, bt, sl = W["pool"], W["shard"], W["qs"], W["bt"], W["sl"]
    n = shard.n_pages
    check_layers = sorted({0, min(args.cut, args.layers - 1)})
    sel_ok, errs, recall = True, [], []
    step = make_step(W, world, group)
    o_all = step().clone()
    torch.cuda.synchronize()
    gsel = W.get("gsel")
    for li in check_layers:
        if gsel is not None:
            sel = gsel.select(pool, li, qs[li], bt, sl, shard)
        else:
            sel = fused.quest_select(pool, li, qs[li], bt, sl, top_k=W["k"], sink_pages=shard.sink_pages)
        lists, counts = fused.selected_lists(sel)
        scores = sel.scores[0].cpu().numpy()                                   # (H, n)
        lay = pool.layers[li]
        stats = lay.stats.cpu().numpy()                                        # (H, n, 2, D)
        q = qs[li, 0].cpu().numpy()
        qp, qn = oq.group_terms(q, G, "sum")
        ref_scores = oq.page_scores(qp, qn, stats[:, :, 0].transpose(1, 0, 2), stats[:, :, 1].transpose(1, 0, 2))
        sel_ok &= bool(np.array_equal(ref_scores.T.view(np.uint32), scores.view(np.uint32)))
        full = None
        if world > 1:   # every rank's oracle scores, in global page order
            dev = pool.device
            sizes = torch.tensor([n], device=dev)
            all_n = [torch.empty_like(sizes) for _ in range(world)]
            dist.all_gather(all_n, sizes, group=group)
            nmax = max(int(x) for x in all_n)
            pad = torch.full((H, nmax), float("nan"), device=dev)
            pad[:, :n] = torch.from_numpy(np.ascontiguousarray(ref_scores.T)).to(dev)
            all_sc = [torch.empty_like(pad) for _ in range(world)]
            dist.all_gather(all_sc, pad, group=group)
            full = np.concatenate([all_sc[r][:, :int(all_n[r])].cpu().numpy() for r in range(world)], axis=1)

        def expected(h):
            if gsel is None:
                return oq.select_pages(ref_scores[:, h], W["k"], shard.sink_pages)
            g_sel = oq.select_pages(full[h], full.shape[1] // 4, 4)      # the one-GPU selection
            mine = g_sel[(g_sel >= shard.page_begin) & (g_sel < shard.page_begin + n)]
            return mine - shard.page_begin

        codes = lay.codes.cpu().numpy()
        rbk, rbv = D * lay.bits_k // 8, D * lay.bits_v // 8
        arena = lay.arena.cpu().numpy()
        dirs = lay.dir.cpu().numpy()
        sc = pool.scales
        kpol = sc.per_layer_keys[li].poles.half().cpu().numpy()
        vpol = sc.per_layer_values[li].poles.half().cpu().numpy()
        o_part = np.zeros((H * G, D))
        lse_part = np.full(H * G, -np.inf)
        for h in range(H):
            pages = expected(h)
            c = int(counts[0, h])
            sel_ok &= bool(np.array_equal(lists[0, h, :c].cpu().numpy(), pages))
            if len(pages) == 0:
                continue
            kr = codes[h, :, :S * rbk].reshape(n, S, rbk)
            vr = codes[h, :, S * rbk:].reshape(n, S, rbv)
            Kd, Vd = dequant_packed_pages(kr, vr, dirs[h], arena, pages, (shard.page_begin + pages) * S,
                                          kpol[h], vpol[h], lay.bits_k, lay.bits_v)
            Kt = np.zeros((Kd.shape[0] * S, H, D), np.float16)
            Vt = np.zeros_like(Kt)
            Kt[:, h], Vt[:, h] = Kd.reshape(-1, D), Vd.reshape(-1, D)
            qh = np.zeros((H * G, D))
            qh[h * G:(h + 1) * G] = q[h * G:(h + 1) * G]
            o, lse = oatt.decode_attention(qh, Kt, Vt)
            o_part[h * G:(h + 1) * G], lse_part[h * G:(h + 1) * G] = o[h * G:(h + 1) * G], lse[h * G:(h + 1) * G]
        if world > 1:
            dev = pool.device
            t = torch.from_numpy(np.concatenate([o_part.reshape(-1), lse_part])).to(dev)
            got = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(got, t, group=group)
            sel_t = torch.tensor([1 if sel_ok else 0], device=dev)
            dist.all_reduce(sel_t, op=dist.ReduceOp.MIN)
            sel_ok = bool(sel_t.item())
            if rank == 0:
                parts = [x.cpu().numpy() for x in got]
                O = np.stack([p[:H * G * D].reshape(H * G, D) for p in parts])
                L_ = np.stack([p[H * G * D:] for p in parts])
                ref_o, _ = oatt.merge_partials(O, L_)
                errs.append(float(np.abs(o_all[li].cpu().numpy() - ref_o).max()))
                nt = full.shape[1]
                from kvquant.splitkv import shard_plan
                hit = tot = 0
                for h in range(H):
                    glob = set(oq.select_pages(full[h], nt // 4, 4).tolist())
                    mine = set()
                    for r in range(world):
                        srd = shard_plan(nt, world, r)
                        if gsel is not None:
                            loc = np.asarray(sorted(p for p in glob if srd.page_begin <= p < srd.page_begin
                                                    + srd.n_pages), dtype=np.int64) - srd.page_begin
                        else:
                            loc = oq.select_pages(full[h, srd.page_begin:srd.page_begin + srd.n_pages],
                                                  srd.n_pages // 4, srd.sink_pages)
                        mine |= set((loc + srd.page_begin).tolist())
                    hit += len(glob & mine)
                    tot += len(glob)
                recall.append(hit / max(tot, 1))
        else:
            errs.append(float(np.abs(o_all[li].cpu().numpy() - o_part).max()))
    if rank != 0:
        return None
    how = ("the one-GPU top-K over every rank's pages (oracle scores gathered), each rank's part"
           if gsel is not None else "pinned scores + top-K on each rank's pages")
    res = {"layers": check_layers, "selection_bit_exact": sel_ok, "decode_max_abs_err": max(errs), "tol": TOL,
           "reference": "oracle: " + how + "; float64 attention over the oracle's decode of the pool bytes"
                        + ("; exact partials merged" if world > 1 else ""),
           "ok": bool(sel_ok and max(errs) < TOL)}
    if world > 1:
        res["page_recall_vs_global_topk"] = round(min(recall), 4)
    return res


# ---------------------------------------------------------------------------
# configs 1-4 (N = 1)

class Timer:
    """CUDA-event timing of one call per iteration, L2 flushed before each."""

    def __init__(self, device, flush_mb=512):
        import torch
        self.flush = torch.empty(flush_mb << 20, dtype=torch.uint8, device=device)

    def __call__(self, fn, warmup=3, iters=10):
        import torch
        times = []
        for i in range(warmup + iters):
            self.flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            if i >= warmup:
                times.append(e0.elapsed_time(e1))
        return statistics.median(times)


def measure_pack(device, peak, src, tokens=CHUNK):
    """The append as the step's pool sees it, warm: one nuq4 layer, `tokens`
    tokens (one 64K chunk) appended in one call to whole pages; L2 flushed
    before each call; median of 10 after 3 warm-up calls."""
    import torch
    from kvquant.compact_pool import CompactKVPool
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=700, device=device)
    npg = tokens // S
    pool = CompactKVPool(1, npg, S, H, D, sc, device=device, outlier_frac=0.03)
    K, V = make_kv(tokens, H, D, seed=701, outlier_frac=0.01, device=device, chan_seed=700)
    pos = torch.arange(tokens, device=device)
    ms = Timer(device)(lambda: pool.write_kv(0, K, V, pos, pos))
    pool.check()
    lay = pool.layers[0]
    ent = int(lay.dir[:, :, :, 2].to(torch.int64).sum())
    b = tokens * H * D * 2 * 2 + npg * H * lay.seg + 4 * ent + npg * H * 2 * D * 2 * 2 + 4096 * H * 16 * 2
    del pool, K, V
    torch.cuda.empty_cache()
    return {"value": round(b / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "tokens": tokens, "us": round(ms * 1e3, 1),
            "what": f"nuq4 append of {tokens} tokens in one call (hx_pack_append: run pre-pass + K and V kernels), "
                    "warm, L2 flushed before each call, median of 10",
            "roofline": roofline(b, ms, peak, src, "pack_kv_kernel<4,4> + pack_count_runs_kernel")}


def run_configs(device, peak, src):
    import torch
    from kvquant import fused
    from kvquant.compact_pool import CompactKVPool
    from kvquant.synthetic import NUQ4, make_kv, make_scales
    timer = Timer(device)
    out = {}

    # ---- config 1: nuq4 pack + unpack round trip, T = 4096
    T = 4096
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=0, device=device)
    K, V = make_kv(T, H, D, seed=0, outlier_frac=0.01, device=device)
    pool = CompactKVPool(1, T // S, S, H, D, sc, device=device, outlier_frac=0.05)
    slots = torch.arange(T, device=device)
    ids = torch.arange(T // S, device=device)
    sk = torch.empty((T // S, S, H, D), dtype=torch.float16, device=device)
    sv = torch.empty_like(sk)
    pool.write_kv(0, K, V, slots, slots)
    pack_ms = timer(lambda: pool.write_kv(0, K, V, slots, slots))
    unpack_ms = timer(lambda: pool.unpack_to_staging(0, ids, ids * S, sk, sv))
    pool.check()
    lay = pool.layers[0]
    ent = int(lay.dir[:, :, :, 2].to(torch.int64).sum())
    pages = T // S
    pack_b = T * H * D * 2 * 2 + pages * H * lay.seg + 4 * ent + pages * H * 2 * D * 2 * 2 + T * H * 16 * 2
    unpack_b = pages * H * (lay.seg + 32) + 4 * ent + 2 * T * H * D * 2 + T * H * 16 * 2
    out["config1_pack_roundtrip"] = {
        "what": "nuq4 quantise + bit-pack (hx_pack_append) and staging unpack (hx_unpack_pages), one layer, "
                "T=4096, H=4, D=128, 1% outliers x10; L2 flushed before each call",
        "pack_us": round(pack_ms * 1e3, 2), "pack_GBps": round(pack_b / (pack_ms * 1e-3) / 1e9, 1),
        "unpack_us": round(unpack_ms * 1e3, 2), "unpack_GBps": round(unpack_b / (unpack_ms * 1e-3) / 1e9, 1),
        "roundtrip_us": round((pack_ms + unpack_ms) * 1e3, 2),
        "roofline": roofline(pack_b, pack_ms, peak, src, "pack_kv_kernel<4,4> + pack_count_runs_kernel"),
        "note": "8 MB of input: one launch is latency-bound at this size (config 4 is the bandwidth case)"}
    del pool, K, V, sk, sv

    # ---- config 2: Quest top-K at 128K (8192 pages), stats of fp16 N(0,1) keys, GQA sum
    P = 8192
    sc = make_scales([NUQ4], H, D, t_cal=64, seed=2, device=device)
    pool = CompactKVPool(1, P, S, H, D, sc, device=device)
    g = torch.Generator(device=device).manual_seed(2)
    Kp = torch.randn((P, S, H, D), generator=g, device=device).to(torch.float16)
    st = pool.layers[0].stats
    st[:, :, 0] = Kp.amin(dim=1).permute(1, 0, 2)
    st[:, :, 1] = Kp.amax(dim=1).permute(1, 0, 2)
    del Kp
    g = torch.Generator(device=device).manual_seed(3)
    q = torch.randn((1, H * G, D), generator=g, device=device).to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device=device).unsqueeze(0)
    sl = torch.tensor([P * S], dtype=torch.int32, device=device)
    scores = torch.empty((1, H, P), dtype=torch.float32, device=device)
    thr = torch.empty((H,), dtype=torch.int64, device=device)
    nsl = int(__import__("hxlib").lib().hx_quest_slices(P))
    slc = torch.empty((H, nsl + 1), dtype=torch.int32, device=device)
    lo = (torch.empty((H, P), dtype=torch.int32, device=device), torch.empty((H,), dtype=torch.int32, device=device))

    def quest():
        fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, scores=scores, thresh=thr,
                           slice_out=slc, list_out=lo)
    q_ms = timer(quest)
    pool.check()
    qb = P * H * 2 * D * 2 + H * G * D * 2 + (P // 4 + 4) * H * 4
    out["config2_quest_128k"] = {
        "what": "Quest scores + exact top-25% threshold + sorted page lists, 8192 pages x 4 KV heads, "
                "28 query heads (GQA sum), k = 2048 + 4 sinks; L2 flushed before each call",
        "us": round(q_ms * 1e3, 2), "GBps": round(qb / (q_ms * 1e-3) / 1e9, 1),
        "roofline": roofline(qb, q_ms, peak, src, "quest_scores + threshold + lists")}
    del pool

    # ---- config 3: one nuq4 layer at 128K, fused decode dense and with Quest 25%
    T = 128 * 1024
    P = T // S
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=300, device=device)
    pool = CompactKVPool(1, P, S, H, D, sc, device=device, outlier_frac=0.03)
    for a in range(0, T, CHUNK):
        K, V = make_kv(CHUNK, H, D, seed=301 + a, outlier_frac=0.01, device=device, chan_seed=300)
        p = torch.arange(a, a + CHUNK, device=device)
        pool.write_kv(0, K, V, p, p)
    del K, V
    g = torch.Generator(device=device).manual_seed(302)
    q = torch.randn((1, H * G, D), generator=g, device=device).to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device=device).unsqueeze(0)
    sl = torch.tensor([T], dtype=torch.int32, device=device)
    o = torch.empty((1, H * G, D), dtype=torch.float32, device=device)
    lse = torch.empty((1, H * G), dtype=torch.float32, device=device)
    scores = torch.empty((1, H, P), dtype=torch.float32, device=device)
    nsl = int(__import__("hxlib").lib().hx_quest_slices(P))
    slc = torch.empty((H, nsl + 1), dtype=torch.int32, device=device)
    dense_ms = timer(lambda: fused.decode(pool, 0, q, bt, sl, o=o, lse=lse))

    def quest_decode():
        s_ = fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, scores=scores, thresh=thr,
                                slice_out=slc)
        fused.decode(pool, 0, q, bt, sl, s_, o=o, lse=lse)
    quest_ms = timer(quest_decode)
    pool.check()
    lay = pool.layers[0]
    dirc = lay.dir[:, :, :, 2].to(torch.int64)
    ent_all = int(dirc.sum())
    dense_b = P * H * (lay.seg + 32) + 4 * ent_all + 256 * H * S * 16 * 2 + H * G * D * 2 + H * G * (D + 1) * 4
    sel = fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, lists=True)
    lists, counts = fused.selected_lists(sel)
    npg = ent = vr = 0
    for h in range(H):
        c = int(counts[0, h])
        pg = lists[0, h, :c].long()
        npg += c
        ent += int(dirc[h, pg].sum())
        vr += int((pg * S < 4096).sum())
    qb = step_layer_bytes(P, npg, ent, vr, lay.seg, 16)
    quest_b = qb["stats"] + qb["threshold"] + qb["decode"]
    out["config3_decode_128k"] = {
        "what": "one nuq4 layer, batch 1, 128K context, 28 query / 4 KV heads; dense = fused decode over every "
                "page, quest = scores + threshold + fused decode over 25% + 4 sinks; L2 flushed before each call",
        "dense_us": round(dense_ms * 1e3, 2), "dense_GBps": round(dense_b / (dense_ms * 1e-3) / 1e9, 1),
        "quest_us": round(quest_ms * 1e3, 2), "quest_GBps": round(quest_b / (quest_ms * 1e-3) / 1e9, 1),
        "roofline": roofline(dense_b, dense_ms, peak, src, "decode_kernel<4,4> (dense)")}
    del pool

    # ---- config 4: B = 64 x 32K, nuq4; a step appends an 8K chunk per sequence, then one decode token each
    B, pre, chunk = 64, 24 * 1024, 8 * 1024
    ctx = pre + chunk + 1
    npg = -(-ctx // S)
    sc = make_scales([NUQ4], H, D, t_cal=4096, seed=400, device=device)
    NB = B * npg
    pool = CompactKVPool(1, NB, S, H, D, sc, device=device, outlier_frac=0.03)
    g = torch.Generator(device=device).manual_seed(401)
    bt = torch.randperm(NB, generator=g, device=device).to(torch.int32).view(B, npg)

    def slots_of(b, p):
        return bt[b, p // S].to(torch.int64) * S + p % S
    for b in range(B):
        K, V = make_kv(pre, H, D, seed=402 + b, outlier_frac=0.01, device=device, chan_seed=400)
        p = torch.arange(pre, device=device)
        pool.write_kv(0, K, V, slots_of(b, p), p)
    Kc, Vc = make_kv(B * chunk, H, D, seed=499, outlier_frac=0.01, device=device, chan_seed=400)
    pc = torch.arange(pre, pre + chunk, device=device)
    sc_slots = torch.cat([slots_of(b, pc) for b in range(B)])
    sc_pos = pc.repeat(B)
    K1, V1 = make_kv(B, H, D, seed=498, outlier_frac=0.01, device=device, chan_seed=400)
    last = torch.full((B,), ctx - 1, device=device)
    s1 = torch.stack([slots_of(b, last[b]) for b in range(B)])
    pool.write_kv(0, Kc, Vc, sc_slots, sc_pos)
    pool.write_kv(0, K1, V1, s1, last)
    append_ms = timer(lambda: pool.write_kv(0, Kc, Vc, sc_slots, sc_pos))
    g = torch.Generator(device=device).manual_seed(403)
    q = torch.randn((B, H * G, D), generator=g, device=device).to(torch.float16)
    sl = torch.full((B,), ctx, dtype=torch.int32, device=device)
    o = torch.empty((B, H * G, D), dtype=torch.float32, device=device)
    lse = torch.empty((B, H * G), dtype=torch.float32, device=device)
    scores = torch.empty((B, H, npg), dtype=torch.float32, device=device)
    thr4 = torch.empty((B * H,), dtype=torch.int64, device=device)
    nsl = int(__import__("hxlib").lib().hx_quest_slices(npg))
    slc = torch.empty((B * H, nsl + 1), dtype=torch.int32, device=device)

    def decode_step():
        pool.write_kv(0, K1, V1, s1, last)
        s_ = fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, scores=scores, thresh=thr4,
                                slice_out=slc)
        fused.decode(pool, 0, q, bt, sl, s_, o=o, lse=lse)
    dec_ms = timer(decode_step)
    pool.check()
    lay = pool.layers[0]
    dirc = lay.dir[:, :, :, 2].to(torch.int64)
    tok = B * chunk
    ent_chunk = int(dirc[:, bt[:, pre // S:(pre + chunk) // S].reshape(-1).long()].sum())
    append_b = tok * H * D * 2 * 2 + (tok // S) * H * lay.seg + 4 * ent_chunk + (tok // S) * H * 2 * D * 2 * 2 \
        + tok * H * 16 * 2 * 0  # positions past t_cal: the shared tail row
    sel = fused.quest_select(pool, 0, q, bt, sl, top_frac=(1, 4), sink_pages=4, lists=True)
    lists, counts = fused.selected_lists(sel)
    dec_b = 0
    for b in range(B):
        npg_b = ent = vr = 0
        for h in range(H):
            c = int(counts[b, h])
            pg = lists[b, h, :c].long()
            npg_b += c
            ent += int(dirc[h, bt[b, pg].long()].sum())
            vr += int((pg * S < 4096).sum())
        x = step_layer_bytes(npg, npg_b, ent, vr, lay.seg, 16)
        dec_b += x["stats"] + x["threshold"] + x["decode"]
    out["config4_batched"] = {
        "what": "B=64 sequences x 32K context on a shuffled block table, nuq4: append of an 8K-token chunk per "
                "sequence in one call (524,288 tokens), then per step one decode token per sequence "
                "(append + Quest 25% + 4 sinks + fused decode); L2 flushed before each call",
        "append_us": round(append_ms * 1e3, 1), "append_GBps": round(append_b / (append_ms * 1e-3) / 1e9, 1),
        "decode_step_us": round(dec_ms * 1e3, 1), "decode_GBps": round(dec_b / (dec_ms * 1e-3) / 1e9, 1),
        "roofline": roofline(append_b, append_ms, peak, src, "pack_kv_kernel<4,4> + pack_count_runs_kernel")}
    del pool, Kc, Vc
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# the reference's torch path on the host (cpu_baseline and --impl reference)

def reference_sample(args, gen_device, threads):
    """Build two whole layers (layer 0, nuq2; layer `cut`, nuq4) of the
    config-5 workload at full context in the reference's dense pool layout
    with its torch write path, on the host; returns them with their queries.
    Inputs are generated with torch (the same seeded tensors as the GPU arm
    when a GPU is present); nothing of this repository's CUDA library runs."""
    import torch
    from oracle.torch_step import write_layer
    from kvquant.synthetic import channel_scales
    torch.set_num_threads(threads)
    layout, scales = layer_scales_all(args, gen_device)
    qs = queries(args, gen_device).cpu()
    picks = sorted({0, min(args.cut, args.layers - 1)})
    layers, write_s = {}, {}
    for li in picks:
        lay = layout[li]
        cs = channel_scales(H, D, layer_seed(li), gen_device)
        Ks, Vs = [], []
        for c in range(-(-args.ctx // CHUNK)):
            K, V = layer_chunk(li, lay, c, gen_device, cs)
            n = min(CHUNK, args.ctx - c * CHUNK)
            Ks.append(K[:n].cpu())
            Vs.append(V[:n].cpu())
        K, V = torch.cat(Ks), torch.cat(Vs)
        del Ks, Vs
        ks, vs = scales.per_layer_keys[li].to("cpu"), scales.per_layer_values[li].to("cpu")
        t0 = time.perf_counter()
        layers[li] = write_layer(K, V, torch.arange(args.ctx), ks.poles, ks.upper_threshold, ks.lower_threshold,
                                 vs.poles, vs.upper_threshold, vs.lower_threshold, page=S)
        write_s[li] = (time.perf_counter() - t0, K.numel() * 2 * 2)
        del K, V
    return layers, qs, write_s


def reference_bytes(layer, sel):
    """Same algorithmic bytes as the GPU arm's step_layer_bytes for this
    layer's selection (packed-format sizes, outliers counted from the masks)."""
    import torch
    n = layer.k_min.shape[0]
    bk = 2 if layer.k_poles.shape[-1] <= 4 else 4
    bv = 2 if layer.v_poles.shape[-1] <= 4 else 4
    seg = S * D * (bk + bv) // 8
    ent = vrows = 0
    for h in range(H):
        pages = sel[:, h]
        tok = (pages.unsqueeze(1) * S + torch.arange(S)).reshape(-1)
        ent += int(layer.k_outm[tok, h].sum()) + int(layer.v_outm[tok, h].sum())
        vrows += int((pages * S < layer.v_poles.shape[1]).sum())
    b = step_layer_bytes(n, sel.numel(), ent, vrows, seg, layer.v_poles.shape[-1])
    return b["stats"] + b["threshold"] + b["decode"]


def time_reference(layers, qs, args, reps):
    """Per-layer decode wall time (median of reps) and its algorithmic bytes."""
    from oracle.torch_step import decode_layer
    res = {}
    for li, layer in layers.items():
        k = layer.k_min.shape[0] // 4
        ts = []
        sel = None
        for _ in range(reps):
            t0 = time.perf_counter()
            _, sel = decode_layer(layer, qs[li, 0], k, 4)
            ts.append(time.perf_counter() - t0)
        res[li] = (statistics.median(ts), reference_bytes(layer, sel))
    return res


def cpu_baseline(args, device):
    import torch
    threads = host_cores()
    layers, qs, write_s = reference_sample(args, device, threads)
    per = time_reference(layers, qs, args, reps=2)
    b = sum(x[1] for x in per.values())
    t = sum(x[0] for x in per.values())
    wb = sum(x[1] for x in write_s.values())
    wt = sum(x[0] for x in write_s.values())
    picks = sorted(layers)
    del layers
    return {"value": round(b / t / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"the reference's torch path (oracle/torch_step.py: page_upper_bound with the GQA sum, "
                      f"topk_pages_with_sinks, dequantisation of the selected pages, fp32 grouped attention) "
                      f"on layers {picks} (nuq2, nuq4), each whole at {args.ctx} ctx, median of 2 decodes each; "
                      f"the rate applies to the 28-layer step, whose time is extrapolated as 16 x nuq2 + 12 x nuq4 "
                      f"layers",
            "layer_s": {str(li): round(x[0], 3) for li, x in per.items()},
            "step_ms_extrapolated": round(1e3 * (min(args.cut, args.layers) * per[picks[0]][0]
                                                 + max(0, args.layers - args.cut) * per[picks[-1]][0]), 1),
            "pack": {"GBps": round(wb / wt / 1e9, 4), "what": "write_layer (quantise + dense store + fp32 "
                                                              "stats) of the same two layers; GB/s of fp16 "
                                                              "K/V read"}}


def run_reference(args):
    """The reference arm: the reference's torch path on the host cores."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    gen = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))) if torch.cuda.is_available() else \
        torch.device("cpu")
    threads = host_cores()
    layers, qs, write_s = reference_sample(args, gen, threads)
    if gen.type == "cuda":
        torch.cuda.empty_cache()
    time_reference(layers, qs, args, reps=max(1, args.warmup))          # warm-up
    t_run = time.perf_counter()
    steps = []
    for _ in range(args.steps):
        per = time_reference(layers, qs, args, reps=1)
        steps.append((sum(x[0] for x in per.values()), sum(x[1] for x in per.values())))
    run_s = time.perf_counter() - t_run
    t = statistics.median(s[0] for s in steps)
    b = steps[0][1]
    v = round(b / t / 1e9, 4)
    picks = sorted(layers)
    wb = sum(x[1] for x in write_s.values())
    wt = sum(x[0] for x in write_s.values())
    cfg = workload(args, world)
    return {"metric": METRIC, "impl": "reference", "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 values, uint8 codes (reference layout), fp32 softmax (torch CPU)",
            "data": "synthetic (the same seeded tensors as the GPU arm)", "config": cfg,
            "step_is": f"layers {picks} (one nuq2, one nuq4) of the config-5 step, each whole at {args.ctx} ctx; "
                       "value is the rate (same algorithmic bytes as the GPU arm / wall time)",
            "timed_region_s": round(run_s, 2),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"oracle/torch_step.py (the reference's torch path) on layers {picks}, "
                                       f"whole at {args.ctx} ctx, one decode each per step",
                             "pack": {"GBps": round(wb / wt / 1e9, 4)}},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the GPU arm

def run_ours(args):
    import torch
    import torch.distributed as dist
    import hxlib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        group = dist.group.WORLD

    W = build_world(args, rank, world, device)
    L = args.layers
    exchange = "none"
    if world > 1:
        # the layer exchange over peer memory (symmetric buffers, one merge
        # kernel per layer); every rank takes it or none does
        pex, err = None, ""
        if args.exchange == "p2p":
            from kvquant.splitkv import PeerExchange
            try:
                pex = PeerExchange(H * G, D, L, device, group)
            except Exception as e:  # no symmetric memory here: NCCL all-gather + merge
                err = f"{type(e).__name__}: {e}"
        agree = torch.tensor([1 if pex is not None else 0], dtype=torch.int32, device=device)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN)
        if int(agree.item()) == 0:
            pex = None
            if err:
                print(f"[bench] peer-memory exchange unavailable, using NCCL: {err}", file=sys.stderr)
        W["pex"] = pex
        exchange = "p2p (hx_exchange_merge over symmetric memory)" if pex is not None else \
            "nccl (all_gather_into_tensor + hx_merge_gathered)"

    # ---- device-resident timing (CUDA graph replay)
    step = make_step(W, world, group)
    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    # launches of this library's kernels in one step (counted at the C ABI)
    hxlib.launch_count[0] = 0
    step()
    torch.cuda.synchronize()
    launches_per_step = hxlib.launch_count[0]
    q_static = W["qs"].clone()
    graph = None
    # the whole step, the per-layer NCCL exchange included (the communicator
    # exists from the warm-up steps), is captured once and replayed
    use_graph = not args.no_graph
    if use_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step(q_static)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph):
                o_graph = step(q_static)
            torch.cuda.synchronize()
        except Exception as e:  # capture not possible: eager replay
            graph = None
            use_graph = False
            print(f"[bench] graph capture failed, timing eager steps: {e}", file=sys.stderr)
        if world > 1:  # every rank replays the graph or none does (same collectives on all ranks)
            agree = torch.tensor([1 if use_graph else 0], dtype=torch.int32, device=device)
            dist.all_reduce(agree, op=dist.ReduceOp.MIN)
            if int(agree.item()) == 0:
                graph = None
                use_graph = False
    run = (lambda: graph.replay()) if graph is not None else (lambda: step(q_static))
    for _ in range(args.warmup):
        run()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
    ms_dev = e0.elapsed_time(e1) / args.steps
    launches_graph = launches_per_step * args.steps
    if args.profile:
        if world > 1:
            dist.destroy_process_group()
        return None

    # ---- per-kernel timing (eager steps with events between the launches)
    timing = {"ev": [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(L)]}
    tstep = make_step(W, world, group, timing)
    tstep()
    torch.cuda.synchronize()
    sel_ms, dec_ms = [], []
    for _ in range(max(2, min(args.steps, 5))):
        tstep()
        torch.cuda.synchronize()
        for li in range(L):
            ev = timing["ev"][li]
            sel_ms.append(ev[0].elapsed_time(ev[1]))
            dec_ms.append(ev[1].elapsed_time(ev[2]))

    # ---- e2e: queries from pinned host memory into the step's input, the step,
    # the outputs back to host, every step (the captured step when there is one)
    q_host = W["qs"].cpu().pin_memory()
    o_host = torch.empty((L, H * G, D), dtype=torch.float32).pin_memory()
    o_dev = o_graph if graph is not None else None

    def e2e_step():
        q_static.copy_(q_host, non_blocking=True)
        if graph is not None:
            graph.replay()
            o_host.copy_(o_dev, non_blocking=True)
        else:
            o_host.copy_(step(q_static), non_blocking=True)
        torch.cuda.synchronize()
    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    ms_e2e = (time.perf_counter() - t0) * 1e3 / args.steps
    W["pool"].check()

    if world > 1:
        t = torch.tensor([ms_dev, ms_e2e, sum(sel_ms) / len(sel_ms), sum(dec_ms) / len(dec_ms)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_dev, ms_e2e, sel_avg, dec_avg = (float(x) for x in t.tolist())
    else:
        sel_avg, dec_avg = sum(sel_ms) / len(sel_ms), sum(dec_ms) / len(dec_ms)

    # bytes: all ranks (each rank's shard has its own selection; sum them)
    mine = sum(p["stats"] + p["threshold"] + p["decode"] for p in W["per_layer"])
    dec_b = sum(p["decode"] for p in W["per_layer"]) / L
    sc_b = sum(p["stats"] for p in W["per_layer"]) / L
    pack = W["pack"]
    if world > 1:
        v = torch.tensor([mine, pack["bytes"], pack["tokens"]], dtype=torch.float64, device=device)
        dist.all_reduce(v)
        tot_bytes, pack_bytes, pack_tokens = (float(x) for x in v.tolist())
        pm = torch.tensor([pack["ms"]], dtype=torch.float64, device=device)
        dist.all_reduce(pm, op=dist.ReduceOp.MAX)
        pack_ms = float(pm.item())
    else:
        tot_bytes, pack_bytes, pack_tokens, pack_ms = mine, pack["bytes"], pack["tokens"], pack["ms"]

    peak0, src0 = peaks()
    pack_warm = measure_pack(device, peak0, src0)
    if world > 1:   # every rank appends its own chunk at once: total tokens over the slowest rank
        pv = torch.tensor([pack_warm["us"]], dtype=torch.float64, device=device)
        dist.all_reduce(pv, op=dist.ReduceOp.MAX)
        us = float(pv.item())
        pack_warm["value"] = round(pack_warm["value"] * world * pack_warm["us"] / us, 2)
        pack_warm["us"] = round(us, 1)
        pack_warm["tokens"] *= world
    parity = None if args.no_parity else check_parity(W, args, world, rank, group)
    if graph is not None:
        del graph
    res = None
    if rank == 0:
        peak, peak_src = peaks()
        gbs = tot_bytes / (ms_dev * 1e-3) / 1e9
        # dominant kernel: the fused decode (per-launch algorithmic bytes / event time)
        dom = "decode" if dec_avg >= sel_avg else "quest_select"
        dom_b = dec_b if dom == "decode" else sc_b
        dom_ms = dec_avg if dom == "decode" else sel_avg
        res = {
            "metric": METRIC,
            "value": round(gbs, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_dev, 4),
            "decode_step_us": round(ms_dev * 1e3, 1),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp16 values, nuq2/nuq4 codes, fp32 softmax",
            "data": "synthetic (seeded N(0,1) x log-uniform channel scales, x10 outliers; random queries)",
            "config": workload(args, world),
            "run": {"cuda_graph": use_graph, "n_splits_per_head": W["ns"], "steps_replayed": args.steps,
                    "exchange": exchange, "decode_cores": W["cores"],
                    "selection_kernels": ("scores + decode (threshold inside the decode)"
                                          if W.get("gsel") is None and W["fused_select"]
                                          and W["shard"].n_pages <= 16384 else "scores + threshold + decode"),
                    "selection": ("top-K of the whole sequence (one GPU's)" if world == 1 or W.get("gsel") is not None
                                  else "top-K of each shard's pages")},
            "roofline": roofline(dom_b, dom_ms, peak, peak_src, dom, read_traffic(dom)),
            "kernels": {"quest_select_ms_per_layer": round(sel_avg, 5), "decode_ms_per_layer": round(dec_avg, 5),
                        "quest_select_GBps": round(sc_b / (sel_avg * 1e-3) / 1e9, 1),
                        "decode_GBps": round(dec_b / (dec_avg * 1e-3) / 1e9, 1)},
            "pack": pack_warm,
            "build_append_one_shot": {"value": round(pack_bytes / (pack_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "tokens": int(pack_tokens), "ms": round(pack_ms, 3),
                     "what": "the pool's build: the first append of every 64K-token chunk of every layer, "
                             "events around each call (host work and first-use preparation inside); "
                             "informational, the warm figure is 'pack'"},
            "e2e": {"value": round(tot_bytes / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(ms_e2e, 4),
                    "how": "queries H2D from pinned host memory, the " + ("captured" if use_graph else "eager")
                           + " step, outputs D2H, synchronise; wall clock",
                    "h2d_bytes_per_step": int(W["qs"].numel() * 2),
                    "d2h_bytes_per_step": int(L * H * G * D * 4)},
            "gpu_launches": launches_graph,
            "clocks": clk.summary(),
            "parity": parity,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and world == 1:
        del W
        torch.cuda.empty_cache()
        peak, peak_src = peaks()
        if not args.no_configs:
            res["configs"] = run_configs(device, peak, peak_src)
        if not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(args, device)
    return res


def main():
    args = parse()
    if args.impl == "reference":
        res = run_reference(args)
    else:
        res = run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
