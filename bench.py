#!/usr/bin/env python
"""Benchmark of the long-context KV hot path (BASELINE config 5 by default).

One step = a full 28-layer decode step at 1M context served from the compact
pool: per layer, Quest page scores over every page (fp16 K min / max), the
exact top-25% + 4 sinks threshold, and the fused-dequant split-KV decode
(layers 0-15 nuq2 with 5% outliers, 16-27 nuq4 with 1%); 4 KV / 28 query
heads, head_dim 128, 16-token pages. With N ranks the sequence's pages are
split N ways (split-KV): each rank selects and attends its shard and one
NCCL all-gather of (o, lse) per layer feeds the merge.

  value   effective KV GB/s: algorithmic bytes of the step (stats scanned +
          selected code segments + their outlier entries and directory
          records + V level rows + q / o) / device step time, all ranks;
          the step replays as a CUDA graph with inputs resident in HBM
  e2e     the same bytes / wall time through the public Python API (eager
          calls) with the 28 queries copied from pinned host memory and the
          outputs read back to host every step

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
    ap.add_argument("--cpu-sample-pages", type=int, default=4096)
    ap.add_argument("--profile", action="store_true", help="setup + warmup + steps only (for ncu)")
    return ap.parse_args()


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
        bits = {"nvmlClocksEventReasonHwSlowdown": 0x8, "nvmlClocksEventReasonHwThermalSlowdown": 0x40,
                "nvmlClocksEventReasonSwThermalSlowdown": 0x20, "nvmlClocksEventReasonSwPowerCap": 0x4}
        names = {getattr(nv, n, b): n for n, b in bits.items()}
        label = {"nvmlClocksEventReasonHwSlowdown": "hw_slowdown",
                 "nvmlClocksEventReasonHwThermalSlowdown": "hw_thermal_slowdown",
                 "nvmlClocksEventReasonSwThermalSlowdown": "sw_thermal_slowdown",
                 "nvmlClocksEventReasonSwPowerCap": "sw_power_cap"}
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
                r = fn(self.h)
                for bit, n in names.items():
                    if bit is not None and r & bit:
                        self.reasons.add(label[n])
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
# workload

def layer_seed(layer):
    return 1234 + 1000 * layer


def build_world(args, rank, world, device):
    import torch
    from kvquant import fused
    from kvquant.compact_pool import CompactKVPool
    from kvquant.splitkv import local_k, shard_plan
    from kvquant.synthetic import NUQ2, NUQ4, channel_scales, make_kv, make_scales, mixed_layout

    n_pages = args.ctx // S
    shard = shard_plan(n_pages, world, rank)
    layout = mixed_layout(args.layers, args.cut)
    scales = make_scales(layout, H, D, t_cal=4096, seed=1234, device=device, calib_tokens=4096)
    fracs = [0.10 if lay is NUQ2 else 0.03 for lay in layout]
    pool = CompactKVPool(args.layers, shard.n_pages, S, H, D, scales, device=device, outlier_frac=fracs)

    # fill: global chunks of 64K tokens so a token's data does not depend on N
    CH = 1 << 16
    t0g, t1g = shard.page_begin * S, (shard.page_begin + shard.n_pages) * S
    pack_ms, pack_tokens = 0.0, 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for li, lay in enumerate(layout):
        cs = channel_scales(H, D, layer_seed(li), device)
        for c in range(t0g // CH, (t1g + CH - 1) // CH):
            a, b = max(c * CH, t0g), min((c + 1) * CH, t1g)
            K, V = make_kv(CH, H, D, seed=layer_seed(li) + 7 * c + 1, outlier_frac=lay[1], device=device,
                           chan_scale=cs)
            K, V = K[a - c * CH:b - c * CH].contiguous(), V[a - c * CH:b - c * CH].contiguous()
            pos = torch.arange(a, b, device=device)
            ev0.record()
            pool.write_kv(li, K, V, pos - t0g, pos)
            ev1.record()
            ev1.synchronize()
            pack_ms += ev0.elapsed_time(ev1)
            pack_tokens += b - a
    pool.check()

    g = torch.Generator(device=device).manual_seed(99)
    qs = torch.randn((args.layers, 1, H * G, D), generator=g, device=device).to(torch.float16)
    bt = torch.arange(shard.n_pages, dtype=torch.int32, device=device).unsqueeze(0)
    sl = torch.tensor([shard.n_pages * S], dtype=torch.int32, device=device)
    kk = local_k(shard)
    ns = fused.default_splits(1, H, shard.n_pages)

    # algorithmic bytes: selection is fixed per layer (fixed queries)
    per_layer = []
    for li in range(args.layers):
        sel = fused.quest_select(pool, li, qs[li], bt, sl, top_k=kk, sink_pages=shard.sink_pages)
        lists, counts = fused.selected_lists(sel)
        lay = pool.layers[li]
        dirc = lay.dir[:, :, :, 2].to(torch.int64)                 # (H, NB, 2)
        ent = 0
        npages = 0
        vrows = 0
        for h in range(H):
            c = int(counts[0, h])
            pg = lists[0, h, :c].long()
            npages += c
            ent += int(dirc[h, pg].sum())
            vrows += int(((shard.page_begin + pg) * S < 4096).sum())
        levels_v = int(scales.per_layer_values[li].poles.shape[-1])
        stats_b = shard.n_pages * H * 2 * D * 2
        dec_b = npages * (lay.seg + 32) + 4 * ent + vrows * S * levels_v * 2 + shard.n_pages * H * 4
        qo_b = H * G * D * 2 + H * G * (D + 1) * 4
        per_layer.append({"stats": stats_b + shard.n_pages * H * 4, "decode": dec_b + qo_b,
                          "threshold": shard.n_pages * H * 4, "pages": npages, "entries": ent})
    pack_bytes = 0
    for li in range(args.layers):
        lay = pool.layers[li]
        pack_bytes += shard.n_pages * S * H * D * 2 * 2                  # fp16 K, V read
        pack_bytes += shard.n_pages * H * lay.seg                        # codes written
        pack_bytes += shard.n_pages * H * 2 * D * 2 * 2                  # stats read + written
        pack_bytes += 4 * int(lay.dir[:, :, :, 2].to(torch.int64).sum())  # outlier entries written
    return dict(pool=pool, shard=shard, qs=qs, bt=bt, sl=sl, k=kk, ns=ns, per_layer=per_layer,
                pack=dict(ms=pack_ms, tokens=pack_tokens, bytes=pack_bytes), scales=scales, layout=layout)


def make_step(W, world, group, timing=None):
    """The decode step over all layers; `timing` records events around each kernel group."""
    import torch
    import hxlib
    from kvquant import fused
    from kvquant.splitkv import exchange_partials

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

    def step(q_in=None):
        q_all = qs if q_in is None else q_in
        for li in range(L):
            if timing is not None:
                timing["ev"][li][0].record()
            sel = fused.quest_select(pool, li, q_all[li], bt, sl, top_k=W["k"], sink_pages=shard.sink_pages,
                                     scores=scores[li], thresh=thresh[li], slice_out=slices[li])
            if timing is not None:
                timing["ev"][li][1].record()
            # one GPU: the decode writes the layer's output in place
            fused.decode(pool, li, q_all[li], bt, sl, sel, page_begin=shard.page_begin, n_splits=W["ns"],
                         o=o_loc[li] if world > 1 else o_out[li].view(1, H * G, D), lse=lse_loc[li])
            if timing is not None:
                timing["ev"][li][2].record()
            if world > 1:
                O, Lz = exchange_partials(o_loc[li].view(H * G, D), lse_loc[li].view(H * G), group)
                om, _ = fused.merge_partials(O, Lz)
                o_out[li].copy_(om)
        return o_out

    return step


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

    # ---- device-resident timing (CUDA graph replay)
    timing = {"ev": [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(L)]}
    step = make_step(W, world, group)
    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    # launches of this library's kernels in one step (counted at the C ABI)
    hxlib.launch_count[0] = 0
    step()
    torch.cuda.synchronize()
    launches_per_step = hxlib.launch_count[0]
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
                step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph):
                step()
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
    run = (lambda: graph.replay()) if graph is not None else step
    for _ in range(args.warmup):
        run()
    hxlib.launch_count[0] = 0
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

    # ---- per-kernel timing (eager steps with events between the launches)
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

    # ---- e2e through the public API with host buffers
    q_host = W["qs"].cpu().pin_memory()
    o_host = torch.empty((L, H * G, D), dtype=torch.float32).pin_memory()
    q_dev = torch.empty_like(W["qs"])
    estep = make_step(W, world, group)
    for _ in range(args.warmup):
        q_dev.copy_(q_host, non_blocking=True)
        o_host.copy_(estep(q_dev), non_blocking=True)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        q_dev.copy_(q_host, non_blocking=True)
        o_host.copy_(estep(q_dev), non_blocking=True)
        torch.cuda.synchronize()
    ms_e2e = (time.perf_counter() - t0) * 1e3 / args.steps
    W["pool"].check()

    if world > 1:
        t = torch.tensor([ms_dev, ms_e2e, sum(sel_ms) / len(sel_ms), sum(dec_ms) / len(dec_ms)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_dev, ms_e2e, sel_avg, dec_avg = (float(x) for x in t.tolist())
    else:
        sel_avg, dec_avg = sum(sel_ms) / len(sel_ms), sum(dec_ms) / len(dec_ms)

    # bytes: all ranks (each rank's shard has its own selection; sum them)
    import torch as _t
    mine = sum(p["stats"] + p["threshold"] + p["decode"] for p in W["per_layer"])
    dec_b = sum(p["decode"] for p in W["per_layer"]) / L
    sc_b = sum(p["stats"] for p in W["per_layer"]) / L
    pack = W["pack"]
    if world > 1:
        v = _t.tensor([mine, pack["bytes"], pack["tokens"]], dtype=_t.float64, device=device)
        dist.all_reduce(v)
        tot_bytes, pack_bytes, pack_tokens = (float(x) for x in v.tolist())
        pm = _t.tensor([pack["ms"]], dtype=_t.float64, device=device)
        dist.all_reduce(pm, op=dist.ReduceOp.MAX)
        pack_ms = float(pm.item())
    else:
        tot_bytes, pack_bytes, pack_tokens, pack_ms = mine, pack["bytes"], pack["tokens"], pack["ms"]

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
        achieved = dom_b / (dom_ms * 1e-3) / 1e9
        traffic = read_traffic(dom)
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
            "config": {"workload": f"config5: {args.layers}-layer mixed nuq2/nuq4 decode step, "
                                   f"{args.ctx} ctx, Quest 25%+4 sinks, split-KV over {world} GPU(s)",
                       "context_tokens": args.ctx, "layers": args.layers, "nuq2_layers": args.cut,
                       "kv_heads": H, "q_heads": H * G, "head_dim": D, "page": S, "batch": 1,
                       "l2": "inputs larger than L2 (stats + selected codes per step >> 126 MB)",
                       "cuda_graph": use_graph, "n_splits_per_head": W["ns"]},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                         "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "algorithmic_bytes_per_launch": int(dom_b),
                         "avg_launch_ms": round(dom_ms, 5)},
            "kernels": {"quest_select_ms_per_layer": round(sel_avg, 5), "decode_ms_per_layer": round(dec_avg, 5),
                        "quest_select_GBps": round(sc_b / (sel_avg * 1e-3) / 1e9, 1),
                        "decode_GBps": round(dec_b / (dec_avg * 1e-3) / 1e9, 1)},
            "pack": {"value": round(pack_bytes / (pack_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "tokens": int(pack_tokens), "ms": round(pack_ms, 3),
                     "what": "append of the whole context for all layers, 64K-token chunks"},
            "e2e": {"value": round(tot_bytes / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(ms_e2e, 4),
                    "h2d_bytes_per_step": int(W["qs"].numel() * 2),
                    "d2h_bytes_per_step": int(L * H * G * D * 4)},
            "gpu_launches": launches_graph,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(W, args, workers=1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


# ---------------------------------------------------------------------------
# CPU port (oracle) baseline

def host_layer(pool, li, n_pages):
    import numpy as np
    from oracle.cpu_step import HostLayer
    lay = pool.layers[li]
    rbk, rbv = D * lay.bits_k // 8, D * lay.bits_v // 8
    codes = lay.codes[:, :n_pages].cpu().numpy()
    kr = codes[:, :, :S * rbk].reshape(H, n_pages, S, rbk)
    vr = codes[:, :, S * rbk:].reshape(H, n_pages, S, rbv)
    stats = lay.stats[:, :n_pages].cpu().numpy()
    d = lay.dir[:, :n_pages].cpu().numpy().astype(np.int64)
    arena = lay.arena.cpu().numpy().astype(np.int64) & 0xFFFFFFFF
    lists = [[], []]
    for kv in range(2):
        for h in range(H):
            row = []
            for p in range(n_pages):
                off, _, cnt, _ = d[h, p, kv]
                e = arena[off:off + cnt]
                row.append(((e >> 24) & 31, (e >> 16) & 255, (e & 0xFFFF).astype(np.uint16).view(np.float16)))
            lists[kv].append(row)
    sc = pool.scales
    return HostLayer(kr, vr, stats, lists[0], lists[1], sc.per_layer_keys[li].poles.cpu().numpy(),
                     sc.per_layer_values[li].poles.cpu().numpy(), lay.bits_k, lay.bits_v,
                     int(sc.per_layer_values[li].poles.shape[1]))


def _cpu_time_layer(hl, q, n_pages, reps):
    from oracle.cpu_step import algorithmic_bytes, decode_layer
    t0 = time.perf_counter()
    for _ in range(reps):
        o, chosen = decode_layer(hl, q, n_pages * S, G)
    dt = (time.perf_counter() - t0) / reps
    return algorithmic_bytes(hl, chosen, H * G, D), dt


def cpu_baseline(W, args, workers=1):
    """Time the CPU port on one nuq2 and one nuq4 layer restricted to the first
    `cpu_sample_pages` pages, then scale to the full step by bytes."""
    pool, shard = W["pool"], W["shard"]
    n = min(args.cpu_sample_pages, shard.n_pages)
    per_type = {}
    picks = {"nuq2": 0, "nuq4": min(args.cut, args.layers - 1)}
    for name, li in picks.items():
        hl = host_layer(pool, li, n)
        q = W["qs"][li, 0].cpu().numpy()
        b, dt = _cpu_time_layer(hl, q, n, reps=1)
        per_type[name] = (b, dt)
    gbs = {k: b / dt / 1e9 for k, (b, dt) in per_type.items()}
    # full-step CPU time: each layer's full-context bytes at its type's rate
    t = 0.0
    tot = 0
    for li, p in enumerate(W["per_layer"]):
        by = p["stats"] + p["threshold"] + p["decode"]
        tot += by
        t += by / (gbs["nuq2" if li < args.cut else "nuq4"] * 1e9)
    return {"value": round(tot / t / 1e9, 4), "unit": "GB/s", "cores": workers, "kind": "port",
            "step_ms_estimate": round(t * 1e3, 1),
            "sample": f"oracle numpy port (scores, top-k, dequant, fp32 attention) on layers "
                      f"{picks['nuq2']} (nuq2) and {picks['nuq4']} (nuq4), first {n} pages "
                      f"({n * S} tokens) each, scaled to the full step by algorithmic bytes",
            "per_layer_GBps": {k: round(v, 4) for k, v in gbs.items()}}


def run_reference(args):
    """The reference arm: the CPU port of the path on this host's cores."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    if not torch.cuda.is_available():
        return {"impl": "reference", "unavailable": "needs the GPU to build the synthetic pool it reads"}
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    W = build_world(args, 0, 1, device)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    vals = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(W, args, workers=1)
        if i >= args.warmup:
            vals.append(cb)
    v = statistics.median(c["value"] for c in vals)
    ms = statistics.median(c["step_ms_estimate"] for c in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    return {"metric": METRIC, "impl": "reference", "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 values, fp32 softmax (numpy)",
            "data": "synthetic (same seeded pool as the GPU arm)",
            "config": {"workload": f"config5: {args.layers}-layer mixed nuq2/nuq4 decode step, {args.ctx} ctx, "
                                   "Quest 25%+4 sinks", "context_tokens": args.ctx},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


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
