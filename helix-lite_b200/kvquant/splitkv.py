"""Split-KV decode across GPUs: shard plan, (o, lse) exchange, merge.

The sequence's pages are split into contiguous ranges, one per rank; each
rank keeps its range in its own CompactKVPool, selects its own top pages
(Quest on local pages; the sinks live on rank 0), runs the fused decode and
produces a normalised (o, lse) per query head. One all-gather moves the
partials (B*Hq*(D+1) floats per rank, a few KB) and a small kernel merges
them: o = sum_r exp(lse_r - M) o_r / sum_r exp(lse_r - M).

The reference runs this path on one GPU only (src/kvquant/compact_backend.py);
the exchange is the one collective the split adds.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    page_begin: int     # first global logical page owned by this rank
    n_pages: int        # pages owned
    sink_pages: int     # sinks selected on this rank (rank 0 only)


def shard_plan(n_pages: int, world: int, rank: int, sink_pages: int = 4) -> Shard:
    """Contiguous, near-equal page ranges; the first `base + 1` ranges take the remainder."""
    base, rem = divmod(n_pages, world)
    begin = rank * base + min(rank, rem)
    size = base + (1 if rank < rem else 0)
    return Shard(rank, world, begin, size, sink_pages if rank == 0 else 0)


def local_k(shard: Shard, frac=(1, 4)) -> int:
    """Pages a shard keeps besides its sinks: floor(n_local * frac)."""
    return shard.n_pages * frac[0] // frac[1]


class Exchange:
    """Preallocated exchange of one layer's split-KV partials.

    Each rank's row is [o (N x D) | lse (N)] fp32 in ``send``; one
    ``all_gather_into_tensor`` fills ``recv`` (R rows) and the merge kernel
    reads it in place (hx_merge_gathered), so a layer costs one collective and
    one small kernel, with no allocation or concatenation (the step can be
    captured in a CUDA graph). The decode may write straight into ``o_view`` /
    ``lse_view``.
    """

    def __init__(self, N: int, D: int, world: int, device, group=None):
        self.N, self.D, self.world, self.group = N, D, world, group
        self.send = torch.empty((N * (D + 1),), dtype=torch.float32, device=device)
        self.recv = torch.empty((world, N * (D + 1)), dtype=torch.float32, device=device)
        self.lse_out = torch.empty((N,), dtype=torch.float32, device=device)
        self.o_view = self.send[:N * D].view(N, D)
        self.lse_view = self.send[N * D:]

    def gather(self, o: torch.Tensor, lse: torch.Tensor):
        """All-gather; returns (R, N, D) and (R, N) views of the received rows."""
        if o.data_ptr() != self.o_view.data_ptr():
            self.o_view.copy_(o.reshape(self.N, self.D))
        if lse.data_ptr() != self.lse_view.data_ptr():
            self.lse_view.copy_(lse.reshape(self.N))
        dist.all_gather_into_tensor(self.recv.view(-1), self.send, group=self.group)
        nd = self.N * self.D
        return self.recv[:, :nd].view(self.world, self.N, self.D), self.recv[:, nd:]

    def merge(self, o: torch.Tensor, lse: torch.Tensor, out: torch.Tensor, out16: torch.Tensor | None = None):
        """Exchange and merge into ``out`` (N, D) fp32; returns (out, lse)."""
        import hxlib
        self.gather(o, lse)
        dev = self.send.device
        with torch.cuda.device(dev):
            hxlib.call("hx_merge_gathered", hxlib.stream(dev), hxlib.ptr(self.recv), self.world, self.N, self.D,
                       hxlib.ptr(out), hxlib.ptr(self.lse_out), hxlib.ptr(out16))
        return out, self.lse_out


class PeerExchange:
    """The exchange of every layer's partials over peer memory (no NCCL).

    Each rank owns symmetric buffers (torch's symmetric memory: every rank
    maps every other rank's allocation, CUDA IPC over NVLink): ``rows``
    (layers, N * (D + 1)) fp32 whose row l the decode of layer l writes
    ([o | lse], through ``o_view`` / ``lse_view``), and ``flags`` (layers,
    R) uint32. ``merge(l, out)`` launches hx_exchange_merge: signal, wait
    for every rank (bounded), merge the R rows read from the peers. One small
    kernel per layer replaces an all-gather plus the merge kernel, and it
    captures into a CUDA graph. Raises if symmetric memory is unavailable
    (callers fall back to ``Exchange``).
    """

    def __init__(self, N: int, D: int, layers: int, device, group=None, max_polls: int = 1 << 20):
        import torch.distributed._symmetric_memory as symm
        self.N, self.D, self.layers = N, D, layers
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        grp = group if group is not None else dist.group.WORLD
        self.rows = symm.empty((layers, N * (D + 1)), dtype=torch.float32, device=device)
        self.flags = symm.empty((layers * self.world,), dtype=torch.int32, device=device)
        self.flags.zero_()
        h_rows = symm.rendezvous(self.rows, grp)
        h_flags = symm.rendezvous(self.flags, grp)
        self.peer_rows = torch.tensor(list(h_rows.buffer_ptrs), dtype=torch.int64, device=device)
        self.peer_flags = torch.tensor(list(h_flags.buffer_ptrs), dtype=torch.int64, device=device)
        self.lse_out = torch.empty((layers, N), dtype=torch.float32, device=device)
        self.max_polls = int(max_polls)
        torch.cuda.synchronize(device)
        dist.barrier(group)

    def o_view(self, layer: int) -> torch.Tensor:
        return self.rows[layer, :self.N * self.D].view(self.N, self.D)

    def lse_view(self, layer: int) -> torch.Tensor:
        return self.rows[layer, self.N * self.D:]

    def merge(self, layer: int, out: torch.Tensor, out16: torch.Tensor | None = None):
        """Exchange and merge layer ``layer`` into ``out`` (N, D) fp32; returns (out, lse)."""
        import hxlib
        dev = self.rows.device
        with torch.cuda.device(dev):
            hxlib.call("hx_exchange_merge", hxlib.stream(dev), hxlib.ptr(self.peer_rows), hxlib.ptr(self.peer_flags),
                       self.world, self.rank, layer, self.N, self.D, hxlib.ptr(out), hxlib.ptr(self.lse_out[layer]),
                       hxlib.ptr(out16), self.max_polls, hxlib.ptr(hxlib.err_word(dev)))
        return out, self.lse_out[layer]


def gather_score_rows(loc: torch.Tensor, gathered: torch.Tensor, glob: torch.Tensor, group=None):
    """Every rank's page scores in global page order.

    loc (B, H, n) this rank's scores of its n pages; gathered (R, B*H, n)
    scratch; glob (B, H, R*n) receives row (b, h) = the R ranks' rows (b, h)
    one after another (rank r's pages are global pages r*n .. r*n + n - 1).
    One all-gather and one strided copy."""
    B, H, n = loc.shape
    R = gathered.shape[0]
    dist.all_gather_into_tensor(gathered.view(-1), loc.reshape(-1), group=group)
    glob.view(B * H, R, n).copy_(gathered.permute(1, 0, 2))
    return glob


class GlobalSelect:
    """Quest selection over the whole sequence when its pages are split.

    With per-shard selection every rank keeps the top quarter of its own
    pages, which is not the single-GPU top-K. Here each rank scores its own
    pages, the scores are all-gathered into global page order (R * n fp32
    per (b, h): 128 KB per rank per layer at 1M tokens on 8 ranks), every
    rank runs the same exact threshold kernel over the global rows (so the
    threshold is the single-GPU one, bit for bit, and the ranks agree), and
    hx_quest_localize turns it into the rank's threshold over its local
    page indices plus the decode's slice counts. The result is a
    ``Selection`` the decode takes as usual. Requires equal shards (n pages
    on every rank; the sequence ends on the last rank). Follows the
    single-GPU selection of src/kvquant/quest_selector.py:70-83.
    """

    def __init__(self, B: int, H: int, n_local: int, world: int, device, group=None, sink_pages: int = 4,
                 top_frac=(1, 4), top_k: int | None = None):
        import hxlib
        self.B, self.H, self.n, self.world, self.group = B, H, n_local, world, group
        self.sinks = sink_pages
        self.kf, self.fn, self.fd = ((int(top_k), 0, 0) if top_k is not None
                                     else (0, int(top_frac[0]), int(top_frac[1])))
        ng = world * n_local
        f32 = dict(dtype=torch.float32, device=device)
        self.loc = torch.empty((B, H, n_local), **f32)
        self.gathered = torch.empty((world, B * H, n_local), **f32)
        self.glob = torch.empty((B, H, ng), **f32)
        self.thresh_g = torch.empty((B * H,), dtype=torch.int64, device=device)
        self.thresh = torch.empty((B * H,), dtype=torch.int64, device=device)
        self.slice_off = torch.empty((B * H, int(hxlib.lib().hx_quest_slices(n_local)) + 1), dtype=torch.int32,
                                     device=device)
        # threshold scratch: left zeroed by the kernel after each use
        self.hist = torch.zeros((B * H * 2 * 4096,), dtype=torch.int32, device=device)
        self.cand = torch.empty((B * H * max(ng, 1),), dtype=torch.int64, device=device)
        self.ctr = torch.zeros((B * H * 2,), dtype=torch.int32, device=device)
        self.seq_glob = torch.empty((B,), dtype=torch.int32, device=device)

    def set_lengths(self, seq_lens_global: torch.Tensor):
        """Tokens of each whole sequence (B,); call before capture or when they change."""
        self.seq_glob.copy_(seq_lens_global.to(self.seq_glob.device, torch.int32))

    def select(self, pool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
               seq_lens: torch.Tensor, shard: Shard, gqa: str = "sum"):
        """This rank's part of the global selection: a Selection over its
        local pages (block_table / seq_lens local, as for splitkv_decode)."""
        import hxlib
        from .fused import Selection, page_scores
        dev = pool.device
        q = query.to(device=dev, dtype=torch.float16).contiguous()
        bt = block_table.to(device=dev, dtype=torch.int32).contiguous()
        sl = seq_lens.to(device=dev, dtype=torch.int32).contiguous()
        S = pool.block_size
        sinks = max(0, min(self.sinks - shard.page_begin, self.n))   # the global sinks on this shard
        with torch.cuda.device(dev):
            st = hxlib.stream(dev)
            page_scores(pool, layer_idx, q, bt, sl, self.n, sinks, self.loc, None, gqa)
            gather_score_rows(self.loc, self.gathered, self.glob, self.group)
            hxlib.call("hx_quest_threshold_slices", st, hxlib.ptr(self.glob), self.B, self.H, hxlib.ptr(self.seq_glob),
                       S, self.world * self.n, self.sinks, self.kf, self.fn, self.fd, 0, hxlib.ptr(self.hist),
                       hxlib.ptr(self.cand), hxlib.ptr(self.ctr), hxlib.ptr(self.thresh_g), None,
                       hxlib.ptr(hxlib.err_word(dev)))
            hxlib.call("hx_quest_localize", st, hxlib.ptr(self.thresh_g), hxlib.ptr(self.loc), self.B, self.H,
                       hxlib.ptr(sl), S, self.n, sinks, shard.page_begin, hxlib.ptr(self.thresh),
                       hxlib.ptr(self.slice_off))
        return Selection(self.loc, self.thresh, sl, S, self.n, sinks, None, None, self.slice_off)


_EXCHANGES: dict = {}


def _exchange(N: int, D: int, device, group=None) -> Exchange:
    world = dist.get_world_size(group)
    key = (N, D, str(device), world, id(group))
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = Exchange(N, D, world, device, group)
    return ex


def exchange_partials(o: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather normalised partials: o (N, D), lse (N,) -> (R, N, D), (R, N).

    o and lse travel in one buffer (cached per shape and device) so the
    exchange is a single collective; the results are views of that buffer,
    valid until the next exchange of the same shape.
    """
    N, D = o.shape
    return _exchange(N, D, o.device, group).gather(o.float(), lse.float())


def splitkv_decode(pool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
                   seq_lens: torch.Tensor, shard: Shard, *, quest: bool = True, frac=(1, 4), gqa: str = "sum",
                   group=None, n_splits: int | None = None, out16: torch.Tensor | None = None):
    """Decode one token per sequence over a sharded sequence.

    ``block_table`` and ``seq_lens`` describe this rank's local pages and
    tokens; ``shard.page_begin`` places them in the global sequence (V's
    position clamp). Returns the merged (o (B, Hq, D) fp32, lse (B, Hq)).
    """
    from .fused import decode, quest_select
    B, Hq, D = query.shape
    sel = None
    if quest:
        sel = quest_select(pool, layer_idx, query, block_table, seq_lens, top_k=local_k(shard, frac),
                           sink_pages=shard.sink_pages, gqa=gqa)
    ex = _exchange(B * Hq, D, query.device, group)
    decode(pool, layer_idx, query, block_table, seq_lens, sel, page_begin=shard.page_begin, n_splits=n_splits,
           o=ex.o_view.view(B, Hq, D), lse=ex.lse_view.view(B, Hq))
    om = torch.empty((B * Hq, D), dtype=torch.float32, device=query.device)
    om, lm = ex.merge(ex.o_view, ex.lse_view, om, out16)
    return om.view(B, Hq, D), lm.clone().view(B, Hq)
