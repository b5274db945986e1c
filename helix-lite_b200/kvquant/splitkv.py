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
