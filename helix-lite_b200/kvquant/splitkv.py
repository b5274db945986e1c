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


def exchange_partials(o: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather normalised partials: o (N, D), lse (N,) -> (R, N, D), (R, N).

    o and lse travel in one buffer so the exchange is a single collective.
    """
    N, D = o.shape
    world = dist.get_world_size(group)
    send = torch.cat([o.reshape(-1).float(), lse.reshape(-1).float()])
    recv = torch.empty((world * send.numel(),), dtype=send.dtype, device=send.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    recv = recv.view(world, send.numel())
    return recv[:, :N * D].reshape(world, N, D), recv[:, N * D:].reshape(world, N)


def splitkv_decode(pool, layer_idx: int, query: torch.Tensor, block_table: torch.Tensor,
                   seq_lens: torch.Tensor, shard: Shard, *, quest: bool = True, frac=(1, 4), gqa: str = "sum",
                   group=None, n_splits: int | None = None, out16: torch.Tensor | None = None):
    """Decode one token per sequence over a sharded sequence.

    ``block_table`` and ``seq_lens`` describe this rank's local pages and
    tokens; ``shard.page_begin`` places them in the global sequence (V's
    position clamp). Returns the merged (o (B, Hq, D) fp32, lse (B, Hq)).
    """
    from .fused import decode, merge_partials, quest_select
    B, Hq, D = query.shape
    sel = None
    if quest:
        sel = quest_select(pool, layer_idx, query, block_table, seq_lens, top_k=local_k(shard, frac),
                           sink_pages=shard.sink_pages, gqa=gqa)
    o, lse = decode(pool, layer_idx, query, block_table, seq_lens, sel, page_begin=shard.page_begin,
                    n_splits=n_splits)
    O, L = exchange_partials(o.view(B * Hq, D), lse.view(B * Hq), group)
    om, lm = merge_partials(O, L, out16)
    return om.view(B, Hq, D), lm.view(B, Hq)
