"""Quest block selection on a CompactKVPool (src/kvquant/quest_selector.py:38-90).

Same call and result as the reference: the union over KV heads of each
head's sinks + top-k blocks, as sorted block ids with their first token
positions (``block_id * block_size``). Scores come from the pool's K min /
max through the CUDA score kernel (one query row per KV head, the bound of
src/quest/reference.py:59-93); the per-head top-k is exact with ties to the
lower block.
"""
from __future__ import annotations

import torch

from .compact_pool import CompactKVPool
from .fused import quest_select, selected_lists


def select_top_blocks_for_layer(pool: CompactKVPool, layer_idx: int, query: torch.Tensor,
                                used_block_ids: torch.Tensor, block_size: int, top_k: int,
                                sink_blocks: int = 4):
    NU = int(used_block_ids.shape[0])
    dev = pool.device
    sinks = max(0, min(sink_blocks, NU))
    keep = max(0, min(top_k, NU - sinks))
    q = query.to(device=dev, dtype=torch.float16).reshape(1, pool.num_kv_heads, -1)
    bt = used_block_ids.to(device=dev, dtype=torch.int32).reshape(1, NU)
    sl = torch.tensor([NU * pool.block_size], dtype=torch.int32, device=dev)
    sel = quest_select(pool, layer_idx, q, bt, sl, top_k=keep, sink_pages=sinks, gqa="sum", max_pages=NU)
    idx, cnt = selected_lists(sel, union=True, max_out=NU)
    n = int(cnt[0].item())
    ids = used_block_ids.to(dev)[idx[0, :n].long()].to(torch.int64)
    ids, _ = ids.sort()
    return ids, ids * block_size
