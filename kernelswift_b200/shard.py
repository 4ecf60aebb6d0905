"""Row sharding of the operators over ranks (one process per GPU).

Every output row of the three operators depends only on its own query row plus
read-only data (kv, keys, sinks, weights), so rows shard with no exchange on
the data path:

* ``contiguous(n, world, rank)`` for uniform-cost rows (Sinkhorn matrices,
  sparse-attention queries);
* ``zigzag(n, world, rank)`` for causal indexer rows, whose cost grows with the
  position: the rows are cut into 2*world chunks and rank r takes chunks r and
  2*world-1-r, so every rank gets the same total causal work (the reference
  balances its cores the same way, by striding rows,
  optimized/indexer_project/op_kernel/indexer_topk.asc:98-106).

``gather_rows`` reassembles a full output from the ranks' shards with one
all-gather (outside any timed region in bench.py).
"""
from __future__ import annotations

import torch


def contiguous(n: int, world: int, rank: int) -> list[tuple[int, int]]:
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    stop = start + base + (1 if rank < rem else 0)
    return [(start, stop)] if stop > start else []


def zigzag(n: int, world: int, rank: int) -> list[tuple[int, int]]:
    """Rank r's causal rows: chunks r and 2*world-1-r of 2*world; the two are one
    range when they touch (world == 1), so a single rank runs one call per op."""
    chunks = contiguous_chunks(n, 2 * world)
    out = [c for c in (chunks[rank], chunks[2 * world - 1 - rank]) if c[1] > c[0]]
    if len(out) == 2 and out[0][1] == out[1][0]:
        out = [(out[0][0], out[1][1])]
    return out


def contiguous_chunks(n: int, parts: int) -> list[tuple[int, int]]:
    return [(contiguous(n, parts, r) or [(0, 0)])[0] for r in range(parts)]


def causal_cost(ranges: list[tuple[int, int]]) -> int:
    """Sum of (s + 1) over the rows: proportional to causal indexer work."""
    return sum((a + b + 1) * (b - a) // 2 for a, b in ranges)


def gather_rows(local: torch.Tensor, ranges_per_rank: list[list[tuple[int, int]]], dim: int,
                group=None) -> torch.Tensor:
    """All-gather row shards (concatenated along ``dim`` in each rank's range
    order) and scatter them back into global row order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    sizes = [sum(b - a for a, b in r) for r in ranges_per_rank]
    maxn = max(sizes)
    shape = list(local.shape)
    shape[dim] = maxn
    pad = local.new_zeros(shape)
    pad.narrow(dim, 0, local.shape[dim]).copy_(local)
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    total = sum(sizes)
    shape[dim] = total
    out = local.new_empty(shape)
    for r in range(world):
        off = 0
        for a, b in ranges_per_rank[r]:
            out.narrow(dim, a, b - a).copy_(bufs[r].narrow(dim, off, b - a))
            off += b - a
    return out
