"""Destination-range partition of a fan-in across ranks.

``fanin_reduce`` writes output row ``dst[e]`` from message row ``flat_src[e]``;
rows of different destinations never interact, in the forward or in either
backward. Splitting the destination rows into contiguous ranges, one per rank,
therefore splits the whole fan-in (sum and logsumexp, forward and backward)
into independent problems with no exchange between ranks: each rank owns the
edges whose destination falls in its range, the message rows those edges read,
and its slice of the output rows. The full output is the concatenation of the
ranks' outputs in rank order.

This is the op-level multi-GPU layout of the skewed stress workload (N=2^22,
E=2^26, 64 hub rows); hub rows stay whole on the rank whose range holds them.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def destination_ranges(dim_size: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, near-equal row ranges ``[lo, hi)`` covering ``[0, dim_size)``."""

    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    if dim_size < 0:
        raise ValueError(f"dim_size must be >= 0, got {dim_size}")
    base, extra = divmod(int(dim_size), int(world))
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


@dataclass
class DestinationShard:
    """One rank's part of a fan-in.

    ``edges``: positions of the rank's edges in the global edge list (in
    order); ``rel_rows``: the global message rows they read
    (``flat_src[edges]``); ``flat_src``: ``arange(len(edges))`` into the rank's
    own message rows ``rel[rel_rows]``; ``dst``: destinations relative to
    ``row_lo``; ``dim_size``: ``row_hi - row_lo``.
    """

    rank: int
    world: int
    row_lo: int
    row_hi: int
    edges: torch.Tensor
    rel_rows: torch.Tensor
    flat_src: torch.Tensor
    dst: torch.Tensor

    @property
    def dim_size(self) -> int:
        return self.row_hi - self.row_lo

    @property
    def num_edges(self) -> int:
        return int(self.edges.numel())


def shard_by_destination(flat_src: torch.Tensor, dst: torch.Tensor, dim_size: int, rank: int,
                         world: int) -> DestinationShard:
    """The edges of ``rank`` under the destination-range partition (one host
    sync for the edge count)."""

    if flat_src.shape != dst.shape or flat_src.dim() != 1:
        raise ValueError("flat_src and dst must be rank-1 tensors of equal length")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in [0, {world})")
    lo, hi = destination_ranges(dim_size, world)[rank]
    keep = (dst >= lo) & (dst < hi)
    edges = keep.nonzero().view(-1)
    rel_rows = flat_src.index_select(0, edges)
    local_dst = dst.index_select(0, edges) - lo
    local_src = torch.arange(edges.numel(), dtype=torch.int64, device=dst.device)
    return DestinationShard(rank, world, lo, hi, edges, rel_rows, local_src, local_dst)


def gather_output(parts: list[torch.Tensor]) -> torch.Tensor:
    """Full fan-in output from the ranks' outputs (rank order)."""

    return torch.cat(parts, dim=0)
