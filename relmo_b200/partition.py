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
``balanced_destination_ranges`` places the range boundaries by cumulative
work (rows + edges) instead of row count, so ranks that hold hub rows get
fewer rows.
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


def balanced_destination_ranges(dst: torch.Tensor, dim_size: int, world: int) -> list[tuple[int, int]]:
    """Contiguous row ranges that split the work (one unit per destination row
    plus one per edge into it, the merge-path items the kernels walk) as evenly
    as contiguous ranges can: boundary r is the first row whose cumulative work
    reaches r/world of the total. One host sync (the boundaries)."""

    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    if dim_size < 0:
        raise ValueError(f"dim_size must be >= 0, got {dim_size}")
    if dim_size == 0 or world == 1:
        return destination_ranges(dim_size, world)
    work = torch.ones(int(dim_size), dtype=torch.int64, device=dst.device)
    work.index_add_(0, dst, torch.ones_like(dst))
    cum = torch.cumsum(work, 0)
    total = int(dim_size) + int(dst.numel())
    targets = torch.tensor([(total * r + world - 1) // world for r in range(1, world)], dtype=torch.int64,
                           device=dst.device)
    cuts = torch.searchsorted(cum, targets, right=False) + 1  # rows [0, cut) reach the target
    bounds = [0] + [min(int(c), int(dim_size)) for c in cuts.tolist()] + [int(dim_size)]
    for i in range(1, len(bounds)):
        bounds[i] = max(bounds[i], bounds[i - 1])
    return [(bounds[i], bounds[i + 1]) for i in range(world)]


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
                         world: int, ranges: list[tuple[int, int]] | None = None) -> DestinationShard:
    """The edges of ``rank`` under a destination-range partition: ``ranges``
    (e.g. ``balanced_destination_ranges``), else equal row counts. One host
    sync for the edge count."""

    if flat_src.shape != dst.shape or flat_src.dim() != 1:
        raise ValueError("flat_src and dst must be rank-1 tensors of equal length")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in [0, {world})")
    if ranges is None:
        ranges = destination_ranges(dim_size, world)
    if len(ranges) != world or ranges[0][0] != 0 or ranges[-1][1] != dim_size or any(
        a[1] != b[0] for a, b in zip(ranges, ranges[1:])
    ):
        raise ValueError("ranges must be world contiguous ranges covering [0, dim_size)")
    lo, hi = ranges[rank]
    keep = (dst >= lo) & (dst < hi)
    edges = keep.nonzero().view(-1)
    rel_rows = flat_src.index_select(0, edges)
    local_dst = dst.index_select(0, edges) - lo
    local_src = torch.arange(edges.numel(), dtype=torch.int64, device=dst.device)
    return DestinationShard(rank, world, lo, hi, edges, rel_rows, local_src, local_dst)


def gather_output(parts: list[torch.Tensor]) -> torch.Tensor:
    """Full fan-in output from the ranks' outputs (rank order)."""

    return torch.cat(parts, dim=0)
