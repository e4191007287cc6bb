"""bench.py host logic on the CPU: which ops a workload times, the compulsory
byte counts, and that a destination-range partition splits those bytes
exactly (every edge, distinct destination row and output row lands on one
rank), so the partitioned job reports the same total as one GPU would."""

from __future__ import annotations

import pytest
import torch

import bench
from relmo_b200 import workloads


def test_ops_of_workloads():
    assert bench.ops_of("cfg5") == bench.FANIN_OPS
    assert bench.ops_of("cfg2-unsorted") == bench.OPS
    assert set(bench.E2E_ORDER) == set(bench.OPS)
    for op in bench.OPS:
        assert op in bench.OP_INPUTS


def test_algorithmic_bytes_cfg1():
    wl = workloads.cfg1(seed=0)
    b = bench.op_bytes(wl)
    e, d, s = wl.num_edges, wl.emb, 4
    assert b["fanin_sum_fwd"] == e * d * s + 16 * e + wl.dim_size * d * s
    assert b["fanout_bwd"] == e * d * s + 16 * e + wl.x.size(0) * d * s
    ud = int(torch.unique(wl.dst).numel())
    assert b["fanin_lse_bwd"] == 2 * e * d * s + 2 * ud * d * s + 16 * e


@pytest.mark.parametrize("world", [2, 3, 8])
def test_partition_splits_bytes_exactly(world):
    wl = workloads.cfg5(seed=1, n=5000, edges=40000, emb=8, hubs=3, per_hub=2000)
    total = sum(bench.op_bytes(wl, bench.FANIN_OPS).values())
    shards = [bench.shard_workload(wl, r, world) for r in range(world)]
    assert sum(sh.flat_src.numel() for sh in shards) == wl.flat_src.numel()
    assert sum(sh.dim_size for sh in shards) == wl.dim_size
    assert sum(sum(bench.op_bytes(sh, bench.FANIN_OPS).values()) for sh in shards) == total
