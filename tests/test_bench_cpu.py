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


def test_lgan_workload_and_bytes():
    """The synthetic LGAN batch has the documented structure, and its byte count
    adds the parts of lgan_pool_reduce and its backward."""

    wl = workloads.lgan(seed=2, entities=300, relations=2000, emb=8)
    R, N, S = wl.relation_count, wl.entity_dim_size, wl.num_slots
    assert torch.equal(torch.bincount(wl.slot_to_rel, minlength=R), wl.arities)
    assert bool((wl.arities >= 1).all()) and bool((wl.arities <= 3).all())
    assert wl.tn_rel.numel() == R and torch.equal(wl.tn_rel, torch.arange(R))
    assert wl.nn_rel.numel() == S - R
    assert wl.rr_src.numel() == 4 * R
    assert int(wl.tn_ent.max()) < N and int(wl.nn_ent.max()) < N
    b = workloads.lgan_algorithmic_bytes(wl)
    rb = 8 * 4
    assert b["lgan_fwd"] > S * rb + 4 * R * rb and b["lgan_bwd"] > S * rb + 6 * R * rb
    assert workloads.lgan_algorithmic_bytes(wl, elem_bytes=2)["lgan_fwd"] < b["lgan_fwd"]


def test_lgan_reference_line_keys(monkeypatch):
    """--impl reference --workload lgan prints the contract's keys (run on a tiny sample)."""

    monkeypatch.setattr(bench, "REF_LIB", bench.ROOT / "oracle" / "_ref" / "missing.so")  # the port: no library load
    orig = workloads.lgan
    monkeypatch.setattr(workloads, "lgan", lambda **kw: orig(**{**kw, "relations": 256, "entities": 64}))
    args = type("A", (), {"gpus": 1, "steps": 1, "warmup": 0})()
    line = bench.lgan_reference_line(args, threads=1)
    for key in ("impl", "metric", "value", "unit", "cpu_baseline", "e2e", "config"):
        assert key in line
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port" and line["value"] > 0
