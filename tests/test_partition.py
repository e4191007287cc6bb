"""Destination-range partition of the fan-in (the op-level multi-GPU layout).

The concatenation of the ranks' outputs must equal the unpartitioned fan-in,
and each rank's message-row gradients must equal the unpartitioned gradients
at its rows, for sum and logsumexp. CPU: ranks emulated in one process and as
two gloo processes (the host logic; outputs through the ops' CPU formulas).
GPU: ranks emulated on one device through the B200 kernels, fp32 tolerance
1e-5 relative / 1e-6 absolute (per-row summation order follows the tiling).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as tmp

from relmo_b200 import partition, workloads
from relmo_b200.ops import mp


def test_destination_ranges_cover_rows():
    for n, w in [(0, 1), (5, 2), (7, 3), (2, 4), (1 << 22, 8)]:
        r = partition.destination_ranges(n, w)
        assert len(r) == w and r[0][0] == 0 and r[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        sizes = [hi - lo for lo, hi in r]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        partition.destination_ranges(4, 0)


def test_balanced_ranges_split_work():
    wl = _problem()
    for world in (1, 2, 3, 8):
        r = partition.balanced_destination_ranges(wl.dst, wl.dim_size, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == wl.dim_size
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        deg = torch.bincount(wl.dst, minlength=wl.dim_size)
        work = [int(hi - lo + deg[lo:hi].sum()) for lo, hi in r]
        total = wl.dim_size + wl.dst.numel()
        # a boundary can only miss its target by the work of one row
        assert max(work) <= total / world + int(deg.max()) + 1
    with pytest.raises(ValueError):
        partition.shard_by_destination(wl.flat_src, wl.dst, wl.dim_size, 0, 2, [(0, 5), (6, wl.dim_size)])


def test_shard_rejects_bad_arguments():
    i = torch.arange(4)
    with pytest.raises(ValueError):
        partition.shard_by_destination(i, i[:3], 4, 0, 2)
    with pytest.raises(ValueError):
        partition.shard_by_destination(i, i, 4, 2, 2)


def _problem(device="cpu", seed=0):
    wl = workloads.cfg5(seed=seed, device=device, n=4096, edges=60000, emb=16, hubs=4, per_hub=3000)
    return wl


def _full(wl, mode):
    rel = wl.msgs.detach().clone().requires_grad_(True)
    out = mp.fanin_reduce(rel, wl.flat_src, wl.dst, wl.dim_size, mode)
    (out * wl.grad_nodes).sum().backward()
    return out.detach(), rel.grad


def _sharded(wl, mode, world, balanced=False):
    outs = []
    grad = torch.zeros_like(wl.msgs)
    ranges = partition.balanced_destination_ranges(wl.dst, wl.dim_size, world) if balanced else None
    for r in range(world):
        sh = partition.shard_by_destination(wl.flat_src, wl.dst, wl.dim_size, r, world, ranges)
        rel = wl.msgs.index_select(0, sh.rel_rows).requires_grad_(True)
        out = mp.fanin_reduce(rel, sh.flat_src, sh.dst, sh.dim_size, mode)
        (out * wl.grad_nodes[sh.row_lo : sh.row_hi]).sum().backward()
        outs.append(out.detach())
        grad.index_copy_(0, sh.rel_rows, rel.grad)
    return partition.gather_output(outs), grad


@pytest.mark.parametrize("balanced", [False, True])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("world", [1, 3, 8])
def test_partition_equals_full_cpu(mode, world, balanced):
    wl = _problem()
    out, grad = _full(wl, mode)
    pout, pgrad = _sharded(wl, mode, world, balanced)
    torch.testing.assert_close(pout, out, rtol=1e-5, atol=1e-6, equal_nan=True)
    torch.testing.assert_close(pgrad, grad, rtol=1e-5, atol=1e-6)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, out_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = _problem()
        sh = partition.shard_by_destination(wl.flat_src, wl.dst, wl.dim_size, rank, world)
        rel = wl.msgs.index_select(0, sh.rel_rows)
        out = mp.fanin_reduce(rel, sh.flat_src, sh.dst, sh.dim_size, 1)
        parts = [None] * world
        dist.all_gather_object(parts, out)  # validation only: the data path has no exchange
        if rank == 0:
            torch.save(partition.gather_output(parts), out_path)
    finally:
        dist.destroy_process_group()


def test_partition_gloo_two_ranks(tmp_path):
    path = tmp_path / "out.pt"
    tmp.spawn(_gloo_worker, args=(2, _free_port(), str(path)), nprocs=2, join=True)
    wl = _problem()
    full, _ = _full(wl, 1)
    torch.testing.assert_close(torch.load(path), full, rtol=1e-5, atol=1e-6, equal_nan=True)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1])
def test_partition_equals_full_gpu(mode):
    """Sums may differ by the reordering of a row's terms: 1e-5 of the sum of
    |terms| of the row on top of 1e-5 relative / 1e-6 absolute."""

    assert mp.available()
    wl = _problem(device="cuda")
    out, grad = _full(wl, mode)
    pout, pgrad = _sharded(wl, mode, 8, balanced=True)
    if mode == 0:
        row_abs = torch.zeros_like(out).index_add_(0, wl.dst, wl.msgs.abs().index_select(0, wl.flat_src))
        assert bool(((pout - out).abs() <= 1e-6 + 1e-5 * out.abs() + 1e-5 * row_abs).all())
        assert torch.equal(pgrad, grad)  # copies of grad rows
    else:
        torch.testing.assert_close(pout, out, rtol=1e-5, atol=1e-6, equal_nan=True)
        torch.testing.assert_close(pgrad, grad, rtol=1e-5, atol=1e-6)
