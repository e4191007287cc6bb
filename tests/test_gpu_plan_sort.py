"""Plan layout on the GPU against numpy: the plan's gathered-row order is the
stable sort of the edges by output row (edge order kept within a row), and
row_ptr[r] is the number of edges with output row < r.

The cases reach every sort shape of the plan build: one radix pass (up to 11
key bits), two passes of 10 and 11 bits (cfg2's 2^20 rows, cfg5's 2^22), three
passes (2^23 and more rows), sub-tile and CTA boundaries of the sort (8192
items per sub-tile), one hot row holding most edges (Zipf), all edges in one
row, reversed and already sorted output indices, and the identity.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from relmo_b200 import capi
from relmo_b200.ops import mp

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _load_library():
    assert mp.available(), "relm_mp library not loadable"


def _expect(out_index: np.ndarray, gather: np.ndarray, rows: int):
    order = np.argsort(out_index, kind="stable")
    gidx = gather[order]
    row_ptr = np.searchsorted(out_index[order], np.arange(rows + 1), side="left")
    return gidx, row_ptr


def _check(out_index: torch.Tensor, gather: torch.Tensor | None, rows: int, gather_rows: int):
    plan = capi.PlanHandle(out_index.cuda(), None if gather is None else gather.cuda(), rows, gather_rows)
    torch.cuda.synchronize()
    o = out_index.numpy()
    g = np.arange(o.size) if gather is None else gather.numpy()
    want_gidx, want_ptr = _expect(o, g, rows)
    assert np.array_equal(plan.row_ptr().numpy(), want_ptr)
    assert np.array_equal(plan.gidx().numpy(), want_gidx)


def _zipf(rows: int, edges: int, gen: torch.Generator, alpha: float = 1.3) -> torch.Tensor:
    ranks = torch.arange(1, rows + 1, dtype=torch.float64)
    w = ranks.pow(-alpha)
    pick = torch.multinomial(w, edges, replacement=True, generator=gen)
    perm = torch.randperm(rows, generator=gen)
    return perm[pick]


CASES = [
    # (rows, edges, kind)
    (1, 1000, "uniform"),
    (2, 8191, "uniform"),
    (3, 8193, "uniform"),
    (100, 100_000, "uniform"),
    (2047, 70_000, "uniform"),
    (2048, 16_384, "uniform"),
    (2049, 300_000, "zipf"),
    (1 << 20, 1 << 21, "zipf"),
    (1 << 20, 3_000_001, "uniform"),
    ((1 << 22) + 5, 1 << 21, "uniform"),
    ((1 << 23) + 1, 1 << 20, "uniform"),
    (1 << 20, 1 << 20, "reversed"),
    (5000, 1 << 20, "one_row"),
    (1 << 16, 1 << 20, "sorted_runs"),
]


@pytest.mark.parametrize("rows,edges,kind", CASES)
def test_plan_matches_stable_sort(rows: int, edges: int, kind: str) -> None:
    gen = torch.Generator().manual_seed(rows * 31 + edges)
    if kind == "uniform":
        out = torch.randint(0, rows, (edges,), generator=gen)
    elif kind == "zipf":
        out = _zipf(rows, edges, gen)
    elif kind == "reversed":
        out = torch.arange(edges - 1, -1, -1) % rows
    elif kind == "one_row":
        out = torch.full((edges,), rows // 2, dtype=torch.int64)
        out[:: 997] = torch.randint(0, rows, (out[:: 997].numel(),), generator=gen)
    else:  # runs of equal rows in order, then a few out of order
        out = torch.sort(torch.randint(0, rows, (edges,), generator=gen)).values
        out[-10:] = torch.randint(0, rows, (10,), generator=gen)
    gather_rows = edges + 7
    gather = torch.randint(0, gather_rows, (edges,), generator=gen)
    _check(out, gather, rows, gather_rows)


def test_identity_gather_and_already_sorted() -> None:
    gen = torch.Generator().manual_seed(5)
    out = torch.sort(torch.randint(0, 1 << 18, (1 << 20,), generator=gen)).values
    _check(out, None, 1 << 18, 1 << 20)
    _check(torch.arange(1 << 20), None, 1 << 20, 1 << 20)


def test_split_build_shares_one_wait_and_reports_the_first_error() -> None:
    """relm_mp_plan_build_start / _finish through the C ABI: three builds
    started back to back, one stream wait, then finished in order, give the
    plans of three separate builds; a bad index in the second pair raises that
    pair's message at its finish."""

    import ctypes

    lib = capi.lib()
    gen = torch.Generator().manual_seed(11)
    dev = torch.device("cuda")
    stream = capi._stream(dev)
    pairs = [
        (torch.randint(0, 5000, (70_000,), generator=gen), torch.randint(0, 9000, (70_000,), generator=gen), 5000, 9000),
        (torch.randint(0, 1 << 20, (1 << 20,), generator=gen), torch.randint(0, 300, (1 << 20,), generator=gen), 1 << 20, 300),
        (torch.randint(0, 77, (1000,), generator=gen), torch.randint(0, 10, (1000,), generator=gen), 77, 10),
    ]

    def run(pairs):
        held = []
        for out_i, gat_i, rows, grows in pairs:
            o, g = out_i.to(dev), gat_i.to(dev)
            e = o.numel()
            mem = capi._workspace(lib.relm_mp_plan_bytes(e, rows), dev)
            scr = capi._workspace(lib.relm_mp_plan_scratch_bytes(e, rows), dev)
            stats = torch.empty(lib.relm_mp_plan_stats_bytes(), dtype=torch.uint8).pin_memory()
            capi.check(lib.relm_mp_plan_build_start(o.data_ptr(), g.data_ptr(), e, rows, rows, grows, mem.data_ptr(),
                                                    mem.numel(), scr.data_ptr(), scr.numel(), stats.data_ptr(), stream))
            held.append((o, g, e, rows, grows, mem, scr, stats))
        torch.cuda.synchronize()
        plans = []
        for o, g, e, rows, grows, mem, scr, stats in held:
            plan = capi.Plan()
            capi.check(lib.relm_mp_plan_build_finish(o.data_ptr(), g.data_ptr(), e, rows, rows, grows, b"out_i", b"gat_i",
                                                     0, mem.data_ptr(), mem.numel(), scr.data_ptr(), scr.numel(),
                                                     stats.data_ptr(), stream, ctypes.byref(plan)))
            plans.append((plan, mem))
        return plans

    for (out_i, gat_i, rows, grows), (plan, _mem) in zip(pairs, run(pairs)):
        want_gidx, want_ptr = _expect(out_i.numpy(), gat_i.numpy(), rows)
        got_ptr = capi._device_int32(plan.row_ptr, rows + 1, dev).cpu().numpy()
        got_gidx = capi._device_int32(plan.gidx, out_i.numel(), dev).cpu().numpy()
        assert np.array_equal(got_ptr, want_ptr)
        assert np.array_equal(got_gidx, want_gidx)

    bad = list(pairs)
    broken = pairs[1][1].clone()
    broken[12345] = 300  # gathered row out of [0, 300)
    bad[1] = (pairs[1][0], broken, pairs[1][2], pairs[1][3])
    with pytest.raises(capi.RelmMpError, match=r"gat_i index out of bounds: 300 not in \[0, 300\)"):
        run(bad)


@pytest.mark.parametrize("rows, gather_rows, edges", [(5000, 9000, 70_000), (1 << 20, 300, 1 << 20), (77, 10, 1000),
                                                      (1 << 17, 1 << 20, 1 << 22)])
def test_trusted_build_equals_the_checked_build(rows: int, gather_rows: int, edges: int) -> None:
    """relm_mp_plan_build_trusted (no validation, no host wait) lays out the
    same plan as the checked build: the stable sort by output row."""

    import ctypes

    lib = capi.lib()
    gen = torch.Generator().manual_seed(rows + edges)
    dev = torch.device("cuda")
    out_i = torch.randint(0, rows, (edges,), generator=gen)
    gat_i = torch.randint(0, gather_rows, (edges,), generator=gen)
    o, g = out_i.to(dev), gat_i.to(dev)
    mem = capi._workspace(lib.relm_mp_plan_bytes(edges, rows), dev)
    scr = capi._workspace(lib.relm_mp_plan_scratch_bytes(edges, rows), dev)
    plan = capi.Plan()
    capi.check(lib.relm_mp_plan_build_trusted(o.data_ptr(), g.data_ptr(), edges, rows, gather_rows, mem.data_ptr(),
                                              mem.numel(), scr.data_ptr(), scr.numel(), capi._stream(dev),
                                              ctypes.byref(plan)))
    torch.cuda.synchronize()
    want_gidx, want_ptr = _expect(out_i.numpy(), gat_i.numpy(), rows)
    assert np.array_equal(capi._device_int32(plan.row_ptr, rows + 1, dev).cpu().numpy(), want_ptr)
    assert np.array_equal(capi._device_int32(plan.gidx, edges, dev).cpu().numpy(), want_gidx)
    checked = capi.PlanHandle(o, g, rows, gather_rows)
    torch.cuda.synchronize()
    assert np.array_equal(checked.gidx().numpy(), want_gidx)


def test_transposed_pair_reuses_the_forward_validation() -> None:
    """A fan-in sum over (dst, flat_src) with a permuted flat_src, then its
    backward over the transposed pair (flat_src, dst): the backward's plan is
    built without a validation of its own (one build more, no index error
    possible) and gives the oracle's gradient; with a new (unvalidated) dst
    tensor the backward validates and raises on a bad index as before."""

    gen = torch.Generator().manual_seed(3)
    dev = torch.device("cuda")
    n, e, d = 5000, 60_000, 32
    rel = torch.randn(e, d, generator=gen).to(dev)
    flat_src = torch.randperm(e, generator=gen).to(dev)
    dst = torch.randint(0, n, (e,), generator=gen).to(dev)
    g = torch.randn(n, d, generator=gen).to(dev)
    ops = torch.ops.relm_mp
    mp.clear_plan_cache()
    ops.fanin_reduce(rel, flat_src, dst, n, 0)
    before = mp.plan_cache_stats()["builds"]
    grad = ops.fanin_reduce_sum_backward(g, flat_src, dst, e)
    assert mp.plan_cache_stats()["builds"] == before + 1
    want = torch.zeros(e, d, dtype=torch.float64)
    want[flat_src.cpu()] = g.double().cpu()[dst.cpu()]
    torch.testing.assert_close(grad.double().cpu(), want, rtol=0, atol=0)
    bad = dst.clone()
    bad[777] = n
    with pytest.raises(RuntimeError, match=r"index out of bounds"):
        ops.fanin_reduce_sum_backward(g, flat_src, bad, e)
