"""Kernel-path selection on the GPU: every path an op can take gives the
reference's result.

* fanin_reduce_sum_backward with a working set above L2 and a cached forward
  plan copies grad rows through the forward's destination-ordered plan; without
  the forward (no cached plan), or with repeated message rows, it reduces over
  the message-row plan. All three are checked against the index formula
  (copies bit-exact, sums within 1e-5 relative / 1e-6 absolute plus 1e-5 of the
  row's sum of |terms|).
* Packed row shapes (rows of 16..256 bytes, several rows per warp load) and the
  one-row-per-load shapes around them, for every storage type.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200.ops import mp
from tests._oracle_blocks import close_violations, col64, run_blocks

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _load_library():
    assert mp.available(), "relm_mp library not loadable"


def _big_fanin(seed=0, rows=1 << 20, edges=1 << 22, emb=32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dst = torch.randint(0, rows, (edges,), device="cuda", generator=g)
    flat_src = torch.randperm(edges, device="cuda", generator=g)
    grad = torch.randn(rows, emb, device="cuda", generator=g)
    return dst, flat_src, grad


def test_sum_backward_scatter_path_after_forward():
    ops = torch.ops.relm_mp
    dst, flat_src, grad = _big_fanin()
    rel = torch.randn(flat_src.numel(), grad.size(1), device="cuda")
    mp.clear_plan_cache()
    cold = ops.fanin_reduce_sum_backward(grad, flat_src, dst, rel.size(0))  # no forward plan: gather path
    ops.fanin_reduce(rel, flat_src, dst, grad.size(0), 0)  # caches the destination-ordered plan
    warm = ops.fanin_reduce_sum_backward(grad, flat_src, dst, rel.size(0))
    expect = torch.empty_like(rel)
    expect[flat_src] = grad[dst]
    assert torch.equal(cold, expect)
    assert torch.equal(warm, expect)


def test_sum_backward_repeated_message_rows_reduce():
    ops = torch.ops.relm_mp
    dst, _, grad = _big_fanin(seed=1)
    rel_rows = dst.numel() // 2
    flat_src = torch.randint(0, rel_rows, dst.shape, device="cuda")
    rel = torch.randn(rel_rows, grad.size(1), device="cuda")
    mp.clear_plan_cache()
    ops.fanin_reduce(rel, flat_src, dst, grad.size(0), 0)
    got = ops.fanin_reduce_sum_backward(grad, flat_src, dst, rel_rows)
    terms = grad.index_select(0, dst)
    expect = torch.zeros_like(rel).index_add_(0, flat_src, terms)
    row_abs = torch.zeros_like(rel).index_add_(0, flat_src, terms.abs())
    assert bool(((got - expect).abs() <= 1e-6 + 1e-5 * expect.abs() + 1e-5 * row_abs).all())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("row_bytes", [16, 32, 48, 64, 128, 256, 272, 512])
def test_row_map_and_scatter_shapes(dtype, row_bytes):
    """Each gathered row used once (row map), fan-out through the source plan
    (scatter), and their logsumexp / backward forms, around the packed sizes."""

    ops = torch.ops.relm_mp
    es = torch.empty((), dtype=dtype).element_size()
    emb = row_bytes // es
    g = torch.Generator(device="cuda").manual_seed(row_bytes)
    n, e = 3000, 5000
    x = torch.randn(n, emb, device="cuda", generator=g).to(dtype)
    src = torch.randint(0, n, (e,), device="cuda", generator=g)
    flat_dst = torch.randperm(e, device="cuda", generator=g)
    out = ops.fanout_scatter(x, src, flat_dst, e + 7)
    expect = torch.zeros(e + 7, emb, device="cuda", dtype=dtype)
    expect[flat_dst] = x[src]
    assert torch.equal(out, expect)
    # one message per destination row: the row map serves fan-in and both backwards
    rel = torch.randn(e, emb, device="cuda", generator=g).to(dtype)
    dst = torch.randperm(e + 7, device="cuda", generator=g)[:e]
    flat_src = torch.randperm(e, device="cuda", generator=g)
    s = ops.fanin_reduce(rel, flat_src, dst, e + 7, 0)
    s_expect = torch.zeros(e + 7, emb, device="cuda", dtype=dtype)
    s_expect[dst] = rel[flat_src]
    assert torch.equal(s, s_expect)
    lse = ops.fanin_reduce(rel, flat_src, dst, e + 7, 1)
    lse_expect = torch.full((e + 7, emb), float("-inf"), device="cuda", dtype=dtype)
    lse_expect[dst] = rel[flat_src]
    assert torch.equal(lse, lse_expect)
    gout = torch.randn(e + 7, emb, device="cuda", generator=g).to(dtype)
    gb = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, e)
    gb_expect = torch.zeros(e, emb, device="cuda", dtype=torch.float64)
    gb_expect[flat_src] = gout[dst].double() * torch.exp(rel[flat_src].double() - lse[dst].double())
    tol = dict(rtol=1e-2, atol=1e-2) if es == 2 else dict(rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gb.double(), gb_expect, **tol)


@pytest.mark.parametrize("extra_rows", [0, 100])
def test_identity_message_index_plans(extra_rows):
    """flat_src = arange (the usual message-row index) builds its plan without a
    sort or segment scan; message rows past the edges get zero gradient."""

    ops = torch.ops.relm_mp
    g = torch.Generator(device="cuda").manual_seed(7)
    e, n, d = 70000, 3000, 24
    rel_rows = e + extra_rows
    rel = torch.randn(rel_rows, d, device="cuda", generator=g)
    flat_src = torch.arange(e, device="cuda")
    dst = torch.randint(0, n, (e,), device="cuda", generator=g)
    gout = torch.randn(n, d, device="cuda", generator=g)
    mp.clear_plan_cache()
    gs = ops.fanin_reduce_sum_backward(gout, flat_src, dst, rel_rows)
    expect = torch.zeros(rel_rows, d, device="cuda")
    expect[:e] = gout[dst]
    assert torch.equal(gs, expect)
    lse = ops.fanin_reduce(rel, flat_src, dst, n, 1)
    gl = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, rel_rows)
    expect_l = torch.zeros(rel_rows, d, device="cuda", dtype=torch.float64)
    expect_l[:e] = gout[dst].double() * torch.exp(rel[:e].double() - lse[dst].double())
    torch.testing.assert_close(gl.double(), expect_l, rtol=1e-5, atol=1e-6)


def _oracle_lse_backward(gout, rel, flat_src, dst, lse, rel_rows, emb):
    """float64 oracle of the logsumexp backward on the op's own inputs."""

    g64 = gout.float().cpu().numpy()
    r64 = rel.float().cpu().numpy()
    o64 = lse.float().cpu().numpy()
    fs, d = flat_src.cpu().numpy(), dst.cpu().numpy()
    blocks: dict[tuple[int, int], np.ndarray] = {}

    def work(c0: int, c1: int):
        blocks[(c0, c1)] = oracle.fanin_reduce_logsumexp_backward(
            col64(g64, c0, c1), col64(r64, c0, c1), fs, d, col64(o64, c0, c1), rel_rows
        )
        return None

    run_blocks(work, emb, 8, rel_rows)
    return blocks


@pytest.mark.parametrize("dtype,emb", [(torch.float32, 32), (torch.bfloat16, 64)])
def test_lse_backward_destination_order_path(dtype, emb):
    """Above the L2 working set, with the forward's plan cached and message rows
    used once, the logsumexp backward walks the forward's plan in destination
    order; without the cached plan it runs per message row. Both against the
    float64 oracle on the same inputs (message rows no edge uses get 0)."""

    ops = torch.ops.relm_mp
    g = torch.Generator(device="cuda").manual_seed(11)
    rows, edges = 1 << 20, 1 << 22
    dst = torch.randint(0, rows, (edges,), device="cuda", generator=g)
    flat_src = torch.randperm(edges + 1000, device="cuda", generator=g)[:edges]  # some message rows unused
    rel = torch.randn(edges + 1000, emb, device="cuda", generator=g).to(dtype)
    gout = torch.randn(rows, emb, device="cuda", generator=g).to(dtype)
    mp.clear_plan_cache()
    lse = ops.fanin_reduce(rel, flat_src, dst, rows, 1)  # caches the destination-ordered plan
    warm = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, rel.size(0)).float().cpu().numpy()
    mp.clear_plan_cache()
    cold = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, rel.size(0)).float().cpu().numpy()
    ref = _oracle_lse_backward(gout, rel, flat_src, dst, lse, rel.size(0), emb)
    rtol, atol = (1e-2, 1e-3) if dtype == torch.bfloat16 else (1e-5, 1e-6)
    for (c0, c1), want in ref.items():
        for name, got in (("warm", warm), ("cold", cold)):
            f = close_violations(got[:, c0:c1], want, rtol, atol)
            assert f is None, f"{name} cols {c0}:{c1}: {f}"


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("n", [9999, 10000])
def test_validation_paths_aligned_and_offset_indices(offset, n):
    """Index validation reads two edges per thread from 16-byte aligned index
    tensors and one per thread otherwise (a view starting at an odd element);
    both give the same plans, and the same first offending edge."""

    ops = torch.ops.relm_mp
    g = torch.Generator(device="cuda").manual_seed(n + offset)
    base_dst = torch.randint(0, 500, (n + 1,), device="cuda", generator=g)
    base_src = torch.randperm(n + 1, device="cuda", generator=g)
    dst, src = base_dst[offset : offset + n], base_src[offset : offset + n] % n
    rel = torch.randn(n, 8, device="cuda", generator=g)
    mp.clear_plan_cache()
    a = ops.fanin_reduce(rel, src, dst, 500, 0)
    mp.clear_plan_cache()
    b = ops.fanin_reduce(rel, src.clone(), dst.clone(), 500, 0)
    assert torch.equal(a, b)
    bad = dst.clone()
    bad[n - 2] = 777  # odd or even position depending on n
    bad[n - 1] = -3
    with pytest.raises(RuntimeError, match="dst_idx index out of bounds: 777 not in"):
        ops.fanin_reduce(rel, src, bad, 500, 0)


def test_large_backwards_with_unpacked_rows():
    """Above the working set with 192-byte rows (not a power of two times 16):
    the sum backward scatters through the general scatter kernel and the
    logsumexp backward falls back to the per-message-row path; both, with and
    without a cached forward plan, against the float64 oracle."""

    ops = torch.ops.relm_mp
    g = torch.Generator(device="cuda").manual_seed(21)
    rows, edges, emb = 1 << 19, 1 << 21, 48
    dst = torch.randint(0, rows, (edges,), device="cuda", generator=g)
    flat_src = torch.randperm(edges, device="cuda", generator=g)
    rel = torch.randn(edges, emb, device="cuda", generator=g)
    gout = torch.randn(rows, emb, device="cuda", generator=g)
    mp.clear_plan_cache()
    lse = ops.fanin_reduce(rel, flat_src, dst, rows, 1)
    got = {"warm_s": ops.fanin_reduce_sum_backward(gout, flat_src, dst, edges),
           "warm_l": ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, edges)}
    mp.clear_plan_cache()
    got["cold_s"] = ops.fanin_reduce_sum_backward(gout, flat_src, dst, edges)
    got["cold_l"] = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, edges)
    got = {k: v.cpu().numpy() for k, v in got.items()}
    # flat_src is a permutation: the sum backward copies one grad row per message row
    ref_s = oracle.fanin_reduce_sum_backward(gout.cpu().numpy(), flat_src.cpu().numpy(), dst.cpu().numpy(), edges)
    assert np.array_equal(got["warm_s"], ref_s) and np.array_equal(got["cold_s"], ref_s)
    ref_l = _oracle_lse_backward(gout, rel, flat_src, dst, lse, edges, emb)
    for (c0, c1), want in ref_l.items():
        for name in ("warm_l", "cold_l"):
            f = close_violations(got[name][:, c0:c1], want, 1e-5, 1e-6)
            assert f is None, f"{name} cols {c0}:{c1}: {f}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("row_bytes", [16, 64, 256])
@pytest.mark.parametrize("longest", [32, 33])
def test_short_and_long_row_plans(dtype, row_bytes, longest):
    """Plans whose rows hold at most 32 edges are reduced a lane group per row
    (k_seg_rows_packed); one longer row switches the plan to the merge-path
    kernels (device flag [1] of the plan). Both give the reference sums,
    logsumexp, both backwards and the fused sum epilogue."""

    from relmo_b200 import capi

    ops = torch.ops.relm_mp
    es = torch.empty((), dtype=dtype).element_size()
    emb = row_bytes // es
    g = torch.Generator(device="cuda").manual_seed(longest * 1000 + row_bytes)
    rows = 3000
    deg = torch.randint(0, 9, (rows,), device="cuda", generator=g)
    deg[17] = longest
    dst = torch.repeat_interleave(torch.arange(rows, device="cuda"), deg)
    dst = dst[torch.randperm(dst.numel(), device="cuda", generator=g)]
    e = dst.numel()
    flat_src = torch.randperm(e, device="cuda", generator=g)
    rel = torch.randn(e, emb, device="cuda", generator=g).to(dtype)
    plan = capi.PlanHandle(dst, flat_src, rows, e)
    flags = capi._device_int32(plan.plan.device_flags, 4, torch.device("cuda")).cpu()
    assert int(flags[0]) == 1 and int(flags[1]) == int(longest > 32)
    tol = dict(rtol=1e-2, atol=1e-2) if es == 2 else dict(rtol=1e-5, atol=1e-5)
    r64 = rel.double()
    s = ops.fanin_reduce(rel, flat_src, dst, rows, 0)
    expect = torch.zeros(rows, emb, dtype=torch.float64, device="cuda").index_add_(0, dst, r64[flat_src])
    torch.testing.assert_close(s.double(), expect, **tol)
    lse = ops.fanin_reduce(rel, flat_src, dst, rows, 1)
    m = torch.full((rows, emb), float("-inf"), dtype=torch.float64, device="cuda")
    m = m.scatter_reduce(0, dst[:, None].expand(-1, emb), r64[flat_src], "amax")
    ex = torch.zeros(rows, emb, dtype=torch.float64, device="cuda").index_add_(0, dst, (r64[flat_src] - m[dst]).exp())
    expect_lse = ex.log() + m
    torch.testing.assert_close(lse.double(), expect_lse, equal_nan=True, **tol)
    gout = torch.randn(rows, emb, device="cuda", generator=g).to(dtype)
    gl = ops.fanin_reduce_logsumexp_backward(gout, rel, flat_src, dst, lse, e)
    expect_gl = torch.zeros(e, emb, dtype=torch.float64, device="cuda")
    expect_gl[flat_src] = gout.double()[dst] * (r64[flat_src] - lse.double()[dst]).exp()
    torch.testing.assert_close(gl.double(), expect_gl, **tol)
    # the source-side plan of a fan-out backward has the same row lengths
    gs = ops.fanout_scatter_backward(rel, dst, flat_src, rows)
    torch.testing.assert_close(gs.double(), expect, **tol)
    base = torch.randn(rows, emb, device="cuda", generator=g).to(dtype)
    got = plan.reduce_ex(rel, base=base, divide_by_count=True)
    cnt = torch.bincount(dst, minlength=rows).double().clamp_min(1.0)[:, None]
    torch.testing.assert_close(got.double(), expect / cnt + base.double(), **tol)


@pytest.mark.parametrize("kind", ["one_edge", "short", "long"])
@pytest.mark.parametrize("emb", [64, 3])
def test_known_plan_flags_launch_one_family(kind, emb):
    """With the plan's flags copied to the host (relm_mp_plan_read_flags; the
    torch layer does it without a sync once the copy after the build landed),
    a planned reduction launches only the kernel family the plan needs - with
    bit-identical results."""

    from relmo_b200 import capi

    g = torch.Generator(device="cuda").manual_seed(len(kind) * 10 + emb)
    rows = 4000
    if kind == "one_edge":
        out_idx = torch.randperm(rows, device="cuda", generator=g)[:3000]
    else:
        deg = torch.randint(0, 6, (rows,), device="cuda", generator=g)
        deg[5] = 40 if kind == "long" else 6
        out_idx = torch.repeat_interleave(torch.arange(rows, device="cuda"), deg)
        out_idx = out_idx[torch.randperm(out_idx.numel(), device="cuda", generator=g)]
    e = out_idx.numel()
    gather = torch.randint(0, 5000, (e,), device="cuda", generator=g)
    table = torch.randn(5000, emb, device="cuda", generator=g)
    plan = capi.PlanHandle(out_idx, gather, rows, 5000)
    launches = capi.lib().relm_mp_kernel_launches
    results = []
    counts = []
    for known in (False, True):
        if known:
            flags = plan.read_flags()
            assert flags & 2
            assert bool(flags & 4) == (kind != "one_edge")
            assert bool(flags & 8) == (kind == "long")
        n0 = launches()
        res = [plan.reduce(table, 0), plan.reduce(table, 1), plan.reduce_ex(table, base=table[:rows].contiguous(),
                                                                         divide_by_count=True)]
        torch.cuda.synchronize()
        counts.append(launches() - n0)
        results.append(res)
    for a, b in zip(*results):
        assert torch.equal(a.isnan(), b.isnan()) and torch.equal(torch.nan_to_num(a), torch.nan_to_num(b))
    assert counts[1] < counts[0]


def test_coverage_pass_keeps_plan_row_flags():
    """The fan-out's coverage pass works in a spare device flag word: the plan's
    row facts (repeats, long rows) survive it, so a fan-out backward over the
    same (shared, cached) plan with long source rows runs the merge-path
    kernels and gives the reference sums - on the first call and on later
    calls, when the host knows the plan's flags."""

    from relmo_b200 import capi

    ops = torch.ops.relm_mp
    g = torch.Generator(device="cuda").manual_seed(77)
    n, e, emb = 2000, 30000, 64
    src = torch.randint(0, n, (e,), device="cuda", generator=g)
    src[:50] = 3  # one source row with 50+ slots: a long row
    flat_dst = torch.randperm(e, device="cuda", generator=g)
    x = torch.randn(n, emb, device="cuda", generator=g)
    grad = torch.randn(e, emb, device="cuda", generator=g)
    expect = torch.zeros(n, emb, dtype=torch.float64, device="cuda").index_add_(0, src, grad.double()[flat_dst])
    for _ in range(3):
        out = ops.fanout_scatter(x, src, flat_dst, e)  # coverage of the source plan
        assert torch.equal(out[flat_dst], x[src])
        gx = ops.fanout_scatter_backward(grad, src, flat_dst, n)
        torch.testing.assert_close(gx.double(), expect, rtol=1e-5, atol=1e-4)
    plan = capi.PlanHandle(src, flat_dst, n, e)
    before = capi._device_int32(plan.plan.device_flags, 3, torch.device("cuda")).cpu().tolist()
    cover, dups = plan.gather_cover()
    after = capi._device_int32(plan.plan.device_flags, 3, torch.device("cuda")).cpu().tolist()
    assert not dups and before == after and before[0] == 1 and before[1] == 1


@pytest.mark.parametrize("gather_rows,edges,repeat", [(1000, 1000, False), (1000, 999, True), (70001, 50000, False),
                                                      (70001, 50000, True), (33, 0, False), (5, 40, True)])
def test_gather_coverage_paths_agree(gather_rows, edges, repeat):
    """The coverage of a plan's gather index three ways: L2 atomics
    (relm_mp_plan_gather_cover), byte marks packed into the bitmap
    (relm_mp_plan_gather_cover_ex), and marks written by the build's
    validation pass (relm_mp_plan_build_cover). Same bitmap, same repeat flag,
    and both equal to the index's own content; the plans themselves equal the
    plain build's."""

    from relmo_b200 import capi

    g = torch.Generator(device="cuda").manual_seed(gather_rows + edges)
    rows = 300
    out_index = torch.randint(0, rows, (edges,), device="cuda", generator=g)
    if repeat:
        gather = torch.randint(0, gather_rows, (edges,), device="cuda", generator=g)
        if edges > 1:
            gather[-1] = gather[0]
    else:
        gather = torch.randperm(gather_rows, device="cuda", generator=g)[:edges]
    plain = capi.PlanHandle(out_index, gather, rows, gather_rows)
    cover_a, dups_a = plain.gather_cover()
    cover_b, dups_b = plain.gather_cover_ex()
    built = capi.PlanHandle(out_index, gather, rows, gather_rows, with_cover=True)
    assert torch.equal(cover_a, cover_b) and torch.equal(cover_a, built.cover)
    assert dups_a == dups_b == built.repeats == (edges > 0 and gather.unique().numel() < edges)
    expect = torch.zeros(max(1, (gather_rows + 31) // 32 * 32), dtype=torch.bool, device="cuda")
    expect[gather] = True
    bits = torch.tensor([1 << k for k in range(32)], dtype=torch.int64, device="cuda")
    words = (expect.view(-1, 32).long() * bits).sum(dim=1)
    assert torch.equal(cover_a.long() & 0xFFFFFFFF, words)
    assert plain.covered == built.covered == int(gather.unique().numel())
    assert torch.equal(plain.row_ptr(), built.row_ptr()) and torch.equal(plain.gidx(), built.gidx())
