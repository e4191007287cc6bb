"""LGAN ops on the B200 (sum / mean): parity with the reference and the oracle.

- Every golden case (the reference's own CPU library on its test fixtures and
  edge cases, tests/golden/ref_lgan.npz) through ``torch.ops.relm_mp.lgan_*``
  and through the C ABI's op-level entry points; out-of-range indices and bad
  modes raise.
- Seeded synthetic LGAN batches against the C oracle in float32, float64,
  bfloat16 and float16, forward and backward, both modes.
- The planned pieces: the fused sum epilogue (base + sum / divisor) over every
  row shape the kernels select (row map, stream, register tiles, long-row
  fixups), in place, the dividing scatter, gather counts and row division.
- The autograd facade against the CPU formulas, and plan reuse.

Tolerances: float32 1e-5 relative / 1e-6 absolute plus 1e-5 of the sum of
|terms| of a row (the GPU sums each row in tile order, the reference in edge
order); float64 1e-10; bfloat16 / float16 against the float32 oracle on the
same (rounded) inputs, 1e-2 relative and absolute plus 1e-2 of the sum of
|terms| (the 2-byte path rounds its intermediate rows to the storage type).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200 import capi, workloads
from relmo_b200.ops import mp
from relmo_b200.ops.mp_lgan import lgan_pool_reduce_python
from tests._golden import load_lgan_cases

pytestmark = pytest.mark.gpu

CASES = load_lgan_cases()


@pytest.fixture(autouse=True, scope="module")
def _loaded():
    assert mp.available(), "relm_mp B200 library must load on a GPU box"
    yield


def _cuda(args):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() if isinstance(a, np.ndarray) else a for a in args]


def _assert_close(got: torch.Tensor, ref, tol_abs_terms=None) -> None:
    ref_t = torch.as_tensor(np.asarray(ref)).to(got.device)
    if got.dtype == torch.float64:
        torch.testing.assert_close(got, ref_t.to(torch.float64), rtol=1e-10, atol=1e-10)
    elif got.dtype in (torch.bfloat16, torch.float16):
        # the 2-byte path rounds its intermediates (x0, x1) to the storage type
        bound = 1e-2 + 1e-2 * ref_t.float().abs()
        if tol_abs_terms is not None:
            bound = bound + 1e-2 * tol_abs_terms
        assert bool(((got.float() - ref_t.float()).abs() <= bound).all()), (got, ref_t)
    else:
        bound = 1e-6 + 1e-5 * ref_t.float().abs()
        if tol_abs_terms is not None:
            bound = bound + 1e-5 * tol_abs_terms
        assert bool(((got.float() - ref_t.float()).abs() <= bound).all()), (got, ref_t)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_torch_ops_match_reference(case) -> None:
    op = getattr(torch.ops.relm_mp, case.op)
    args = _cuda(case.args)
    if case.raises:
        with pytest.raises((RuntimeError, IndexError)):
            op(*args)
            torch.cuda.synchronize()
        return
    out = op(*args)
    outs = out if isinstance(out, (tuple, list)) else (out,)
    assert len(outs) == len(case.outs)
    for g, ref in zip(outs, case.outs):
        assert g.dtype == torch.from_numpy(ref).dtype and tuple(g.shape) == ref.shape
        _assert_close(g, ref)


@pytest.mark.parametrize("case", [c for c in CASES if not c.raises], ids=lambda c: c.name)
def test_c_abi_matches_reference(case) -> None:
    fn = getattr(capi, case.op)
    args = [a.long() if isinstance(a, torch.Tensor) and a.dtype == torch.int32 else a for a in _cuda(case.args)]
    out = fn(*args)
    outs = out if isinstance(out, (tuple, list)) else (out,)
    for g, ref in zip(outs, case.outs):
        _assert_close(g, ref)


def test_c_abi_errors() -> None:
    x = torch.randn(3, 2, device="cuda")
    e = torch.zeros(0, dtype=torch.long, device="cuda")
    bad = torch.tensor([5], device="cuda")
    with pytest.raises(capi.RelmMpError, match="tn_ent index out of bounds: 5 not in \\[0, 5\\)"):
        capi.lgan_relation_graph_step(x, e, e, torch.tensor([0], device="cuda"), bad, e, e, 5, 0)
    with pytest.raises(capi.RelmMpError, match="supports only mode 0=sum or 2=mean"):
        capi.lgan_relation_graph_step(x, e, e, e, e, e, e, 5, 1)


def _row_abs(wl, mode_mean: bool):
    """Per-output bound term: the row sums of |terms| of the float64 formulas."""

    a = wl.to("cpu", torch.float64)
    absw = workloads.LganWorkload(a.name, a.slots.abs(), a.slot_to_rel, a.arities, *a.graph(), a.entity_dim_size,
                                  a.grad_x.abs(), a.grad_tn.abs(), a.grad_nn.abs())
    mode = 2 if mode_mean else 0
    fwd = lgan_pool_reduce_python(absw.slots, absw.slot_to_rel, absw.arities, *absw.graph(), absw.entity_dim_size,
                                  mode)
    bwd = oracle.lgan_pool_reduce_backward(absw.grad_x.numpy(), absw.grad_tn.numpy(), absw.grad_nn.numpy(),
                                           absw.slot_to_rel, absw.arities, *absw.graph(), absw.relation_count, mode)
    return [f.float().cuda() for f in fwd], torch.from_numpy(bwd).float().cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("emb", [64, 24])
def test_synthetic_batch_matches_oracle(dtype, mode, emb) -> None:
    wl = workloads.lgan(seed=7, entities=3000, relations=20000, emb=emb).to("cuda", dtype)
    ops = torch.ops.relm_mp
    outs = ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
    grad = ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities, *wl.graph(),
                                         wl.relation_count, mode)
    odt = np.float64 if dtype == torch.float64 else np.float32
    cpu = [t.cpu().to(torch.float64 if dtype == torch.float64 else torch.float32).numpy().astype(odt)
           for t in (wl.slots, wl.grad_x, wl.grad_tn, wl.grad_nn)]
    graph = [t.cpu() for t in wl.graph()]
    ref = oracle.lgan_pool_reduce(cpu[0], wl.slot_to_rel.cpu(), wl.arities.cpu(), *graph, wl.entity_dim_size, mode)
    ref_g = oracle.lgan_pool_reduce_backward(cpu[1], cpu[2], cpu[3], wl.slot_to_rel.cpu(), wl.arities.cpu(), *graph,
                                             wl.relation_count, mode)
    fwd_abs, bwd_abs = _row_abs(wl, mode == 2) if dtype != torch.float64 else ([None] * 3, None)
    for g, r, a in zip(outs, ref, fwd_abs):
        _assert_close(g, r, a)
    _assert_close(grad, ref_g, bwd_abs)
    # the op-level C ABI gives the same numbers
    c_outs = capi.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
    c_grad = capi.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                            *wl.graph(), wl.relation_count, mode)
    for a, b in zip(c_outs, outs):
        assert torch.equal(a, b)
    assert torch.equal(c_grad, grad)


@pytest.mark.parametrize("mode", [0, 2])
def test_graph_step_matches_oracle(mode) -> None:
    wl = workloads.lgan(seed=3, entities=2000, relations=15000, emb=32).to("cuda")
    x = torch.randn(wl.relation_count, wl.emb, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    outs = torch.ops.relm_mp.lgan_relation_graph_step(x, *wl.graph(), wl.entity_dim_size, mode)
    ref = oracle.lgan_relation_graph_step(x.cpu().numpy(), *[t.cpu() for t in wl.graph()], wl.entity_dim_size, mode)
    for g, r in zip(outs, ref):
        torch.testing.assert_close(g, torch.from_numpy(r).cuda(), rtol=1e-4, atol=1e-4)
    grad = torch.ops.relm_mp.lgan_relation_graph_step_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, *wl.graph(),
                                                               wl.relation_count, mode)
    ref_g = oracle.lgan_relation_graph_step_backward(wl.grad_x.cpu().numpy(), wl.grad_tn.cpu().numpy(),
                                                     wl.grad_nn.cpu().numpy(), *[t.cpu() for t in wl.graph()],
                                                     wl.relation_count, mode)
    torch.testing.assert_close(grad, torch.from_numpy(ref_g).cuda(), rtol=1e-4, atol=1e-4)


# ---- the planned pieces ------------------------------------------------------------------


def _epilogue_expect(table, out_idx, gather_idx, rows, base, row_div, by_count):
    t = table.double()
    acc = torch.zeros(rows, t.size(1), dtype=torch.float64, device=t.device)
    acc.index_add_(0, out_idx, t.index_select(0, gather_idx))
    if row_div is not None:
        d = row_div.double().clamp_min(1.0)
    elif by_count:
        d = torch.bincount(out_idx, minlength=rows).double().clamp_min(1.0)
    else:
        d = torch.ones(rows, dtype=torch.float64, device=t.device)
    res = acc / d[:, None]
    if base is not None:
        res = res + base.double()
    return res


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("emb", [1, 3, 8, 16, 64, 128, 300])
@pytest.mark.parametrize("kind", ["count", "div", "base", "base_count_inplace"])
@pytest.mark.parametrize("dups", [True, False])
def test_reduce_epilogue_shapes(dtype, emb, kind, dups) -> None:
    g = torch.Generator(device="cuda").manual_seed(emb * 7 + len(kind))
    rows, e = 900, 4000
    table = torch.randn(e + 50, emb, device="cuda", generator=g).to(dtype)
    if dups:
        out_idx = torch.randint(0, rows, (e,), device="cuda", generator=g)
    else:  # at most one edge per row: the row map
        out_idx = torch.randperm(rows, device="cuda", generator=g)[: rows // 2]
        e = out_idx.numel()
    gather_idx = torch.randint(0, table.size(0), (e,), device="cuda", generator=g)
    plan = capi.PlanHandle(out_idx, gather_idx, rows, table.size(0))
    base = torch.randn(rows, emb, device="cuda", generator=g).to(dtype) if kind.startswith("base") else None
    row_div = torch.randint(-1, 5, (rows,), device="cuda", generator=g) if kind == "div" else None
    by_count = kind in ("count", "base_count_inplace")
    expect = _epilogue_expect(table, out_idx, gather_idx, rows, base, row_div, by_count)
    out = base if kind == "base_count_inplace" else None
    got = plan.reduce_ex(table, base=base, row_div=row_div, divide_by_count=by_count, out=out)
    if kind == "base_count_inplace":
        assert got.data_ptr() == base.data_ptr()
    tol = 1e-2 if dtype in (torch.bfloat16, torch.float16) else (1e-10 if dtype == torch.float64 else 1e-4)
    torch.testing.assert_close(got.double(), expect, rtol=tol, atol=tol)


@pytest.mark.parametrize("mode_count", [True, False])
def test_reduce_epilogue_long_rows(mode_count) -> None:
    """Rows spanning many merge-path tiles finish in the (long-row) fixups."""

    g = torch.Generator(device="cuda").manual_seed(11)
    rows, e, emb = 64, 400_000, 32
    out_idx = torch.cat([torch.zeros(300_000, dtype=torch.long, device="cuda"),
                         torch.randint(1, rows, (e - 300_000,), device="cuda", generator=g)])
    out_idx = out_idx[torch.randperm(e, device="cuda", generator=g)]
    table = torch.randn(e, emb, device="cuda", generator=g)
    gather_idx = torch.arange(e, device="cuda")
    base = torch.randn(rows, emb, device="cuda", generator=g)
    row_div = None if mode_count else torch.full((rows,), 3, dtype=torch.long, device="cuda")
    plan = capi.PlanHandle(out_idx, gather_idx, rows, e)
    got = plan.reduce_ex(table, base=base, row_div=row_div, divide_by_count=mode_count)
    expect = _epilogue_expect(table, out_idx, gather_idx, rows, base, row_div, mode_count)
    torch.testing.assert_close(got.double(), expect, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("emb", [4, 64, 100])
def test_dividing_scatter_and_counts(dtype, emb) -> None:
    g = torch.Generator(device="cuda").manual_seed(emb)
    R = 3000
    arities = torch.randint(0, 4, (R,), device="cuda", generator=g)
    s2r = torch.repeat_interleave(torch.arange(R, device="cuda"), arities.clamp_min(1))
    s2r = s2r[torch.randperm(s2r.numel(), device="cuda", generator=g)]
    S = s2r.numel()
    plan = capi.PlanHandle(s2r, None, R, S)  # identity gather: edge s is slot s
    assert torch.equal(plan.gidx().sort().values, torch.arange(S))
    table = torch.randn(R, emb, device="cuda", generator=g).to(dtype)
    got = plan.scatter_rows_div(table, arities)
    acc = torch.float64 if dtype == torch.float64 else torch.float32  # the kernels divide in the accumulator type
    expect = (table.to(acc)[s2r] / arities.to(acc).clamp_min(1.0)[s2r, None]).to(dtype)
    torch.testing.assert_close(got, expect, rtol=0, atol=0)
    torch.testing.assert_close(plan.gather_rows_div(s2r, table, arities), expect, rtol=0, atol=0)
    torch.testing.assert_close(plan.gather_rows_div(s2r, table, None), table[s2r], rtol=0, atol=0)
    counts = plan.gather_counts()
    assert torch.equal(counts, torch.ones(S, dtype=torch.int32, device="cuda"))
    pr = capi.PlanHandle(torch.randint(0, 50, (999,), device="cuda", generator=g),
                         torch.randint(0, R, (999,), device="cuda", generator=g), 50, R)
    c2 = pr.gather_counts()
    assert torch.equal(c2.long(), torch.bincount(pr.gidx().cuda(), minlength=R))
    div = capi.divide_rows(table, c2)
    expect = (table.to(acc) / c2.to(acc).clamp_min(1.0)[:, None]).to(dtype)
    torch.testing.assert_close(div, expect, rtol=0, atol=0)


@pytest.mark.parametrize("mode", ["sum", "mean"])
def test_autograd_matches_cpu_formulas(mode) -> None:
    wl = workloads.lgan(seed=5, entities=500, relations=3000, emb=16).to("cuda", torch.float64)
    slots = wl.slots.clone().requires_grad_(True)
    outs = mp._lgan_pool_reduce(slots, wl.slot_to_rel, wl.arities, *wl.graph(), entity_dim_size=wl.entity_dim_size,
                                mode=mode)
    # gradients of two of the three outputs only (the third's is None in backward)
    torch.autograd.backward((outs[0], outs[2]), (wl.grad_x, wl.grad_nn))
    c = wl.to("cpu")
    slots_c = c.slots.clone().requires_grad_(True)
    outs_c = mp._lgan_pool_reduce(slots_c, c.slot_to_rel, c.arities, *c.graph(), entity_dim_size=c.entity_dim_size,
                                  mode=mode)
    torch.autograd.backward((outs_c[0], outs_c[2]), (c.grad_x, c.grad_nn))
    for a, b in zip(outs, outs_c):
        torch.testing.assert_close(a.detach().cpu(), b.detach(), rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(slots.grad.cpu(), slots_c.grad, rtol=1e-10, atol=1e-10)
    x = wl.grad_x.clone().requires_grad_(True)
    o = mp._lgan_relation_graph_step(x, *wl.graph(), entity_dim_size=wl.entity_dim_size, mode=mode)
    o[1].sum().backward()
    xc = c.grad_x.clone().requires_grad_(True)
    oc = mp._lgan_relation_graph_step(xc, *c.graph(), entity_dim_size=c.entity_dim_size, mode=mode)
    oc[1].sum().backward()
    torch.testing.assert_close(x.grad.cpu(), xc.grad, rtol=1e-10, atol=1e-10)


def test_plans_are_reused_across_layers() -> None:
    wl = workloads.lgan(seed=9, entities=800, relations=4000, emb=32).to("cuda")
    ops = torch.ops.relm_mp
    mp.clear_plan_cache()
    before = mp.plan_cache_stats()["builds"]
    ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, 2)
    ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities, *wl.graph(),
                                  wl.relation_count, 2)
    builds = mp.plan_cache_stats()["builds"]
    for _ in range(3):
        ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, 2)
        ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities, *wl.graph(),
                                      wl.relation_count, 2)
    assert mp.plan_cache_stats()["builds"] == builds
    assert builds - before == 7  # pool, rr, tn, nn forward; tn, nn, rr reverse


@pytest.mark.parametrize("mode", [0, 2])
def test_side_stream_plan_builds_are_awaited(mode) -> None:
    """The torch ops lay out an op's plans side by side on pool streams and
    each op waits for its own plan only: with the plan cache cleared before
    every repetition (all plans built inside the call, the backward's over the
    forward's transposed pairs), forward and backward equal the C ABI's
    (sequential builds) bit for bit, at a size where the layouts take long
    enough to overlap the first op."""

    wl = workloads.lgan(seed=11, entities=1 << 15, relations=1 << 18, emb=32).to("cuda", torch.float32)
    ops = torch.ops.relm_mp
    want = capi.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
    want_g = capi.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                            *wl.graph(), wl.relation_count, mode)
    for _ in range(4):
        mp.clear_plan_cache()
        outs = ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
        grad = ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                             *wl.graph(), wl.relation_count, mode)
        for a, b in zip(outs, want):
            assert torch.equal(a, b)
        assert torch.equal(grad, want_g)


def test_side_stream_plan_builds_on_a_user_stream() -> None:
    """The same with the ops issued on a stream of the caller's (the plan
    layouts fork from and are awaited on that stream, not the default one),
    and the default stream reading the results after waiting for it."""

    wl = workloads.lgan(seed=12, entities=1 << 14, relations=1 << 17, emb=16).to("cuda", torch.float32)
    ops = torch.ops.relm_mp
    want = capi.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, 2)
    want_g = capi.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                            *wl.graph(), wl.relation_count, 2)
    torch.cuda.synchronize()
    user = torch.cuda.Stream()
    for _ in range(3):
        mp.clear_plan_cache()
        user.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(user):
            outs = ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, 2)
            grad = ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                                 *wl.graph(), wl.relation_count, 2)
        torch.cuda.current_stream().wait_stream(user)
        for a, b in zip(outs, want):
            assert torch.equal(a, b)
        assert torch.equal(grad, want_g)
