"""The smoothed logsumexp of relmo's models as a kernel path.

relmo's models aggregate "logsumexp" with LogSumExpAggregation
(relmo/models/aggr.py:96-123): per column
``m + (1/beta) log(1e-16 + sum exp(beta (x - m)))``, m the row max without
gradient, ``(1/beta) log(1e-16)`` for rows without messages, beta = 12. The
B200 library computes it in the logsumexp kernels themselves (the exponent
scale, epsilon and empty-row value are runtime constants of every logsumexp
kernel), forward and backward. Checked here against that formula evaluated in
float64 (``smoothed_logsumexp_reference``), on row shapes that reach every
kernel family: one edge per row (row map), rows of at most 32 edges (short-row
kernel), a hub row over many tiles (merge-path stream kernel and long-row
fixup), rows that are not a multiple of 16 bytes (register kernel), and the
destination-ordered backward above the L2 working set. fp32 within 1e-5
relative / 1e-6 absolute (gradients 1e-5 of the row's gradient scale), fp64
1e-12, bf16 storage 1e-2.
"""

from __future__ import annotations

import math

import pytest
import torch

from relmo_b200 import capi, hetero_mp
from relmo_b200.ops import mp

pytestmark = pytest.mark.gpu

BETA, EPS = 12.0, 1e-16
TOL = {torch.float32: (1e-5, 1e-6), torch.float64: (1e-12, 1e-12), torch.bfloat16: (1e-2, 1e-2)}


def _problem(seed, rows, edges, emb, dtype, hub_frac=0.0, one_per_row=False):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(edges, emb, generator=g, dtype=torch.float64) * 2).to(dtype)
    if one_per_row:
        dst = torch.randperm(rows, generator=g)[:edges]
    else:
        dst = torch.randint(0, rows, (edges,), generator=g)
        if hub_frac:
            dst[torch.rand(edges, generator=g) < hub_frac] = 3
    dst[dst == 1] = 2  # row 1 never receives a message
    flat_src = torch.randperm(edges, generator=g)
    return x.cuda(), flat_src.cuda(), dst.cuda()


def _reference(x, flat_src, dst, rows):
    x64 = x.double().requires_grad_(True)
    out = hetero_mp.smoothed_logsumexp_reference(x64.index_select(0, flat_src), dst, rows, BETA)
    return x64, out


CASES = [
    # (rows, edges, emb, hub_frac, one_per_row): kernel family reached
    (3000, 2500, 32, 0.0, True),      # row map (rows hold at most one edge)
    (4000, 30000, 32, 0.0, False),    # short-row kernel (no row above 32 edges)
    (2000, 200000, 64, 0.6, False),   # merge-path stream kernel, hub over many tiles (long-row fixup)
    (1500, 40000, 5, 0.3, False),     # 20-byte rows: register segment kernel
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
@pytest.mark.parametrize("case", CASES, ids=["row_map", "short_rows", "hub_stream", "unaligned_rows"])
def test_smoothed_logsumexp_forward_and_backward(case, dtype):
    rows, edges, emb, hub, one = case
    x, flat_src, dst = _problem(rows + emb, rows, edges, emb, dtype, hub, one)
    mp.clear_plan_cache()
    xk = x.clone().requires_grad_(True)
    got = mp.fanin_reduce_smoothed_logsumexp(xk, flat_src, dst, rows, BETA, EPS)
    x64, ref = _reference(x, flat_src, dst, rows)
    rtol, atol = TOL[dtype]
    assert got.dtype == dtype
    torch.testing.assert_close(got.double(), ref.detach(), rtol=rtol, atol=atol)
    # rows without messages: (1/beta) log(eps), evaluated in the accumulator type
    empty = torch.ones(rows, dtype=torch.bool, device="cuda")
    empty[dst] = False
    assert bool(empty[1])
    want = (1.0 / BETA) * math.log(EPS) if dtype == torch.float64 else float(
        torch.tensor(1.0 / BETA, dtype=torch.float32) * torch.tensor(EPS, dtype=torch.float32).log()
    )
    assert torch.equal(got[empty].double(), torch.full_like(got[empty], want).double())
    # backward: exp(beta (x - out)) weights
    w = torch.randn(rows, emb, dtype=torch.float64, device="cuda")
    (gk,) = torch.autograd.grad((got.double() * w).sum(), xk)
    (gr,) = torch.autograd.grad((ref * w).sum(), x64)
    scale = w.abs().max().item()
    torch.testing.assert_close(gk.double(), gr, rtol=rtol, atol=atol * scale)


def test_smoothed_backward_destination_order_path():
    """Above the L2 working set with the forward's plan cached and message rows
    used once, the backward walks the forward's plan in destination order
    (relm_mp_plan_scatter_logsumexp_backward_ex); without the cached plan it
    runs per message row. Both against the float64 formula."""

    rows, edges, emb = 1 << 20, 1 << 21, 32
    x, flat_src, dst = _problem(5, rows, edges, emb, torch.float32)
    gout = torch.randn(rows, emb, device="cuda")
    ops = torch.ops.relm_mp_b200
    mp.clear_plan_cache()
    out = ops.fanin_reduce_smoothed_logsumexp(x, flat_src, dst, rows, BETA, EPS)
    warm = ops.fanin_reduce_smoothed_logsumexp_backward(gout, x, flat_src, dst, out, edges, BETA)
    mp.clear_plan_cache()
    cold = ops.fanin_reduce_smoothed_logsumexp_backward(gout, x, flat_src, dst, out, edges, BETA)
    expect = torch.zeros(edges, emb, dtype=torch.float64, device="cuda")
    expect[flat_src] = gout[dst].double() * torch.exp(BETA * (x[flat_src].double() - out[dst].double()))
    torch.testing.assert_close(warm.double(), expect, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(cold.double(), expect, rtol=1e-5, atol=1e-6)


def test_smoothed_form_through_the_c_abi():
    """relm_mp_plan_reduce_lse / relm_mp_plan_logsumexp_backward_ex with a form;
    the NULL form is the plain logsumexp of fanin_reduce mode 1."""

    rows, edges, emb = 700, 20000, 16
    x, flat_src, dst = _problem(9, rows, edges, emb, torch.float32, 0.2)
    plan = capi.PlanHandle(dst, flat_src, rows, edges)
    plain = plan.reduce_lse(x)
    assert torch.equal(plain, plan.reduce(x, 1))
    smooth = plan.reduce_lse(x, BETA, EPS)
    _, ref = _reference(x, flat_src, dst, rows)
    torch.testing.assert_close(smooth.double(), ref.detach(), rtol=1e-5, atol=1e-6)
    # backward through the message-row plan (output rows = message rows)
    mplan = capi.PlanHandle(flat_src, dst, edges, rows)
    gout = torch.randn(rows, emb, device="cuda")
    got = mplan.logsumexp_backward(gout, smooth, x, BETA)
    expect = torch.zeros(edges, emb, dtype=torch.float64, device="cuda")
    expect[flat_src] = gout[dst].double() * torch.exp(BETA * (x[flat_src].double() - smooth[dst].double()))
    torch.testing.assert_close(got.double(), expect, rtol=1e-5, atol=1e-6)


def test_bad_form_is_rejected():
    x, flat_src, dst = _problem(1, 10, 30, 4, torch.float32)
    with pytest.raises(RuntimeError, match="beta > 0"):
        torch.ops.relm_mp_b200.fanin_reduce_smoothed_logsumexp(x, flat_src, dst, 10, 0.0, EPS)
