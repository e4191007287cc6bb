"""LGAN ops (sum / mean): the C oracle pinned to the reference, and the CPU side.

The golden vectors (tests/golden/ref_lgan.npz, made by make_golden.py) are the
outputs of the reference's own CPU library (``torch.ops.relm_mp.lgan_*`` of
maichmueller/relmo built from src/_ops/mp/mp_ops.cpp) on the fixtures of its
tests/python/test_flat_lgan_relational_gnn.py and on edge cases. The oracle
(oracle/relm_mp_oracle.c) must reproduce them within 1e-6 (it adds in the same
edge order and divides in the element type; ATen's vectorised index_add_ and
the division can differ in the last bit). The Python CPU formulas of
relmo_b200.ops.mp_lgan (what CPU tensors run) must match the oracle, and the
C ABI must export the LGAN entry points. Runs on CPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200.ops import mp
from relmo_b200.ops.mp_lgan import lgan_pool_reduce_python, lgan_relation_graph_step_python
from tests._golden import close, load_lgan_cases

CASES = load_lgan_cases()


def run_oracle(op: str, args: list):
    fn = getattr(oracle, op)
    out = fn(*args)
    return list(out) if isinstance(out, tuple) else [out]


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_lgan(case) -> None:
    if case.raises:
        exc = ValueError if "mode" in (case.message or "") else IndexError
        with pytest.raises(exc):
            run_oracle(case.op, case.args)
        return
    got = run_oracle(case.op, case.args)
    assert len(got) == len(case.outs)
    for g, ref in zip(got, case.outs):
        assert g.dtype == ref.dtype or ref.dtype == np.float32
        tol = 1e-12 if ref.dtype == np.float64 else 1e-6
        assert close(g, ref, rtol=tol, atol=tol), case.name


def test_reference_fixture_values() -> None:
    """test_flat_lgan_relational_gnn.py:297-311: the expected literal values."""

    case = {c.name: c for c in CASES}["pool_lit_sum"]
    x, tn, nn = case.outs
    np.testing.assert_allclose(x, [[0.5, 0.5], [2.0, 1.0], [1.5, 2.5]], atol=1e-6, rtol=0)
    expect_tn = np.zeros((5, 2), np.float32)
    expect_tn[:3] = x
    np.testing.assert_allclose(tn, expect_tn, atol=1e-6, rtol=0)
    expect_nn = np.zeros((5, 2), np.float32)
    expect_nn[2], expect_nn[4] = x[1], x[2]
    np.testing.assert_allclose(nn, expect_nn, atol=1e-6, rtol=0)


def _torch_args(args):
    return [torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a for a in args]


@pytest.mark.parametrize("case", [c for c in CASES if not c.raises and not c.op.endswith("_backward")],
                         ids=lambda c: c.name)
def test_python_formulas_match_reference(case) -> None:
    args = _torch_args(case.args)
    fn = lgan_pool_reduce_python if case.op == "lgan_pool_reduce" else lgan_relation_graph_step_python
    got = fn(*args)
    for g, ref in zip(got, case.outs):
        tol = 1e-12 if ref.dtype == np.float64 else 1e-6
        assert close(g.numpy(), ref, rtol=tol, atol=tol), case.name


@pytest.mark.parametrize("mode", ["sum", "mean"])
def test_cpu_autograd_matches_reference_backward(mode) -> None:
    """The facade on CPU tensors differentiates the Python formulas; the result
    equals the reference's own backward op on the same upstream gradients."""

    mode_int = 0 if mode == "sum" else 2
    case = {c.name: c for c in CASES}[f"random_{mode}_bwd"]
    fwd = {c.name: c for c in CASES}[f"random_{mode}"]
    gx, gtn, gnn, s2r, ar, *graph, relation_count, _ = _torch_args(case.args)
    slots = torch.from_numpy(fwd.args[0]).requires_grad_(True)
    outs = mp._lgan_pool_reduce(slots, s2r, ar, *graph, entity_dim_size=int(fwd.args[-2]), mode=mode)
    torch.autograd.backward(outs, (gx, gtn, gnn))
    assert close(slots.grad.numpy(), case.outs[0], rtol=1e-5, atol=1e-6)
    assert mode_int in (0, 2)


def test_mode_strings() -> None:
    x = torch.zeros(2, 3)
    e = torch.zeros(0, dtype=torch.long)
    with pytest.raises(ValueError, match="supports only mode='sum' or mode='mean'"):
        mp._lgan_relation_graph_step(x, e, e, e, e, e, e, entity_dim_size=1, mode="logsumexp")
    out = mp._lgan_relation_graph_step(x, e, e, e, e, e, e, entity_dim_size=1, mode=" MEAN ")
    assert out[1].shape == (1, 3)


def _random_graph(rng, R, N, S):
    def pairs(n, a, b):
        return rng.integers(0, a, n), rng.integers(0, b, n)

    rr = pairs(int(rng.integers(0, 3 * R + 1)), R, R)
    tn = pairs(int(rng.integers(0, 2 * R + 1)), R, max(N, 1)) if N > 0 else (np.zeros(0, int), np.zeros(0, int))
    nn = pairs(int(rng.integers(0, 2 * R + 1)), R, max(N, 1)) if N > 0 else (np.zeros(0, int), np.zeros(0, int))
    s2r = rng.integers(0, R, S) if R > 0 else np.zeros(0, int)
    arities = rng.integers(-1, 4, R)  # zero and negative arities clamp to 1
    return [np.asarray(a, dtype=np.int64) for a in (*rr, *tn, *nn)], s2r.astype(np.int64), arities.astype(np.int64)


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("mode", [0, 2])
def test_oracle_matches_python_formulas_on_random_graphs(seed, mode):
    """The C oracle and the Python ATen formulas (relmo's mp_fallbacks) agree on
    random small LGAN graphs - empty edge sets, repeated targets, relations
    without slots, zero arities - forward and backward, in float64."""

    rng = np.random.default_rng(seed)
    R, N, S, D = int(rng.integers(1, 30)), int(rng.integers(0, 12)), int(rng.integers(0, 60)), int(rng.integers(1, 6))
    graph, s2r, ar = _random_graph(rng, R, N, S)
    slots = rng.standard_normal((S, D))
    x1, tn, nn = oracle.lgan_pool_reduce(slots, s2r, ar, *graph, N, mode)
    tg = [torch.from_numpy(a) for a in graph]
    ts = torch.from_numpy(slots).requires_grad_(True)
    px1, ptn, pnn = lgan_pool_reduce_python(ts, torch.from_numpy(s2r), torch.from_numpy(ar), *tg, N, mode)
    for a, b in ((x1, px1), (tn, ptn), (nn, pnn)):
        np.testing.assert_allclose(a, b.detach().numpy(), rtol=1e-12, atol=1e-12)
    gx, gtn, gnn = rng.standard_normal((R, D)), rng.standard_normal((N, D)), rng.standard_normal((N, D))
    g_or = oracle.lgan_pool_reduce_backward(gx, gtn, gnn, s2r, ar, *graph, R, mode)
    torch.autograd.backward((px1, ptn, pnn), (torch.from_numpy(gx), torch.from_numpy(gtn), torch.from_numpy(gnn)))
    np.testing.assert_allclose(g_or, ts.grad.numpy(), rtol=1e-12, atol=1e-12)
    x = rng.standard_normal((R, D))
    y = oracle.lgan_relation_graph_step(x, *graph, N, mode)
    py = lgan_relation_graph_step_python(torch.from_numpy(x), *tg, N, mode)
    for a, b in zip(y, py):
        np.testing.assert_allclose(a, b.numpy(), rtol=1e-12, atol=1e-12)
