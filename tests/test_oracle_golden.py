"""Pins the C oracle to the reference's own CPU op library.

The golden vectors were produced by the reference ``relm_mp`` library built
from ``src/_ops/mp/mp_ops.cpp`` (tests/golden/make_golden.py). The oracle must
reproduce them: bit-exactly for fan-out, sums in edge order and index errors;
within 1e-6 abs / 1e-5 rel for logsumexp (the reference uses ATen's vectorized
exp). Runs on CPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200 import workloads
from tests._golden import close, load_cases, load_cfg1, sha256

CASES = load_cases()
BIT_EXACT_OPS = {"fanout_scatter", "fanout_scatter_backward", "fanin_reduce_sum_backward"}


def run_oracle(op: str, args: list):
    if op == "fanout_scatter":
        return oracle.fanout_scatter(*args)
    if op == "fanout_scatter_backward":
        return oracle.fanout_scatter_backward(*args)
    if op == "fanin_reduce":
        return oracle.fanin_reduce(*args)
    if op == "fanin_reduce_sum_backward":
        return oracle.fanin_reduce_sum_backward(*args)
    if op == "fanin_reduce_logsumexp_backward":
        return oracle.fanin_reduce_logsumexp_backward(*args)
    raise ValueError(op)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_case(case) -> None:
    if case.raises:
        with pytest.raises(IndexError):
            run_oracle(case.op, case.args)
        return
    got = run_oracle(case.op, case.args)
    assert got.dtype == case.out.dtype
    exact = case.op in BIT_EXACT_OPS or (case.op == "fanin_reduce" and case.args[-1] == 0)
    if exact:
        assert np.array_equal(got, case.out, equal_nan=True)
    else:
        assert close(got, case.out, rtol=1e-5, atol=1e-6)


def test_oracle_error_names_match_reference_messages() -> None:
    for case in CASES:
        if not case.raises or case.op == "fanin_reduce" and case.args[-1] == 1:
            continue
        with pytest.raises(oracle.OracleIndexError) as info:
            run_oracle(case.op, case.args)
        # reference message: "<name> index out of bounds: <value> not in [0, <n>)."
        assert case.message.startswith(f"{info.value.name} index out of bounds: {info.value.value} ")


def test_cfg1_inputs_are_reproducible() -> None:
    meta, _ = load_cfg1()
    wl = workloads.cfg1(seed=0)
    tensors = {
        "x": wl.x, "src": wl.src, "dst": wl.dst, "msgs": wl.msgs, "flat_dst": wl.flat_dst,
        "grad_slots": wl.grad_slots, "grad_nodes": wl.grad_nodes,
    }
    for name, t in tensors.items():
        assert sha256(t.numpy()) == meta["input_sha256"][name], name


def test_oracle_matches_reference_cfg1() -> None:
    meta, ref = load_cfg1()
    wl = workloads.cfg1(seed=0)
    x, msgs = wl.x.numpy(), wl.msgs.numpy()
    fan = oracle.fanout_scatter(x, wl.src, wl.flat_dst, wl.out_rows)
    assert sha256(fan) == meta["out_sha256"]["fanout_fwd"]
    fan_bwd = oracle.fanout_scatter_backward(wl.grad_slots.numpy(), wl.src, wl.flat_dst, x.shape[0])
    assert np.array_equal(fan_bwd, ref["fanout_bwd"])
    fsum = oracle.fanin_reduce(msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    assert np.array_equal(fsum, ref["fanin_sum_fwd"])
    flse = oracle.fanin_reduce(msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    assert close(flse, ref["fanin_lse_fwd"], rtol=1e-5, atol=1e-6)
    sum_bwd = oracle.fanin_reduce_sum_backward(wl.grad_nodes.numpy(), wl.flat_src, wl.dst, msgs.shape[0])
    assert sha256(sum_bwd) == meta["out_sha256"]["fanin_sum_bwd"]
    lse_bwd = oracle.fanin_reduce_logsumexp_backward(
        wl.grad_nodes.numpy(), msgs, wl.flat_src, wl.dst, ref["fanin_lse_fwd"], msgs.shape[0]
    )
    rows = ref["fanin_lse_bwd_rows"]
    assert close(lse_bwd[rows], ref["fanin_lse_bwd_sample"], rtol=1e-5, atol=1e-6)
    d = lse_bwd.astype(np.float64)
    ck = meta["fanin_lse_bwd_checksum"]
    assert abs(d.sum() - ck["sum"]) <= 1e-6 * max(1.0, abs(ck["sum"])) + 1e-3
    assert abs((d * d).sum() - ck["sumsq"]) <= 1e-5 * ck["sumsq"]


def test_oracle_float64_matches_torch_formulas() -> None:
    """The float64 oracle against the reference's ATen formulas (test_mp_ops.py:7-49)."""

    g = torch.Generator().manual_seed(7)
    rel = torch.randn(50, 6, dtype=torch.float64, generator=g)
    src = torch.randint(0, 50, (120,), generator=g)
    dst = torch.randint(0, 9, (120,), generator=g)
    out = torch.zeros(9, 6, dtype=torch.float64).index_add_(0, dst, rel[src])
    assert np.allclose(oracle.fanin_reduce(rel.numpy(), src, dst, 9, 0), out.numpy(), rtol=1e-12, atol=1e-12)
    lse = torch.full((9, 6), float("-inf"), dtype=torch.float64)
    idx = dst.view(-1, 1).expand(-1, 6)
    lse.scatter_reduce_(0, idx, rel[src], reduce="amax", include_self=True)
    s = torch.zeros(9, 6, dtype=torch.float64).scatter_add_(0, idx, (rel[src] - lse[dst]).exp())
    ref = s.log() + lse
    assert np.allclose(oracle.fanin_reduce(rel.numpy(), src, dst, 9, 1), ref.numpy(), rtol=1e-12, atol=1e-12, equal_nan=True)
