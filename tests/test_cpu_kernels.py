"""The library's CPU kernels against the reference's own CPU library.

relmo's facade sends CPU tensors to ``torch.ops.relm_mp`` whenever its library
loads (src/relmo/ops/mp.py:49-51, 65-68), so the drop-in library registers CPU
kernels too (``relm_mp_cpu.cpp``). The golden vectors were produced by the
reference library built from src/_ops/mp/mp_ops.cpp (tests/golden/make_golden.py):
its CPU outputs and its error messages. The CPU kernels run the reference's
loops and ATen formulas, so every output must equal the golden bit for bit, and
every error must carry the reference's message. Runs on CPU.
"""

from __future__ import annotations

import re

import numpy as np
import pytest
import torch

from relmo_b200 import workloads
from relmo_b200.ops import mp
from tests._golden import load_cases, load_cfg1, load_lgan_cases, load_pack_cases, sha256

CASES = load_cases()
LGAN_CASES = load_lgan_cases()
PACK_CASES = load_pack_cases()


@pytest.fixture(autouse=True, scope="module")
def _library():
    assert mp.available(), "relm_mp library not loadable"


def _cpu(args):
    return [torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a for a in args]


def _equal(got: torch.Tensor, ref: np.ndarray) -> bool:
    g = got.numpy()
    return g.dtype == ref.dtype and g.shape == ref.shape and np.array_equal(g, ref, equal_nan=True)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_cpu_op_equals_reference_library(case) -> None:
    op = getattr(torch.ops.relm_mp, case.op)
    if case.raises:
        with pytest.raises(Exception, match=re.escape(case.message)):
            op(*_cpu(case.args))
        return
    assert _equal(op(*_cpu(case.args)), case.out)


@pytest.mark.parametrize("case", LGAN_CASES, ids=[c.name for c in LGAN_CASES])
def test_cpu_lgan_op_equals_reference_library(case) -> None:
    op = getattr(torch.ops.relm_mp, case.op)
    if case.raises:
        with pytest.raises(Exception, match=re.escape(case.message)):
            op(*_cpu(case.args))
        return
    got = op(*_cpu(case.args))
    got = list(got) if isinstance(got, (tuple, list)) else [got]
    assert len(got) == len(case.outs)
    for g, ref in zip(got, case.outs):
        assert _equal(g, ref), case.name


def _pack_args(args, device="cpu"):
    out = []
    for a in args:
        if isinstance(a, list) and a and isinstance(a[0], np.ndarray):
            out.append([torch.from_numpy(np.ascontiguousarray(t)).to(device) for t in a])
        else:
            out.append(a)
    return out


@pytest.mark.parametrize("case", PACK_CASES, ids=[c.name for c in PACK_CASES])
def test_cpu_pack_op_equals_reference_library(case) -> None:
    """The pack ops (index arithmetic + concatenation, mp_ops.cpp:412-570,
    2511-2773) on CPU tensors, against the reference library's outputs."""

    op = getattr(torch.ops.relm_mp, case.op)
    if case.raises:
        with pytest.raises(Exception, match=re.escape(case.message)):
            op(*_pack_args(case.args))
        return
    got = op(*_pack_args(case.args))
    assert len(got) == 3
    for g, ref in zip(got, case.outs):
        assert _equal(g, ref), case.name


def test_cpu_ops_equal_reference_on_cfg1() -> None:
    meta, ref = load_cfg1()
    wl = workloads.cfg1(seed=0)
    ops = torch.ops.relm_mp
    assert sha256(ops.fanout_scatter(wl.x, wl.src, wl.flat_dst, wl.out_rows).numpy()) == meta["out_sha256"]["fanout_fwd"]
    assert _equal(ops.fanout_scatter_backward(wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0)), ref["fanout_bwd"])
    assert _equal(ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0), ref["fanin_sum_fwd"])
    lse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    assert _equal(lse, ref["fanin_lse_fwd"])
    sum_bwd = ops.fanin_reduce_sum_backward(wl.grad_nodes, wl.flat_src, wl.dst, wl.msgs.size(0))
    assert sha256(sum_bwd.numpy()) == meta["out_sha256"]["fanin_sum_bwd"]
    lse_bwd = ops.fanin_reduce_logsumexp_backward(wl.grad_nodes, wl.msgs, wl.flat_src, wl.dst, lse, wl.msgs.size(0))
    rows = ref["fanin_lse_bwd_rows"]
    assert _equal(lse_bwd[torch.from_numpy(rows)], ref["fanin_lse_bwd_sample"])


def test_facade_sends_cpu_tensors_to_the_library(monkeypatch: pytest.MonkeyPatch) -> None:
    """With the library loaded, CPU calls run its kernels, as relmo's do; with
    RELM_MP_ENABLE=0 they run the Python formulas (same values)."""

    from relmo_b200.ops import mp_dispatch

    monkeypatch.delenv("RELM_MP_ENABLE", raising=False)
    x = torch.randn(6, 3)
    assert mp_dispatch.route("fanout_scatter", x) == mp_dispatch.CUSTOM
    src, dst = torch.tensor([0, 5, 2]), torch.tensor([2, 0, 3])
    lib = mp.fanout_scatter(x, src, dst, 4)
    monkeypatch.setenv("RELM_MP_ENABLE", "0")
    assert mp_dispatch.route("fanout_scatter", x) == mp_dispatch.PYTHON
    assert torch.equal(mp.fanout_scatter(x, src, dst, 4), lib)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
def test_cpu_autograd_through_the_library(dtype) -> None:
    """The reference's autograd wrappers over the CPU kernels: gradcheck in fp64,
    agreement with the ATen formulas in the other dtypes."""

    g = torch.Generator().manual_seed(3)
    rel = torch.randn(12, 5, generator=g, dtype=torch.float64)
    fs = torch.tensor([0, 2, 7, 5, 2, 1, 11, 3])
    di = torch.tensor([1, 0, 2, 2, 1, 0, 4, 3])  # no empty row: gradcheck cannot difference -inf
    if dtype == torch.float64:
        for mode in (0, 1):
            r = rel.clone().requires_grad_(True)
            assert torch.autograd.gradcheck(lambda t: mp.fanin_reduce(t, fs, di, 5, mode), (r,))
        x = rel[:7].clone().requires_grad_(True)
        assert torch.autograd.gradcheck(lambda t: mp.fanout_scatter(t, torch.tensor([0, 3, 6, 3]),
                                                                     torch.tensor([1, 0, 3, 2]), 5), (x,))
        return
    r = rel.to(dtype).requires_grad_(True)
    out = mp.fanin_reduce(r, fs, di, 5, 0)
    out.backward(torch.ones_like(out))
    expect = torch.zeros(12, 5, dtype=dtype).index_add_(0, fs, torch.ones(8, 5, dtype=dtype))
    assert torch.equal(r.grad, expect)
