"""CUDA parity: the B200 kernels against the CPU oracle and the reference goldens.

Every test runs the C ABI (``relmo_b200.capi`` -> ``librelm_mp_b200.so``) and,
where it applies, the drop-in ``torch.ops.relm_mp`` path (``relmo_b200.ops.mp``)
on the same seeded inputs as the oracle (``oracle/``).

Tolerances:
* fanout forward, index handling, index errors: bit-exact;
* fp32 sum / logsumexp: 1e-5 relative / 1e-6 absolute, where a sum is also
  allowed 1e-5 of the sum of |terms| of its row (the kernel adds a row's terms
  in a different order than the reference's sequential loop);
* fp64: 1e-12 relative on the same scale;
* bf16 / fp16 storage with fp32 accumulation: 1e-2 relative against the fp32
  oracle on upcast inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200 import capi, workloads
from relmo_b200.ops import mp
from tests._golden import close, load_cases, load_cfg1, sha256

pytestmark = pytest.mark.gpu

DEV = "cuda"
CASES = load_cases()


@pytest.fixture(autouse=True, scope="module")
def _load_library():
    assert mp.available(), "relm_mp library not loadable"


def _t(a, device=DEV):
    if isinstance(a, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return a


def capi_call(op: str, args: list):
    a = [_t(x) for x in args]
    if op == "fanout_scatter":
        return capi.fanout_scatter(*a)
    if op == "fanout_scatter_backward":
        return capi.fanout_scatter_backward(*a)
    if op == "fanin_reduce":
        return capi.fanin_reduce(*a)
    if op == "fanin_reduce_sum_backward":
        return capi.fanin_reduce_sum_backward(*a)
    if op == "fanin_reduce_logsumexp_backward":
        g, rel, src, dst, out, rows = a
        return capi.fanin_reduce_logsumexp_backward(g, rel, src, dst, out, rows)
    raise ValueError(op)


def torch_call(op: str, args: list):
    return getattr(torch.ops.relm_mp, op)(*[_t(x) for x in args])


def sum_scale(values: np.ndarray, gather: np.ndarray, scatter: np.ndarray, rows: int) -> np.ndarray:
    """Per output element: sum over the row's terms of |term| (summation condition)."""

    out = np.zeros((rows, values.shape[1]), dtype=np.float64)
    np.add.at(out, scatter, np.abs(values[gather].astype(np.float64)))
    return out


def assert_sum_close(got: np.ndarray, ref: np.ndarray, scale: np.ndarray, rtol=1e-5, atol=1e-6) -> None:
    got64 = got.astype(np.float64)
    ref64 = ref.astype(np.float64)
    err = np.abs(got64 - ref64)
    bound = atol + rtol * np.maximum(np.abs(ref64), scale)
    bad = ~(err <= bound)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance; worst {err[bad].max() if bad.any() else 0}"


# ---- golden cases ----------------------------------------------------------------


@pytest.mark.parametrize("path", ["capi", "torch"])
@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_golden_case(case, path: str) -> None:
    call = capi_call if path == "capi" else torch_call
    if case.raises:
        with pytest.raises(RuntimeError) as info:
            call(case.op, case.args)
            torch.cuda.synchronize()
        if not (case.op == "fanin_reduce" and case.args[-1] == 1):
            # same text as the reference CPU op (mp_ops.cpp:59-64)
            assert case.message in str(info.value)
        return
    got = call(case.op, case.args).cpu().numpy()
    assert got.shape == case.out.shape and got.dtype == case.out.dtype
    if case.op == "fanout_scatter":
        assert np.array_equal(got, case.out, equal_nan=True)
    elif case.op == "fanin_reduce" and case.args[-1] == 1:
        assert close(got, case.out, rtol=1e-5, atol=1e-6)
    else:
        assert close(got, case.out, rtol=1e-5, atol=1e-6)


# ---- cfg1 (reference golden + oracle) ------------------------------------------


@pytest.fixture(scope="module")
def cfg1():
    return workloads.cfg1(seed=0)


@pytest.mark.parametrize("path", ["capi", "torch"])
def test_cfg1_against_reference_golden(cfg1, path: str) -> None:
    meta, ref = load_cfg1()
    wl = cfg1.to(DEV)
    call = capi_call if path == "capi" else torch_call
    fan = call("fanout_scatter", [wl.x, wl.src, wl.flat_dst, wl.out_rows]).cpu().numpy()
    assert sha256(fan) == meta["out_sha256"]["fanout_fwd"]  # bit-exact
    sum_bwd = call("fanin_reduce_sum_backward", [wl.grad_nodes, wl.flat_src, wl.dst, wl.msgs.size(0)]).cpu().numpy()
    assert sha256(sum_bwd) == meta["out_sha256"]["fanin_sum_bwd"]  # one term per row: exact
    fan_bwd = call("fanout_scatter_backward", [wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0)]).cpu().numpy()
    assert close(fan_bwd, ref["fanout_bwd"], rtol=1e-5, atol=1e-6)
    fsum = call("fanin_reduce", [wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0]).cpu().numpy()
    assert close(fsum, ref["fanin_sum_fwd"], rtol=1e-5, atol=1e-6)
    flse_t = call("fanin_reduce", [wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1])
    assert close(flse_t.cpu().numpy(), ref["fanin_lse_fwd"], rtol=1e-5, atol=1e-6)
    lse_bwd = call(
        "fanin_reduce_logsumexp_backward", [wl.grad_nodes, wl.msgs, wl.flat_src, wl.dst, flse_t, wl.msgs.size(0)]
    ).cpu().numpy()
    rows = ref["fanin_lse_bwd_rows"]
    assert close(lse_bwd[rows], ref["fanin_lse_bwd_sample"], rtol=1e-5, atol=1e-6)


def test_cfg1_autograd_matches_oracle(cfg1) -> None:
    wl = cfg1.to(DEV)
    x = wl.x.clone().requires_grad_(True)
    out = mp.fanout_scatter(x, wl.src, wl.flat_dst, wl.out_rows)
    out.backward(wl.grad_slots)
    ref_x = oracle.fanout_scatter_backward(cfg1.grad_slots.numpy(), cfg1.src, cfg1.flat_dst, cfg1.x.size(0))
    assert close(x.grad.cpu().numpy(), ref_x, rtol=1e-5, atol=1e-6)
    for mode in (0, 1):
        rel = wl.msgs.clone().requires_grad_(True)
        y = mp.fanin_reduce(rel, wl.flat_src, wl.dst, wl.dim_size, mode)
        y.backward(wl.grad_nodes)
        fwd = oracle.fanin_reduce(cfg1.msgs.numpy(), cfg1.flat_src, cfg1.dst, cfg1.dim_size, mode)
        assert close(y.detach().cpu().numpy(), fwd, rtol=1e-5, atol=1e-6)
        if mode == 0:
            g = oracle.fanin_reduce_sum_backward(cfg1.grad_nodes.numpy(), cfg1.flat_src, cfg1.dst, cfg1.msgs.size(0))
        else:
            g = oracle.fanin_reduce_logsumexp_backward(
                cfg1.grad_nodes.numpy(), cfg1.msgs.numpy(), cfg1.flat_src, cfg1.dst, fwd, cfg1.msgs.size(0)
            )
        assert close(rel.grad.cpu().numpy(), g, rtol=1e-5, atol=1e-6)


# ---- shapes, dtypes, distributions --------------------------------------------------


def _random_problem(seed: int, n_src: int, n_dst: int, edges: int, emb: int, hub_frac: float = 0.0):
    g = torch.Generator().manual_seed(seed)
    vals = torch.randn(n_src, emb, generator=g, dtype=torch.float64).float()
    src = torch.randint(0, n_src, (edges,), generator=g)
    dst = torch.randint(0, n_dst, (edges,), generator=g)
    if hub_frac > 0:
        hub = torch.rand(edges, generator=g) < hub_frac
        dst[hub] = 3 % n_dst
    return vals, src, dst


EMBS = [1, 3, 4, 5, 8, 16, 31, 32, 33, 64, 100, 128, 256, 300, 512, 513, 1024, 1030]


@pytest.mark.parametrize("emb", EMBS)
def test_emb_sizes_all_ops(emb: int) -> None:
    vals, src, dst = _random_problem(emb, 300, 97, 1500, emb)
    v = vals.numpy()
    fsum = capi.fanin_reduce(vals.to(DEV), src.to(DEV), dst.to(DEV), 97, 0).cpu().numpy()
    assert_sum_close(fsum, oracle.fanin_reduce(v, src, dst, 97, 0), sum_scale(v, src.numpy(), dst.numpy(), 97))
    flse = capi.fanin_reduce(vals.to(DEV), src.to(DEV), dst.to(DEV), 97, 1).cpu().numpy()
    ref_lse = oracle.fanin_reduce(v, src, dst, 97, 1)
    assert close(flse, ref_lse, rtol=1e-5, atol=1e-6)
    perm = torch.randperm(1500, generator=torch.Generator().manual_seed(emb))
    fan = capi.fanout_scatter(vals.to(DEV), src.to(DEV), perm.to(DEV), 1600).cpu().numpy()
    assert np.array_equal(fan, oracle.fanout_scatter(v, src, perm, 1600))
    go = torch.randn(97, emb, generator=torch.Generator().manual_seed(1), dtype=torch.float64).float()
    lse_t = torch.from_numpy(ref_lse)
    gl = capi.fanin_reduce_logsumexp_backward(go.to(DEV), vals.to(DEV), src.to(DEV), dst.to(DEV), lse_t.to(DEV), 300)
    ref_gl = oracle.fanin_reduce_logsumexp_backward(go.numpy(), v, src, dst, ref_lse, 300)
    assert_sum_close(gl.cpu().numpy(), ref_gl, np.abs(ref_gl) * 4)
    # fanout backward with (src=dst, flat_dst=src): grad_x[dst[e]] += go'[src[e]] over a [300, emb] grad_out
    go2 = torch.randn(300, emb, generator=torch.Generator().manual_seed(2), dtype=torch.float64).float()
    gb = capi.fanout_scatter_backward(go2.to(DEV), dst.to(DEV), src.to(DEV), 97).cpu().numpy()
    ref_gb = oracle.fanout_scatter_backward(go2.numpy(), dst, src, 97)
    assert_sum_close(gb, ref_gb, sum_scale(go2.numpy(), src.numpy(), dst.numpy(), 97))


@pytest.mark.parametrize("hub_frac", [0.3, 0.9])
@pytest.mark.parametrize("emb", [32, 64])
def test_hub_rows_spanning_many_tiles(hub_frac: float, emb: int) -> None:
    """One destination row receives most messages: exercises the long-row fixup."""

    edges = 300_000
    vals, src, dst = _random_problem(11, edges, 5000, edges, emb, hub_frac)
    v = vals.numpy()
    for mode in (0, 1):
        got = capi.fanin_reduce(vals.to(DEV), src.to(DEV), dst.to(DEV), 5000, mode).cpu().numpy()
        ref64 = oracle.fanin_reduce(v.astype(np.float64), src, dst, 5000, mode)
        if mode == 0:
            assert_sum_close(got, ref64, sum_scale(v, src.numpy(), dst.numpy(), 5000))
        else:
            assert close(got, ref64, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_storage_fp32_accumulation(dtype) -> None:
    vals, src, dst = _random_problem(5, 4000, 700, 30000, 64, 0.2)
    lowp = vals.to(dtype)
    up = lowp.float().numpy()
    for mode in (0, 1):
        got = capi.fanin_reduce(lowp.to(DEV), src.to(DEV), dst.to(DEV), 700, mode)
        assert got.dtype == dtype
        ref = oracle.fanin_reduce(up, src, dst, 700, mode)
        scale = sum_scale(up, src.numpy(), dst.numpy(), 700) if mode == 0 else np.abs(ref)
        assert_sum_close(got.float().cpu().numpy(), ref, scale * 1e-3, rtol=1e-2, atol=1e-3)
    fan = capi.fanout_scatter(lowp.to(DEV), src.to(DEV), torch.randperm(30000).to(DEV), 30000)
    assert fan.dtype == dtype


def test_float64_tight() -> None:
    vals, src, dst = _random_problem(9, 3000, 400, 40000, 48, 0.1)
    v = vals.double()
    for mode in (0, 1):
        got = capi.fanin_reduce(v.to(DEV), src.to(DEV), dst.to(DEV), 400, mode).cpu().numpy()
        ref = oracle.fanin_reduce(v.numpy(), src, dst, 400, mode)
        scale = sum_scale(v.numpy(), src.numpy(), dst.numpy(), 400) if mode == 0 else np.abs(ref)
        assert_sum_close(got, ref, scale, rtol=1e-12, atol=1e-12)


# ---- properties ---------------------------------------------------------------------------


def test_sorted_and_unsorted_inputs_agree_bitwise() -> None:
    """A stable destination sort with permuted messages leaves every row's
    message sequence unchanged, so the results must be bit-identical."""

    wl = workloads.cfg2(seed=3, device=DEV, n=1 << 14, edges=1 << 18, emb=64)
    order = torch.sort(wl.dst, stable=True).indices
    for mode in (0, 1):
        a = capi.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, mode)
        b = capi.fanin_reduce(wl.msgs[order], wl.flat_src, wl.dst[order], wl.dim_size, mode)
        assert torch.equal(a.isnan(), b.isnan())
        assert torch.equal(torch.nan_to_num(a), torch.nan_to_num(b))


def test_deterministic_across_runs() -> None:
    wl = workloads.cfg2(seed=4, device=DEV, n=1 << 14, edges=1 << 18, emb=64)
    for mode in (0, 1):
        a = capi.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, mode)
        b = capi.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, mode)
        assert torch.equal(torch.nan_to_num(a), torch.nan_to_num(b))
    g1 = capi.fanout_scatter_backward(wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0))
    g2 = capi.fanout_scatter_backward(wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0))
    assert torch.equal(g1, g2)


def test_plan_cache_hits_and_invalidation() -> None:
    mp.clear_plan_cache()
    wl = workloads.cfg1(seed=0).to(DEV)
    a = torch.ops.relm_mp.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    s0 = mp.plan_cache_stats()
    b = torch.ops.relm_mp.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    s1 = mp.plan_cache_stats()
    assert s1["hits"] == s0["hits"] + 1 and s1["builds"] == s0["builds"]
    assert torch.equal(a, b)
    # in-place change of the index bumps its version: the stale plan must not be used
    wl.dst[:100] = 0
    c = torch.ops.relm_mp.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    msgs, fsrc, dst = wl.msgs.cpu().numpy(), wl.flat_src.cpu().numpy(), wl.dst.cpu().numpy()
    ref = oracle.fanin_reduce(msgs, fsrc, dst, wl.dim_size, 0)
    assert_sum_close(c.cpu().numpy(), ref, sum_scale(msgs, fsrc, dst, wl.dim_size))
    assert mp.plan_cache_stats()["builds"] == s1["builds"] + 1


def test_noncontiguous_and_rectangular_inputs() -> None:
    base = torch.randn(6, 9, device=DEV)
    x = base.t()  # [9, 6] non-contiguous
    src = torch.tensor([0, 4, 2, 5, 8], device=DEV)
    dst = torch.tensor([2, 1, 0, 3, 6], device=DEV)
    out = mp.fanout_scatter(x, src, dst, 7)
    ref = oracle.fanout_scatter(x.cpu().numpy(), src.cpu(), dst.cpu(), 7)
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("mode", [0, 1])
def test_gradcheck_float64(mode: int) -> None:
    rel = torch.randn(8, 4, dtype=torch.float64, device=DEV, requires_grad=True)
    src = torch.tensor([0, 2, 5, 7, 1, 3], device=DEV)
    dst = torch.tensor([1, 0, 3, 2, 0, 1], device=DEV)
    assert torch.autograd.gradcheck(lambda t: mp.fanin_reduce(t, src, dst, 4, mode), (rel,), eps=1e-6, atol=1e-4, rtol=1e-3)
    x = torch.randn(6, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    s2 = torch.tensor([0, 5, 2, 1], device=DEV)
    d2 = torch.tensor([1, 0, 3, 2], device=DEV)
    assert torch.autograd.gradcheck(lambda t: mp.fanout_scatter(t, s2, d2, 5), (x,), eps=1e-6, atol=1e-4, rtol=1e-3)


def test_errors_match_reference_semantics() -> None:
    x = torch.randn(4, 3, device=DEV)
    with pytest.raises(RuntimeError, match="must be rank 2"):
        torch.ops.relm_mp.fanout_scatter(x[0], torch.tensor([0], device=DEV), torch.tensor([0], device=DEV), 2)
    with pytest.raises(RuntimeError, match="must have dtype torch.int64"):
        torch.ops.relm_mp.fanout_scatter(x, torch.tensor([0], device=DEV, dtype=torch.int32), torch.tensor([0], device=DEV), 2)
    with pytest.raises(RuntimeError, match="equal length"):
        torch.ops.relm_mp.fanin_reduce(x, torch.tensor([0, 1], device=DEV), torch.tensor([0], device=DEV), 2, 0)
    with pytest.raises((ValueError, RuntimeError), match="Unsupported fanin_reduce mode"):
        torch.ops.relm_mp.fanin_reduce(x, torch.tensor([0], device=DEV), torch.tensor([0], device=DEV), 2, 5)
    with pytest.raises(RuntimeError, match="out_rows must be >= 0"):
        torch.ops.relm_mp.fanout_scatter(x, torch.tensor([0], device=DEV), torch.tensor([0], device=DEV), -1)
    # the GPU has no Python fallback
    import os

    os.environ["RELM_MP_ENABLE"] = "0"
    try:
        with pytest.raises(RuntimeError, match="no GPU fallback"):
            mp.fanin_reduce(x, torch.tensor([0], device=DEV), torch.tensor([0], device=DEV), 2, 0)
    finally:
        del os.environ["RELM_MP_ENABLE"]


@pytest.mark.parametrize("flat_src_kind", ["arange", "permutation"])
@pytest.mark.parametrize("extra_rows", [0, 5])
def test_backward_plan_from_the_forward(flat_src_kind: str, extra_rows: int) -> None:
    """A fan-in backward after its forward: with flat_src = arange the
    backward's plan comes from the forward's validated destination index
    without a validation pass of its own (no extra validated build); with a
    permuted flat_src it is built the usual way. Both backwards, both cases,
    against the oracle; rel_rows above the edge count leaves the extra message
    rows zero."""

    mp.clear_plan_cache()
    g = torch.Generator(device=DEV).manual_seed(3)
    rows, edges, emb = 700, 20_000, 32
    dst = torch.randint(0, rows, (edges,), device=DEV, generator=g)
    if flat_src_kind == "arange":
        fsrc = torch.arange(edges, device=DEV)
    else:
        fsrc = torch.randperm(edges, device=DEV, generator=g)
    rel_rows = edges + extra_rows
    msgs = torch.randn(rel_rows, emb, device=DEV, generator=g)
    grad = torch.randn(rows, emb, device=DEV, generator=g)
    ops = torch.ops.relm_mp
    lse = ops.fanin_reduce(msgs, fsrc, dst, rows, 1)
    s0 = mp.plan_cache_stats()
    gs = ops.fanin_reduce_sum_backward(grad, fsrc, dst, rel_rows)
    gl = ops.fanin_reduce_logsumexp_backward(grad, msgs, fsrc, dst, lse, rel_rows)
    s1 = mp.plan_cache_stats()
    assert s1["builds"] == s0["builds"] + 1  # one plan of (flat_src, dst), shared by both backwards
    m, f, d, gr = msgs.cpu().numpy(), fsrc.cpu().numpy(), dst.cpu().numpy(), grad.cpu().numpy()
    ref_s = oracle.fanin_reduce_sum_backward(gr, f, d, rel_rows)
    assert np.array_equal(gs.cpu().numpy(), ref_s)  # every message row is one copied grad row
    ref_lse = oracle.fanin_reduce(m, f, d, rows, 1)
    ref_l = oracle.fanin_reduce_logsumexp_backward(gr, m, f, d, ref_lse, rel_rows)
    assert np.allclose(gl.cpu().numpy(), ref_l, rtol=1e-5, atol=1e-6)
    if extra_rows:
        assert not gs[edges:].any() and not gl[edges:].any()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("emb", [64, 32])
def test_half_storage_logsumexp_special_values(dtype, emb: int) -> None:
    """2-byte logsumexp on rows long enough for the merge-path kernels (more
    than 32 edges, one row over many tiles): a row of only -inf gives NaN, an
    empty row -inf, a +inf or NaN value NaN, -inf values among finite ones
    contribute nothing, a single value comes back as itself; the rest within
    1e-2 of the float32 oracle on the same (2-byte) values."""

    g = torch.Generator().manual_seed(17)
    rows, special = 300, 6
    counts = torch.randint(33, 120, (rows,), generator=g)
    counts[0] = 40  # only -inf
    counts[1] = 40  # one +inf among finite
    counts[2] = 40  # one NaN among finite
    counts[3] = 40  # half -inf, half finite
    counts[4] = 0  # empty
    counts[5] = 1  # a single value
    counts[7] = 6000  # spans many tiles, with -inf values inside
    dst = torch.repeat_interleave(torch.arange(rows), counts)
    edges = int(dst.numel())
    perm = torch.randperm(edges, generator=g)
    dst = dst[perm]
    vals = torch.randn(edges, emb, generator=g) * 3
    pos = torch.empty(edges, dtype=torch.int64)
    pos[perm] = torch.arange(edges)  # edge of each (row-ordered) slot
    start = torch.cumsum(counts, 0) - counts
    vals[pos[start[0]:start[0] + 40]] = -float("inf")
    vals[pos[start[1] + 7], 3] = float("inf")
    vals[pos[start[2] + 11], 5] = float("nan")
    vals[pos[start[3]:start[3] + 20]] = -float("inf")
    vals[pos[start[7]:start[7] + 6000:3], :emb // 2] = -float("inf")
    flat_src = torch.arange(edges)
    lowp = vals.to(dtype)
    up = lowp.float().numpy()
    got = torch.ops.relm_mp.fanin_reduce(lowp.to(DEV), flat_src.to(DEV), dst.to(DEV), rows, 1)
    got = got.float().cpu().numpy()
    ref = oracle.fanin_reduce(up, flat_src, dst, rows, 1)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref)) and np.array_equal(got[np.isinf(got)], ref[np.isinf(ref)])
    assert np.isnan(got[0]).all() and np.isneginf(got[4]).all()
    assert np.isnan(got[1, 3]) and np.isnan(got[2, 5])
    single = lowp[pos[start[5]]].float().numpy()
    assert np.array_equal(got[5], single)
    fin = np.isfinite(ref)
    assert np.allclose(got[fin], ref[fin], rtol=1e-2, atol=1e-2)
