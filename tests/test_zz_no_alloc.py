"""The allocation-free fanin_reduce entry point against the regular one.

``relm_mp_fanin_reduce_noalloc`` serves callers that cannot allocate device
memory where they call the op (their memory belongs to another allocator, or
they cannot afford cudaMalloc's implicit synchronization while other work is
in flight): it takes its workspace from a static device array inside the
library instead of a caller workspace. It runs the same plan and kernels as
``relm_mp_fanin_reduce``, which are deterministic, so its results must be
bit-identical to that entry point's, call after call, although every call
reuses the scratch the previous one left behind.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200 import capi

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _problem(seed: int, n_src: int, n_dst: int, edges: int, emb: int, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    rel = torch.randn(n_src, emb, generator=g, dtype=torch.float64).to(dtype)
    src = torch.randint(0, n_src, (edges,), generator=g)
    dst = torch.randint(0, n_dst, (edges,), generator=g)
    hub = torch.rand(edges, generator=g) < 0.3
    dst[hub] = 1  # one long row, so partials and the fixup pass are exercised
    return rel.to(DEV), src.to(DEV), dst.to(DEV)


def _assert_identical(got: torch.Tensor, ref: torch.Tensor) -> None:
    # NaN positions must agree; every other element bit for bit (-inf included).
    assert got.dtype == ref.dtype and got.shape == ref.shape
    assert torch.equal(got.isnan(), ref.isnan())
    assert torch.equal(torch.nan_to_num(got, nan=0.0), torch.nan_to_num(ref, nan=0.0))


PROBLEMS = [(20000, 3000, 60000, 64), (5000, 700, 21000, 32)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_regular_entry_point_on_consecutive_calls(mode: int, dtype) -> None:
    # Problem A, problem B, then A again: the later calls find the earlier
    # ones' plan and partials in the shared scratch and must not be affected.
    for seed in (0, 1, 0):
        n_src, n_dst, edges, emb = PROBLEMS[seed]
        rel, src, dst = _problem(seed, n_src, n_dst, edges, emb, dtype)
        ref = capi.fanin_reduce(rel, src, dst, n_dst, mode)
        got = capi.fanin_reduce_noalloc(rel, src, dst, n_dst, mode)
        torch.cuda.synchronize()
        _assert_identical(got, ref)


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_against_the_oracle(mode: int) -> None:
    n_src, n_dst, edges, emb = PROBLEMS[0]
    rel, src, dst = _problem(0, n_src, n_dst, edges, emb)
    got = capi.fanin_reduce_noalloc(rel, src, dst, n_dst, mode).cpu().numpy().astype(np.float64)
    v = rel.cpu().numpy()
    s, d = src.cpu().numpy(), dst.cpu().numpy()
    ref = oracle.fanin_reduce(v.astype(np.float64), s, d, n_dst, mode)
    if mode == 0:
        # 1e-5 of the row's sum of |terms|: the kernel adds a row's terms in
        # another order than the reference's sequential loop.
        scale = oracle.fanin_reduce(np.abs(v).astype(np.float64), s, d, n_dst, 0)
        bound = 1e-6 + 1e-5 * np.maximum(np.abs(ref), scale)
        assert bool((np.abs(got - ref) <= bound).all())
    else:
        assert bool(np.allclose(got, ref, rtol=1e-5, atol=1e-6, equal_nan=True))


def test_noalloc_rejects_problems_beyond_its_scratch() -> None:
    lib = capi.lib()
    edges, rows, emb = 1 << 24, 1 << 20, 64
    need = lib.relm_mp_fanin_reduce_workspace_bytes(edges, rows, emb, capi.FLOAT32, 0)
    assert need > capi.NOALLOC_SCRATCH_BYTES
    # Rejected before any pointer is touched.
    rc = lib.relm_mp_fanin_reduce_noalloc(capi.FLOAT32, None, edges, emb, None, None, edges, rows, 0, None, None)
    assert rc == 3  # RELM_MP_ERR_WORKSPACE_TOO_SMALL
    assert b"static scratch" in lib.relm_mp_last_error()
