"""The allocation-free fanin_reduce entry point against the regular one.

``relm_mp_fanin_reduce_noalloc`` serves callers that cannot allocate device
memory where they call the op: it takes its workspace from a static device
array inside the library instead of a caller workspace. Its results must match
``relm_mp_fanin_reduce`` (same kernels, same plan), call after call, although
every call reuses the scratch the previous one left behind.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import pytest
import torch

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


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_regular_entry_point_on_consecutive_calls(mode: int) -> None:
    # Two different problems in a row: the second call finds the first one's
    # plan and partials in the shared scratch and must not be affected by them.
    for seed, (n_src, n_dst, edges, emb) in enumerate([(20000, 3000, 60000, 64), (5000, 700, 21000, 32)]):
        rel, src, dst = _problem(seed, n_src, n_dst, edges, emb)
        ref = capi.fanin_reduce(rel, src, dst, n_dst, mode)
        got = capi.fanin_reduce_noalloc(rel, src, dst, n_dst, mode)
        torch.cuda.synchronize()
        assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6, equal_nan=True)


def test_noalloc_rejects_problems_beyond_its_scratch() -> None:
    lib = capi.lib()
    edges, rows, emb = 1 << 24, 1 << 20, 64
    need = lib.relm_mp_fanin_reduce_workspace_bytes(edges, rows, emb, capi.FLOAT32, 0)
    assert need > capi.NOALLOC_SCRATCH_BYTES
    # Rejected before any pointer is touched.
    rc = lib.relm_mp_fanin_reduce_noalloc(capi.FLOAT32, None, edges, emb, None, None, edges, rows, 0, None, None)
    assert rc == 3  # RELM_MP_ERR_WORKSPACE_TOO_SMALL
    assert b"static scratch" in lib.relm_mp_last_error()

