"""Fan ops over cached plans inside a CUDA graph: once an op's plans are built
(by an uncaptured call), the op queues only kernels and stream-ordered
allocations, so a captured call replays with the values its input tensors
hold at replay time.
"""

from __future__ import annotations

import pytest
import torch

from relmo_b200.ops import mp

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _loaded():
    assert mp.available(), "relm_mp B200 library must load on a GPU box"
    yield


@pytest.mark.parametrize("mode", [0, 1])
def test_cached_plan_fanin_replays_in_a_cuda_graph(mode: int) -> None:
    gen = torch.Generator().manual_seed(21 + mode)
    n, e, d = 4096, 50_000, 64
    dev = torch.device("cuda")
    rel = torch.randn(e, d, generator=gen).to(dev)
    flat_src = torch.randperm(e, generator=gen).to(dev)
    dst = torch.randint(0, n, (e,), generator=gen).to(dev)
    ops = torch.ops.relm_mp
    mp.clear_plan_cache()
    want = ops.fanin_reduce(rel, flat_src, dst, n, mode)  # builds and caches the plan
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            ops.fanin_reduce(rel, flat_src, dst, n, mode)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    builds = mp.plan_cache_stats()["builds"]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = ops.fanin_reduce(rel, flat_src, dst, n, mode)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert mp.plan_cache_stats()["builds"] == builds
    if mode == 0:
        rel.mul_(2.0)  # exact: every sum doubles exactly
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want * 2.0)
