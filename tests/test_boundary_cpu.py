"""The drop-in boundary, checked without a GPU.

* The C-ABI library loads and exports every function ``include/relm_mp.h``
  declares, and the ctypes binding declares exactly those.
* The torch library registers the reference's schemas (mp_ops.cpp:3754-3838)
  for the hot path and pack ops, plus ``build_info`` in the reference format.
* Shape-only (Meta) kernels and the CPU path of the facade.
"""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from relmo_b200 import capi
from relmo_b200.ops import mp, mp_runtime

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "relm_mp.h"

# Verbatim from maichmueller/relmo src/_ops/mp/mp_ops.cpp:3756-3788.
REFERENCE_SCHEMAS = {
    "fanout_scatter": "relm_mp::fanout_scatter(Tensor x_cat, Tensor src_global_idx, Tensor flat_dst, int out_rows) -> Tensor",
    "fanout_scatter_backward": "relm_mp::fanout_scatter_backward(Tensor grad_out, Tensor src_global_idx, Tensor flat_dst, int x_rows) -> Tensor",
    "fanin_reduce": "relm_mp::fanin_reduce(Tensor rel_flat, Tensor flat_src, Tensor dst_idx, int dim_size, int mode) -> Tensor",
    "fanin_reduce_sum_backward": "relm_mp::fanin_reduce_sum_backward(Tensor grad_out, Tensor flat_src, Tensor dst_idx, int rel_rows) -> Tensor",
    "fanin_reduce_logsumexp_backward": "relm_mp::fanin_reduce_logsumexp_backward(Tensor grad_out, Tensor rel_flat, Tensor flat_src, Tensor dst_idx, Tensor out, int rel_rows) -> Tensor",
    "fanout_pack_multi": "relm_mp::fanout_pack_multi(Tensor[] x_parts, Tensor[] src_idx_parts, Tensor[] flat_dst_parts) -> (Tensor, Tensor, Tensor)",
    "fanin_pack_multi": "relm_mp::fanin_pack_multi(Tensor[] rel_parts, Tensor[] flat_src_parts, Tensor[] dst_idx_parts) -> (Tensor, Tensor, Tensor)",
    "fanout_pack_from_edges": "relm_mp::fanout_pack_from_edges(Tensor[] x_parts, Tensor[] edge_src_parts, Tensor[] edge_dst_parts, int[] src_part_ids, int[] arity_parts, int[] pos_parts, int[] slot_offset_parts) -> (Tensor, Tensor, Tensor)",
    "fanin_pack_from_edges": "relm_mp::fanin_pack_from_edges(Tensor[] rel_parts, Tensor[] edge_src_parts, Tensor[] edge_dst_parts, int[] rel_part_ids, int[] arity_parts, int[] pos_parts, int mode) -> (Tensor, Tensor, Tensor)",
    "build_info": "relm_mp::build_info() -> str",
    # mp_ops.cpp:3777-3788
    "lgan_pool_reduce": "relm_mp::lgan_pool_reduce(Tensor slot_messages, Tensor slot_to_relation_instance, Tensor relation_instance_arities, Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int entity_dim_size, int mode) -> (Tensor, Tensor, Tensor)",
    "lgan_pool_reduce_backward": "relm_mp::lgan_pool_reduce_backward(Tensor grad_relation_pair_x, Tensor grad_tn_msgs, Tensor grad_nn_msgs, Tensor slot_to_relation_instance, Tensor relation_instance_arities, Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int relation_count, int mode) -> Tensor",
    "lgan_relation_graph_step": "relm_mp::lgan_relation_graph_step(Tensor relation_pair_x, Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int entity_dim_size, int mode) -> (Tensor, Tensor, Tensor)",
    "lgan_relation_graph_step_backward": "relm_mp::lgan_relation_graph_step_backward(Tensor grad_relation_pair_x, Tensor grad_tn_msgs, Tensor grad_nn_msgs, Tensor rr_src, Tensor rr_dst, Tensor tn_rel, Tensor tn_ent, Tensor nn_rel, Tensor nn_ent, int relation_count, int mode) -> Tensor",
}


def header_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"RELM_MP_API\s+[\w\s\*]+?\b(relm_mp_\w+)\s*\(", text))


def test_header_declares_the_op_entry_points() -> None:
    names = header_functions()
    for op in ("fanout_scatter", "fanout_scatter_backward", "fanin_reduce", "fanin_reduce_sum_backward",
               "fanin_reduce_logsumexp_backward"):
        assert f"relm_mp_{op}" in names
        assert f"relm_mp_{op}_workspace_bytes" in names
    assert "relm_mp_build_info" in names


def test_library_exports_every_declared_symbol() -> None:
    lib = capi.lib()
    names = header_functions()
    assert names == set(capi.SIGNATURES), "ctypes binding out of sync with the header"
    for name in names:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert names <= exported
    assert lib.relm_mp_build_info().decode().startswith("lib=relm_mp_b200;arch=sm_100a")
    assert lib.relm_mp_status_string(2) == b"RELM_MP_ERR_INDEX_OUT_OF_RANGE"


def test_workspace_queries_without_gpu() -> None:
    lib = capi.lib()
    e, n, d = 1 << 24, 1 << 20, 64
    plan = lib.relm_mp_plan_bytes(e, n)
    assert plan >= 4 * e + 4 * (n + 1)
    ws = lib.relm_mp_fanin_reduce_workspace_bytes(e, n, d, capi.FLOAT32, 1)
    assert ws > plan
    assert lib.relm_mp_fanout_scatter_workspace_bytes(-1, n, n, d, capi.FLOAT32) == 0
    # LGAN: one workspace for the four entry points; grows with the edge lists and the slots
    g = capi.LganGraph(None, None, 4 << 20, None, None, 1 << 20, None, None, 1 << 20, 1 << 20, 1 << 17)
    small = lib.relm_mp_lgan_workspace_bytes(capi.ctypes.byref(g), 0, d, capi.FLOAT32)
    pooled = lib.relm_mp_lgan_workspace_bytes(capi.ctypes.byref(g), 1 << 24, d, capi.FLOAT32)
    assert small >= 2 * (1 << 20) * d * 4 and pooled > small
    assert lib.relm_mp_lgan_workspace_bytes(None, 0, d, capi.FLOAT32) == 0


def test_torch_library_registers_reference_schemas() -> None:
    assert mp.available()
    for name, schema in REFERENCE_SCHEMAS.items():
        op = getattr(torch.ops.relm_mp, name)
        assert str(op.default._schema) == schema
    info = mp_runtime.parse_build_info(torch.ops.relm_mp.build_info())
    assert info["build_torch"].split(".")[:2] == torch.__version__.split(".")[:2]
    assert info["abi_lane"] == "nonstable"
    assert info["arch"] == "sm_100a"


def test_meta_kernels_give_shapes() -> None:
    x = torch.empty(10, 7, device="meta")
    i = torch.empty(30, dtype=torch.int64, device="meta")
    assert torch.ops.relm_mp.fanout_scatter(x, i, i, 31).shape == (31, 7)
    assert torch.ops.relm_mp.fanin_reduce(x, i, i, 4, 1).shape == (4, 7)
    assert torch.ops.relm_mp.fanin_reduce_sum_backward(x, i, i, 12).shape == (12, 7)
    assert torch.ops.relm_mp.fanin_reduce_logsumexp_backward(x, x, i, i, x, 9).shape == (9, 7)
    assert torch.ops.relm_mp.fanout_scatter_backward(x, i, i, 3).shape == (3, 7)
    # LGAN ops: (relation rows, entity rows, entity rows) and the input gradients
    slots = torch.empty(12, 7, device="meta")
    ar = torch.empty(5, dtype=torch.int64, device="meta")
    e = torch.empty(8, dtype=torch.int64, device="meta")
    x1, tn, nn = torch.ops.relm_mp.lgan_pool_reduce(slots, i[:12], ar, e, e, e, e, e, e, 6, 2)
    assert x1.shape == (5, 7) and tn.shape == (6, 7) and nn.shape == (6, 7)
    g = torch.ops.relm_mp.lgan_pool_reduce_backward(x1, tn, nn, i[:12], ar, e, e, e, e, e, e, 5, 0)
    assert g.shape == (12, 7)
    y, tn2, _ = torch.ops.relm_mp.lgan_relation_graph_step(x1, e, e, e, e, e, e, 4, 0)
    assert y.shape == (5, 7) and tn2.shape == (4, 7)
    assert torch.ops.relm_mp.lgan_relation_graph_step_backward(y, tn2, tn2, e, e, e, e, e, e, 5, 2).shape == (5, 7)


def test_cpu_facade_follows_reference_formulas() -> None:
    """CPU tensors keep the reference's ATen formulas (test_mp_ops.py:171-207)."""

    g = torch.Generator().manual_seed(0)
    x = torch.randn(7, 5, generator=g)
    src, dst = torch.tensor([0, 3, 5, 2, 3]), torch.tensor([4, 1, 0, 2, 3])
    assert np.array_equal(mp.fanout_scatter(x, src, dst, 6).numpy(), oracle.fanout_scatter(x.numpy(), src, dst, 6))
    rel = torch.randn(10, 4, generator=g)
    fs, di = torch.tensor([0, 2, 7, 5, 2, 1]), torch.tensor([1, 0, 2, 2, 1, 0])
    for mode in (0, 1):
        got = mp.fanin_reduce(rel, fs, di, 4, mode).numpy()
        ref = oracle.fanin_reduce(rel.numpy(), fs, di, 4, mode)
        assert np.allclose(got, ref, rtol=1e-5, atol=1e-6, equal_nan=True)


def test_pack_ops_through_the_library() -> None:
    x_a, x_b = torch.randn(5, 3), torch.randn(4, 3)
    src_a, src_b = torch.tensor([0, 2, 4]), torch.tensor([1, 3])
    dst_a, dst_b = torch.tensor([3, 1, 5]), torch.tensor([0, 4])
    x_cat, src, dst = mp.fanout_pack_multi([x_a, x_b], [src_a, src_b], [dst_a, dst_b])
    assert torch.equal(x_cat, torch.cat([x_a, x_b]))
    assert torch.equal(src, torch.tensor([0, 2, 4, 6, 8]))
    assert torch.equal(dst, torch.tensor([3, 1, 5, 0, 4]))
    _, s2, d2 = mp.fanout_pack_from_edges(
        [x_a, x_b], [torch.tensor([0, 2]), torch.tensor([1])], [torch.tensor([1, 0]), torch.tensor([3])],
        [0, 1], [2, 3], [0, 1], [0, 8],
    )
    assert torch.equal(s2, torch.tensor([0, 2, 6]))
    assert torch.equal(d2, torch.tensor([2, 0, 18]))
    _, s3, d3 = mp.fanin_pack_from_edges(
        [x_a, x_b], [torch.tensor([0, 2]), torch.tensor([0])], [torch.tensor([1, 0]), torch.tensor([2])],
        [0, 1], [2, 3], [1, 2], 0,
    )
    assert torch.equal(s3, torch.tensor([1, 5, 7]))
    assert torch.equal(d3, torch.tensor([1, 0, 2]))
