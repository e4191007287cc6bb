"""Generate golden vectors from the reference's own CPU op library.

Run in a process of its own (the reference library registers the ``relm_mp``
torch namespace, the same one ``relmo_b200`` registers):

    python oracle/build_ref.py          # builds oracle/_ref/relm_mp_ref.so
    python tests/golden/make_golden.py  # writes tests/golden/*.npz
    python tests/golden/make_golden.py --only-lgan   # ref_lgan.npz alone
    python tests/golden/make_golden.py --only-pack   # ref_lgan.npz and ref_pack.npz

Inputs come from the reference's own test fixtures
(``tests/python/test_mp_ops.py:171-347`` of maichmueller/relmo: the literal index
vectors, with seeded values instead of unseeded ``randn``), a set of edge cases
(empty inputs, zero rows, duplicate slots, non-finite values, out-of-range
indices) and the cfg1 parity workload. Outputs are what
``torch.ops.relm_mp.*`` of the reference returns on CPU.

Files:
* ``ref_cases.npz`` - small cases, inputs and outputs stored in full.
* ``ref_lgan.npz`` - the LGAN ops (``lgan_pool_reduce``, ``lgan_relation_graph_step``
  and their backwards, sum and mean modes): the literal fixtures of
  ``tests/python/test_flat_lgan_relational_gnn.py:270-626`` of maichmueller/relmo
  (seeded values where the test draws unseeded ``randn``), edge cases and a
  seeded random case; inputs and outputs stored in full. Tuple outputs are
  stored as ``<case>__out0``, ``__out1``, ...
* ``ref_pack.npz`` - the four pack ops (``fanout_pack_multi``, ``fanin_pack_multi``,
  ``fanout_pack_from_edges``, ``fanin_pack_from_edges``; mp_ops.cpp:412-570,
  2511-2773): one part, several parts, more than 64 parts, empty parts, strided
  index views, no edge parts, both ``fanin_pack_from_edges`` modes, and the
  reference's argument errors. Tensor-list arguments are stored as
  ``<case>__arg<i>_<k>``; outputs as ``<case>__out0..2``.
* ``ref_cfg1.npz`` - cfg1 (N=2000, D=32, E=20000, seed 0). Inputs are regenerated
  from the seed and pinned by SHA-256; outputs stored in full when they are
  [N, D], by SHA-256 when bit-exact [E, D], and by a row sample plus float64
  checksums for the [E, D] logsumexp gradient.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from relmo_b200 import workloads  # noqa: E402  (pure-python module, loads no library)

REF_LIB = ROOT / "oracle" / "_ref" / "relm_mp_ref.so"


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()


def load_reference():
    if not REF_LIB.is_file():
        raise SystemExit(f"{REF_LIB} missing: run python oracle/build_ref.py first")
    torch.ops.load_library(str(REF_LIB))
    return torch.ops.relm_mp


def small_cases():
    """(name, op, args) with the reference test fixtures and edge cases."""

    g = torch.Generator().manual_seed(1234)

    def randn(*shape, dtype=torch.float32):
        return torch.randn(*shape, generator=g, dtype=torch.float64).to(dtype)

    def idx(*v):
        return torch.tensor(v, dtype=torch.int64)

    cases = []
    # test_mp_ops.py:171-188 (python fallback fixture)
    cases.append(("fallback_fanout", "fanout_scatter", [randn(6, 3), idx(0, 4, 1), idx(3, 0, 1), 5]))
    for mode in (0, 1):
        cases.append((f"fallback_fanin_m{mode}", "fanin_reduce",
                      [randn(8, 3), idx(0, 2, 4, 1), idx(2, 0, 1, 0), 4, mode]))
    # test_mp_ops.py:191-207
    cases.append(("parity_fanout", "fanout_scatter", [randn(7, 5), idx(0, 3, 5, 2, 3), idx(4, 1, 0, 2, 3), 6]))
    # test_mp_ops.py:210-230: grad of out.sum() -> grad_out = ones
    cases.append(("grad_fanout_bwd", "fanout_scatter_backward",
                  [torch.ones(5, 4), idx(0, 5, 2, 6), idx(1, 0, 3, 2), 8]))
    # test_mp_ops.py:233-252 (empty destination row 3)
    for mode in (0, 1):
        cases.append((f"parity_fanin_m{mode}", "fanin_reduce",
                      [randn(10, 4), idx(0, 2, 7, 5, 2, 1), idx(1, 0, 2, 2, 1, 0), 4, mode]))
    # test_mp_ops.py:255-281 (dim_size 5 with two empty rows) forward and backward
    rel = randn(12, 3)
    fs, di = idx(0, 1, 8, 4, 9, 10), idx(2, 0, 1, 1, 0, 2)
    cases.append(("grad_fanin_m0_fwd", "fanin_reduce", [rel, fs, di, 5, 0]))
    cases.append(("grad_fanin_m0_bwd", "fanin_reduce_sum_backward", [torch.ones(5, 3), fs, di, 12]))
    cases.append(("grad_fanin_m1_fwd", "fanin_reduce", [rel, fs, di, 5, 1]))
    cases.append(("grad_fanin_m1_bwd", "fanin_reduce_logsumexp_backward",
                  [torch.ones(5, 3), rel, fs, di, "@grad_fanin_m1_fwd", 12]))
    # test_mp_ops.py:302-347 gradcheck fixtures, in float64, with random upstream grads
    cases.append(("f64_fanout", "fanout_scatter", [randn(6, 3, dtype=torch.float64), idx(0, 5, 2, 1), idx(1, 0, 3, 2), 5]))
    cases.append(("f64_fanout_bwd", "fanout_scatter_backward",
                  [randn(5, 3, dtype=torch.float64), idx(0, 5, 2, 1), idx(1, 0, 3, 2), 6]))
    rel64 = randn(8, 4, dtype=torch.float64)
    cases.append(("f64_sum", "fanin_reduce", [rel64, idx(0, 2, 5, 7, 1), idx(1, 0, 3, 2, 0), 5, 0]))
    cases.append(("f64_sum_bwd", "fanin_reduce_sum_backward",
                  [randn(5, 4, dtype=torch.float64), idx(0, 2, 5, 7, 1), idx(1, 0, 3, 2, 0), 8]))
    fs6, di6 = idx(0, 2, 5, 7, 1, 3), idx(1, 0, 3, 2, 0, 1)
    cases.append(("f64_lse", "fanin_reduce", [rel64, fs6, di6, 4, 1]))
    cases.append(("f64_lse_bwd", "fanin_reduce_logsumexp_backward",
                  [randn(4, 4, dtype=torch.float64), rel64, fs6, di6, "@f64_lse", 8]))
    # edge cases
    e0 = torch.empty(0, dtype=torch.int64)
    cases.append(("empty_edges_fanout", "fanout_scatter", [randn(4, 3), e0, e0, 3]))
    cases.append(("empty_edges_sum", "fanin_reduce", [randn(4, 3), e0, e0, 3, 0]))
    cases.append(("empty_edges_lse", "fanin_reduce", [randn(4, 3), e0, e0, 3, 1]))
    cases.append(("zero_rows_fanout", "fanout_scatter", [randn(4, 3), idx(1, 2), idx(0, 1), 0]))
    cases.append(("zero_dim_lse", "fanin_reduce", [randn(4, 3), idx(1, 2), idx(0, 1), 0, 1]))
    cases.append(("dup_slots_fanout", "fanout_scatter",
                  [randn(6, 4), idx(0, 1, 2, 3, 4, 5), idx(2, 0, 2, 1, 2, 0), 4]))
    cases.append(("dup_src_sum_bwd", "fanin_reduce_sum_backward",
                  [randn(3, 4), idx(1, 1, 0, 1, 3), idx(0, 2, 1, 1, 2), 5]))
    nf = randn(5, 3)
    nf[1, 0] = float("nan")
    nf[2, 1] = float("inf")
    nf[3, 2] = float("-inf")
    nf[4, :] = float("-inf")
    cases.append(("nonfinite_lse", "fanin_reduce", [nf, idx(0, 1, 2, 3, 4, 4), idx(0, 0, 1, 1, 2, 3), 4, 1]))
    cases.append(("nonfinite_sum", "fanin_reduce", [nf, idx(0, 1, 2, 3, 4, 4), idx(0, 0, 1, 1, 2, 3), 4, 0]))
    cases.append(("wide_emb_sum", "fanin_reduce",
                  [randn(40, 300), torch.randint(0, 40, (90,), generator=g), torch.randint(0, 17, (90,), generator=g), 17, 0]))
    cases.append(("wide_emb_lse", "fanin_reduce",
                  [randn(40, 300), torch.randint(0, 40, (90,), generator=g), torch.randint(0, 17, (90,), generator=g), 17, 1]))
    # out-of-range indices: the reference CPU op raises
    cases.append(("oob_fanout_src", "fanout_scatter", [randn(4, 3), idx(0, 4), idx(0, 1), 3]))
    cases.append(("oob_fanout_dst", "fanout_scatter", [randn(4, 3), idx(0, 1), idx(0, 3), 3]))
    cases.append(("oob_fanout_neg", "fanout_scatter", [randn(4, 3), idx(-1, 1), idx(0, 1), 3]))
    cases.append(("oob_sum_dst", "fanin_reduce", [randn(4, 3), idx(0, 1), idx(0, 5), 3, 0]))
    cases.append(("oob_sum_src", "fanin_reduce", [randn(4, 3), idx(0, 9), idx(0, 1), 3, 0]))
    cases.append(("oob_lse_dst", "fanin_reduce", [randn(4, 3), idx(0, 1), idx(0, 5), 3, 1]))
    cases.append(("oob_fanout_bwd_src", "fanout_scatter_backward", [randn(3, 3), idx(0, 7), idx(0, 1), 4]))
    cases.append(("oob_sum_bwd_dst", "fanin_reduce_sum_backward", [randn(3, 3), idx(0, 1), idx(0, 3), 4]))
    return cases


def run_small(ops) -> dict[str, np.ndarray]:
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    results: dict[str, torch.Tensor] = {}
    for name, op, args in small_cases():
        call_args = [results[a[1:]] if isinstance(a, str) and a.startswith("@") else a for a in args]
        entry = {"op": op, "args": []}
        for i, a in enumerate(call_args):
            if isinstance(a, torch.Tensor):
                key = f"{name}__arg{i}"
                arrays[key] = a.numpy()
                entry["args"].append({"tensor": key})
            else:
                entry["args"].append({"int": int(a)})
        try:
            out = getattr(ops, op)(*call_args)
            results[name] = out
            arrays[f"{name}__out"] = out.numpy()
            entry["raises"] = None
        except Exception as exc:  # the reference raises for out-of-range indices
            entry["raises"] = type(exc).__name__
            entry["message"] = str(exc).splitlines()[0]
        meta[name] = entry
    arrays["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    return arrays


def lgan_cases():
    """(name, op, args) for the LGAN ops; "@case:k" refers to output k of an earlier case."""

    g = torch.Generator().manual_seed(4321)

    def randn(*shape, dtype=torch.float32):
        return torch.randn(*shape, generator=g, dtype=torch.float64).to(dtype)

    def idx(*v, dtype=torch.int64):
        return torch.tensor(v, dtype=dtype)

    def graph(rr, tn, nn, dtype=torch.int64):
        return [idx(*rr[0], dtype=dtype), idx(*rr[1], dtype=dtype), idx(*tn[0], dtype=dtype),
                idx(*tn[1], dtype=dtype), idx(*nn[0], dtype=dtype), idx(*nn[1], dtype=dtype)]

    cases = []
    # test_flat_lgan_relational_gnn.py:270-311 (pool, literal values)
    slots = torch.tensor([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0], [2.0, 0.0], [0.0, 2.0]])
    g1 = graph(((0, 1), (1, 2)), ((0, 1, 2), (0, 1, 2)), ((1, 2), (2, 4)))
    for mode, tag in ((0, "sum"), (2, "mean")):
        cases.append((f"pool_lit_{tag}", "lgan_pool_reduce", [slots, idx(0, 0, 1, 1, 2), idx(2, 2, 1), *g1, 5, mode]))
        cases.append((f"pool_lit_{tag}_bwd", "lgan_pool_reduce_backward",
                      [torch.ones(3, 2), torch.ones(5, 2), torch.ones(5, 2), idx(0, 0, 1, 1, 2), idx(2, 2, 1), *g1,
                       3, mode]))
    # test_flat_lgan_relational_gnn.py:534-585 (indices of the CUDA backward test, seeded values)
    s2r = idx(0, 0, 1, 1, 1, 2, 3, 3, 4)
    ar = idx(2, 3, 1, 2, 1)
    g2 = graph(((0, 1, 2, 3), (1, 2, 3, 4)), ((0, 2, 4), (0, 3, 5)), ((1, 3, 4), (2, 4, 6)))
    for mode, tag in ((0, "sum"), (2, "mean")):
        cases.append((f"pool_bwdfix_{tag}", "lgan_pool_reduce", [randn(9, 4), s2r, ar, *g2, 7, mode]))
        cases.append((f"pool_bwdfix_{tag}_bwd", "lgan_pool_reduce_backward",
                      [randn(5, 4), randn(7, 4), randn(7, 4), s2r, ar, *g2, 5, mode]))
    # test_flat_lgan_relational_gnn.py:587-626 (graph step, literal values)
    x = torch.tensor([[0.5, 0.5], [1.0, 0.5], [0.0, 2.0]])
    for mode, tag in ((0, "sum"), (2, "mean")):
        cases.append((f"step_lit_{tag}", "lgan_relation_graph_step", [x, *g1, 5, mode]))
        cases.append((f"step_lit_{tag}_bwd", "lgan_relation_graph_step_backward",
                      [randn(3, 2), randn(5, 2), randn(5, 2), *g1, 3, mode]))
    # repeated targets (mean counts > 1), a relation without slots, arity 0 (clamped to 1)
    g3 = graph(((0, 1, 2, 3, 3, 0), (1, 1, 1, 0, 2, 2)), ((0, 1, 2, 3, 1), (0, 0, 0, 2, 2)),
               ((3, 2, 2), (1, 1, 3)))
    for mode, tag in ((0, "sum"), (2, "mean")):
        cases.append((f"dups_{tag}", "lgan_pool_reduce",
                      [randn(6, 5), idx(0, 1, 1, 3, 3, 3), idx(1, 2, 0, 3), *g3, 4, mode]))
        cases.append((f"dups_{tag}_bwd", "lgan_pool_reduce_backward",
                      [randn(4, 5), randn(4, 5), randn(4, 5), idx(0, 1, 1, 3, 3, 3), idx(1, 2, 0, 3), *g3, 4,
                       mode]))
        cases.append((f"dups_step_{tag}", "lgan_relation_graph_step", [randn(4, 5), *g3, 4, mode]))
        cases.append((f"dups_step_{tag}_bwd", "lgan_relation_graph_step_backward",
                      [randn(4, 5), randn(4, 5), randn(4, 5), *g3, 4, mode]))
    # empty edge sets, zero entities, float64, int32 indices
    e0 = ((), ())
    g4 = graph(e0, ((0, 1), (1, 0)), e0)
    cases.append(("empty_rr_nn", "lgan_relation_graph_step", [randn(3, 4), *g4, 2, 2]))
    cases.append(("empty_rr_nn_bwd", "lgan_relation_graph_step_backward",
                  [randn(3, 4), randn(2, 4), randn(2, 4), *g4, 3, 2]))
    g5 = graph(((0,), (1,)), e0, e0)
    cases.append(("zero_entities", "lgan_pool_reduce", [randn(3, 4), idx(0, 1, 1), idx(1, 2), *g5, 0, 0]))
    cases.append(("no_slots", "lgan_pool_reduce", [torch.zeros(0, 4), idx(), idx(1, 2), *g5, 2, 2]))
    cases.append(("f64_pool_mean", "lgan_pool_reduce",
                  [randn(9, 3, dtype=torch.float64), s2r, ar, *g2, 7, 2]))
    cases.append(("f64_pool_mean_bwd", "lgan_pool_reduce_backward",
                  [randn(5, 3, dtype=torch.float64), randn(7, 3, dtype=torch.float64),
                   randn(7, 3, dtype=torch.float64), s2r, ar, *g2, 5, 2]))
    g2i = graph(((0, 1, 2, 3), (1, 2, 3, 4)), ((0, 2, 4), (0, 3, 5)), ((1, 3, 4), (2, 4, 6)), dtype=torch.int32)
    cases.append(("int32_step_mean", "lgan_relation_graph_step", [randn(5, 4), *g2i, 7, 2]))
    # seeded random graph
    R, N, S, D = 50, 20, 120, 16
    rnd = [torch.randint(0, R, (200,), generator=g), torch.randint(0, R, (200,), generator=g),
           torch.randint(0, R, (100,), generator=g), torch.randint(0, N, (100,), generator=g),
           torch.randint(0, R, (80,), generator=g), torch.randint(0, N, (80,), generator=g)]
    s2r_r = torch.randint(0, R, (S,), generator=g)
    ar_r = torch.randint(0, 4, (R,), generator=g)
    for mode, tag in ((0, "sum"), (2, "mean")):
        cases.append((f"random_{tag}", "lgan_pool_reduce", [randn(S, D), s2r_r, ar_r, *rnd, N, mode]))
        cases.append((f"random_{tag}_bwd", "lgan_pool_reduce_backward",
                      [randn(R, D), randn(N, D), randn(N, D), s2r_r, ar_r, *rnd, R, mode]))
    # out-of-range indices: the reference raises
    cases.append(("oob_tn_ent", "lgan_relation_graph_step", [randn(3, 2), *graph(e0, ((0,), (5,)), e0), 5, 0]))
    cases.append(("oob_rr_src", "lgan_relation_graph_step", [randn(3, 2), *graph(((-1,), (0,)), e0, e0), 5, 0]))
    cases.append(("oob_slot", "lgan_pool_reduce", [randn(2, 2), idx(0, 3), idx(1, 1), *graph(e0, e0, e0), 2, 0]))
    cases.append(("bad_mode", "lgan_relation_graph_step", [randn(3, 2), *g1, 5, 1]))
    return cases


def run_lgan(ops) -> dict[str, np.ndarray]:
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    for name, op, args in lgan_cases():
        entry = {"op": op, "args": []}
        for i, a in enumerate(args):
            if isinstance(a, torch.Tensor):
                key = f"{name}__arg{i}"
                arrays[key] = a.numpy()
                entry["args"].append({"tensor": key})
            else:
                entry["args"].append({"int": int(a)})
        try:
            out = getattr(ops, op)(*args)
            outs = out if isinstance(out, (tuple, list)) else (out,)
            for k, o in enumerate(outs):
                arrays[f"{name}__out{k}"] = o.numpy()
            entry["outputs"] = len(outs)
            entry["raises"] = None
        except Exception as exc:  # the reference raises for out-of-range indices and bad modes
            entry["raises"] = type(exc).__name__
            entry["message"] = str(exc).splitlines()[0]
        meta[name] = entry
    arrays["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    return arrays


def pack_cases():
    """(name, op, args) for the pack ops; list arguments are Python lists."""

    g = torch.Generator().manual_seed(77)

    def randn(*shape):
        return torch.randn(*shape, generator=g)

    def ridx(n, hi):
        return torch.randint(0, max(hi, 1), (n,), generator=g)

    cases = []
    # fanout_pack_multi / fanin_pack_multi: (value parts, gather-index parts, other-index parts)
    for name, parts in (("one", [(5, 7)]), ("three", [(4, 3), (0, 0), (6, 9)]), ("many", [(3, 2)] * 70)):
        xs = [randn(r, 4) for r, _ in parts]
        src = [ridx(e, r) for r, e in parts]
        dst = [ridx(e, 50) for _, e in parts]
        cases.append((f"fanout_multi_{name}", "fanout_pack_multi", [xs, src, dst]))
        cases.append((f"fanin_multi_{name}", "fanin_pack_multi", [xs, src, dst]))
    base = ridx(40, 6)
    cases.append(("fanout_multi_strided", "fanout_pack_multi",
                  [[randn(6, 2), randn(3, 2)], [base[::2], base[1:8:3] % 3], [ridx(20, 9), ridx(3, 9)]]))
    cases.append(("fanout_multi_len_mismatch", "fanout_pack_multi", [[randn(3, 2)], [ridx(4, 3)], [ridx(2, 3)]]))
    cases.append(("fanin_multi_emb_mismatch", "fanin_pack_multi",
                  [[randn(3, 2), randn(3, 5)], [ridx(2, 3), ridx(2, 3)], [ridx(2, 3), ridx(2, 3)]]))

    # fanout_pack_from_edges(x_parts, edge_src, edge_dst, src_part_ids, arity, pos, slot_offsets)
    def from_edges(n_parts, n_x=3, n_edges=5):
        xs = [randn(4 + i, 3) for i in range(n_x)]
        src, dst, part, ar, pos, off = [], [], [], [], [], []
        for i in range(n_parts):
            k = i % n_x
            a = 1 + i % 3
            e = 0 if i % 11 == 5 else n_edges
            src.append(ridx(e, 4 + k))
            dst.append(ridx(e, 8))
            part.append(k)
            ar.append(a)
            pos.append(i % a)
            off.append(100 * i)
        return xs, src, dst, part, ar, pos, off

    for name, n in (("one", 1), ("six", 6), ("many", 67), ("none", 0)):
        xs, src, dst, part, ar, pos, off = from_edges(n)
        cases.append((f"fanout_edges_{name}", "fanout_pack_from_edges", [xs, src, dst, part, ar, pos, off]))
        for mode in (0, 1):
            cases.append((f"fanin_edges_{name}_m{mode}", "fanin_pack_from_edges", [xs, src, dst, part, ar, pos, mode]))
    xs, src, dst, part, ar, pos, off = from_edges(3)
    cases.append(("fanout_edges_bad_part", "fanout_pack_from_edges", [xs, src, dst, [0, 5, 1], ar, pos, off]))
    cases.append(("fanout_edges_bad_pos", "fanout_pack_from_edges", [xs, src, dst, part, [1, 2, 3], [0, 2, 1], off]))
    cases.append(("fanout_edges_zero_arity", "fanout_pack_from_edges", [xs, src, dst, part, [1, 0, 3], [0, 0, 1], off]))
    cases.append(("fanin_edges_bad_mode", "fanin_pack_from_edges", [xs, src, dst, part, ar, pos, 2]))
    cases.append(("fanin_edges_bad_pos", "fanin_pack_from_edges", [xs, src, dst, part, [1, 2, 3], [0, 2, 1], 0]))
    return cases


def run_pack(ops) -> dict[str, np.ndarray]:
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}
    for name, op, args in pack_cases():
        entry = {"op": op, "args": []}
        for i, a in enumerate(args):
            if isinstance(a, list) and a and isinstance(a[0], torch.Tensor):
                keys = []
                for k, t in enumerate(a):
                    key = f"{name}__arg{i}_{k}"
                    arrays[key] = t.contiguous().numpy()
                    keys.append(key)
                entry["args"].append({"tensors": keys})
            elif isinstance(a, list):
                entry["args"].append({"ints": [int(v) for v in a]})
            else:
                entry["args"].append({"int": int(a)})
        try:
            outs = getattr(ops, op)(*args)
            for k, o in enumerate(outs):
                arrays[f"{name}__out{k}"] = o.numpy()
            entry["raises"] = None
        except Exception as exc:  # the reference's argument checks
            entry["raises"] = type(exc).__name__
            entry["message"] = str(exc).splitlines()[0]
        meta[name] = entry
    arrays["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    return arrays


def run_cfg1(ops) -> dict[str, np.ndarray]:
    wl = workloads.cfg1(seed=0)
    arrays: dict[str, np.ndarray] = {}
    inputs = {
        "x": wl.x, "src": wl.src, "dst": wl.dst, "msgs": wl.msgs, "flat_dst": wl.flat_dst,
        "grad_slots": wl.grad_slots, "grad_nodes": wl.grad_nodes,
    }
    meta = {"input_sha256": {k: sha(v) for k, v in inputs.items()}}
    fan = ops.fanout_scatter(wl.x, wl.src, wl.flat_dst, wl.out_rows)
    fan_bwd = ops.fanout_scatter_backward(wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0))
    fsum = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    flse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    sum_bwd = ops.fanin_reduce_sum_backward(wl.grad_nodes, wl.flat_src, wl.dst, wl.msgs.size(0))
    lse_bwd = ops.fanin_reduce_logsumexp_backward(
        wl.grad_nodes, wl.msgs, wl.flat_src, wl.dst, flse, wl.msgs.size(0)
    )
    meta["out_sha256"] = {"fanout_fwd": sha(fan), "fanin_sum_bwd": sha(sum_bwd)}
    arrays["fanout_bwd"] = fan_bwd.numpy()
    arrays["fanin_sum_fwd"] = fsum.numpy()
    arrays["fanin_lse_fwd"] = flse.numpy()
    rows = np.arange(0, lse_bwd.size(0), 10)
    arrays["fanin_lse_bwd_rows"] = rows
    arrays["fanin_lse_bwd_sample"] = lse_bwd.numpy()[rows]
    d = lse_bwd.double()
    meta["fanin_lse_bwd_checksum"] = {"sum": float(d.sum()), "sumsq": float((d * d).sum())}
    arrays["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    return arrays


def main() -> int:
    torch.set_num_threads(1)
    ops = load_reference()
    info = ops.build_info()
    lgan = run_lgan(ops)
    lgan["__build_info__"] = np.frombuffer(info.encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "ref_lgan.npz", **lgan)
    print("wrote", HERE / "ref_lgan.npz")
    if "--only-lgan" in sys.argv:
        return 0
    pack = run_pack(ops)
    pack["__build_info__"] = np.frombuffer(info.encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "ref_pack.npz", **pack)
    print("wrote", HERE / "ref_pack.npz")
    if "--only-pack" in sys.argv:
        return 0
    small = run_small(ops)
    small["__build_info__"] = np.frombuffer(info.encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "ref_cases.npz", **small)
    cfg = run_cfg1(ops)
    cfg["__build_info__"] = np.frombuffer(info.encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "ref_cfg1.npz", **cfg)
    print("wrote", HERE / "ref_cases.npz", HERE / "ref_cfg1.npz", "from", info)
    return 0


if __name__ == "__main__":
    sys.exit(main())
