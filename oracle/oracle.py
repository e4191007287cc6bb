"""ctypes front-end for the C oracle (``oracle/relm_mp_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` leg of ``bench.py``. The ``relmo_b200`` package never imports
it. Each wrapper mirrors one reference CPU op (maichmueller/relmo
``src/_ops/mp/mp_ops.cpp``; the C file cites the exact lines) and takes/returns
numpy arrays. bf16 callers upcast to float32 first: the reference has no bf16
accumulation kernel, so the bf16 oracle is the float32 oracle on upcast inputs.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "relm_mp_oracle.c"
BUILD_DIR = HERE / "_build"
LIB_PATH = BUILD_DIR / "librelm_mp_oracle.so"

_LIB: ctypes.CDLL | None = None

_I64P = ctypes.POINTER(ctypes.c_int64)


class OracleIndexError(IndexError):
    """Raised when an index is out of range, as the reference CPU op raises."""

    def __init__(self, which: int, pos: int, value: int, names: tuple[str, str]):
        self.which = which
        self.pos = pos
        self.value = value
        self.name = names[which - 1]
        super().__init__(f"{self.name} index out of bounds at edge {pos}: {value}")


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc (seconds); the output is git-ignored."""

    if LIB_PATH.is_file() and not force and LIB_PATH.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    tmp = str(LIB_PATH) + f".tmp{os.getpid()}"
    subprocess.run(
        ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fno-fast-math", str(SOURCE), "-o", tmp, "-lm"],
        check=True,
    )
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(str(build()))
    return _LIB


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def _suffix(dtype: np.dtype) -> str:
    if dtype == np.float32:
        return "f32"
    if dtype == np.float64:
        return "f64"
    raise TypeError(f"oracle supports float32/float64, got {dtype}")


def _idx(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _vals(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype not in (np.float32, np.float64):
        a = a.astype(np.float32)
    return np.ascontiguousarray(a)


def _call(name: str, names: tuple[str, str], *args) -> None:
    bad_pos = ctypes.c_int64(-1)
    bad_val = ctypes.c_int64(0)
    fn = getattr(lib(), name)
    fn.restype = ctypes.c_int
    rc = fn(*args, ctypes.byref(bad_pos), ctypes.byref(bad_val))
    if rc != 0:
        raise OracleIndexError(rc, bad_pos.value, bad_val.value, names)


def fanout_scatter(x, src_global_idx, flat_dst, out_rows: int) -> np.ndarray:
    x = _vals(x)
    src = _idx(src_global_idx)
    dst = _idx(flat_dst)
    emb = x.shape[1]
    out = np.empty((int(out_rows), emb), dtype=x.dtype)
    _call(
        f"relm_oracle_fanout_scatter_{_suffix(x.dtype)}",
        ("src_global_idx", "flat_dst"),
        _ptr(x), ctypes.c_int64(x.shape[0]), ctypes.c_int64(emb), _ptr(src), _ptr(dst),
        ctypes.c_int64(src.shape[0]), ctypes.c_int64(int(out_rows)), _ptr(out),
    )
    return out


def fanout_scatter_backward(grad_out, src_global_idx, flat_dst, x_rows: int) -> np.ndarray:
    g = _vals(grad_out)
    src = _idx(src_global_idx)
    dst = _idx(flat_dst)
    emb = g.shape[1]
    out = np.empty((int(x_rows), emb), dtype=g.dtype)
    _call(
        f"relm_oracle_fanout_scatter_backward_{_suffix(g.dtype)}",
        ("src_global_idx", "flat_dst"),
        _ptr(g), ctypes.c_int64(g.shape[0]), ctypes.c_int64(emb), _ptr(src), _ptr(dst),
        ctypes.c_int64(src.shape[0]), ctypes.c_int64(int(x_rows)), _ptr(out),
    )
    return out


def fanin_reduce(rel_flat, flat_src, dst_idx, dim_size: int, mode: int) -> np.ndarray:
    rel = _vals(rel_flat)
    src = _idx(flat_src)
    dst = _idx(dst_idx)
    emb = rel.shape[1]
    out = np.empty((int(dim_size), emb), dtype=rel.dtype)
    common = (
        _ptr(rel), ctypes.c_int64(rel.shape[0]), ctypes.c_int64(emb), _ptr(src), _ptr(dst),
        ctypes.c_int64(src.shape[0]), ctypes.c_int64(int(dim_size)), _ptr(out),
    )
    if int(mode) == 0:
        _call(f"relm_oracle_fanin_sum_{_suffix(rel.dtype)}", ("flat_src", "dst_idx"), *common)
    elif int(mode) == 1:
        scratch = np.empty_like(out)
        _call(
            f"relm_oracle_fanin_logsumexp_{_suffix(rel.dtype)}",
            ("flat_src", "dst_idx"),
            *common,
            _ptr(scratch),
        )
    else:
        raise ValueError("Unsupported fanin_reduce mode. Supported: 0=sum, 1=logsumexp.")
    return out


def fanin_reduce_sum_backward(grad_out, flat_src, dst_idx, rel_rows: int) -> np.ndarray:
    g = _vals(grad_out)
    src = _idx(flat_src)
    dst = _idx(dst_idx)
    emb = g.shape[1]
    out = np.empty((int(rel_rows), emb), dtype=g.dtype)
    _call(
        f"relm_oracle_fanin_sum_backward_{_suffix(g.dtype)}",
        ("flat_src", "dst_idx"),
        _ptr(g), ctypes.c_int64(g.shape[0]), ctypes.c_int64(emb), _ptr(src), _ptr(dst),
        ctypes.c_int64(src.shape[0]), ctypes.c_int64(int(rel_rows)), _ptr(out),
    )
    return out


def fanin_reduce_logsumexp_backward(grad_out, rel_flat, flat_src, dst_idx, out, rel_rows: int) -> np.ndarray:
    g = _vals(grad_out)
    rel = _vals(rel_flat).astype(g.dtype, copy=False)
    o = _vals(out).astype(g.dtype, copy=False)
    src = _idx(flat_src)
    dst = _idx(dst_idx)
    emb = g.shape[1]
    res = np.empty((int(rel_rows), emb), dtype=g.dtype)
    _call(
        f"relm_oracle_fanin_logsumexp_backward_{_suffix(g.dtype)}",
        ("flat_src", "dst_idx"),
        _ptr(g), _ptr(np.ascontiguousarray(rel)), _ptr(np.ascontiguousarray(o)),
        ctypes.c_int64(o.shape[0]), ctypes.c_int64(emb), _ptr(src), _ptr(dst),
        ctypes.c_int64(src.shape[0]), ctypes.c_int64(int(rel_rows)), _ptr(res),
    )
    return res


LGAN_INDEX_NAMES = ("rr_src", "rr_dst", "tn_rel", "tn_ent", "nn_rel", "nn_ent", "slot_to_relation_instance")


def _lgan_mode(mode: int, op: str) -> int:
    if int(mode) not in (0, 2):
        raise ValueError(f"{op} supports only mode 0=sum or 2=mean.")
    return 1 if int(mode) == 2 else 0


def _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent):
    ix = [_idx(a) for a in (rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)]
    args = []
    for k in range(0, 6, 2):
        args += [_ptr(ix[k]), _ptr(ix[k + 1]), ctypes.c_int64(ix[k].shape[0])]
    return ix, args


def lgan_relation_graph_step(x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, entity_dim_size: int, mode: int):
    """mp_ops.cpp:3627-3656 (ATen formulas): (x + agg_rr(x), agg_tn(x1), agg_nn(x1))."""

    mean = _lgan_mode(mode, "lgan_relation_graph_step")
    x = _vals(x)
    ix, graph = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
    rows, emb = x.shape
    x1 = np.empty_like(x)
    tn = np.empty((int(entity_dim_size), emb), dtype=x.dtype)
    nn = np.empty_like(tn)
    _call(
        f"relm_oracle_lgan_relation_graph_step_{_suffix(x.dtype)}", LGAN_INDEX_NAMES,
        _ptr(x), ctypes.c_int64(rows), ctypes.c_int64(emb), *graph, ctypes.c_int64(int(entity_dim_size)),
        ctypes.c_int(mean), _ptr(x1), _ptr(tn), _ptr(nn),
    )
    return x1, tn, nn


def lgan_relation_graph_step_backward(grad_x, grad_tn, grad_nn, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                                      relation_count: int, mode: int):
    """mp_ops.cpp:3715-3743 (ATen formulas)."""

    mean = _lgan_mode(mode, "lgan_relation_graph_step_backward")
    gx = _vals(grad_x)
    gtn = _vals(grad_tn).astype(gx.dtype, copy=False)
    gnn = _vals(grad_nn).astype(gx.dtype, copy=False)
    ix, graph = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
    emb = gx.shape[1]
    out = np.empty((int(relation_count), emb), dtype=gx.dtype)
    gtn = np.ascontiguousarray(gtn)
    gnn = np.ascontiguousarray(gnn)
    _call(
        f"relm_oracle_lgan_relation_graph_step_backward_{_suffix(gx.dtype)}", LGAN_INDEX_NAMES,
        _ptr(gx), _ptr(gtn), _ptr(gnn), ctypes.c_int64(gtn.shape[0]), ctypes.c_int64(emb), *graph,
        ctypes.c_int64(int(relation_count)), ctypes.c_int(mean), _ptr(out),
    )
    return out


def lgan_pool_reduce(slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel,
                     tn_ent, nn_rel, nn_ent, entity_dim_size: int, mode: int):
    """mp_ops.cpp:3424-3469 (ATen formulas): pool the slots to relation instances
    (sum / max(arity, 1)), then the relation graph step."""

    mean = _lgan_mode(mode, "lgan_pool_reduce")
    slots = _vals(slot_messages)
    s2r = _idx(slot_to_relation_instance)
    ar = _idx(relation_instance_arities)
    ix, graph = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
    emb = slots.shape[1]
    x1 = np.empty((ar.shape[0], emb), dtype=slots.dtype)
    tn = np.empty((int(entity_dim_size), emb), dtype=slots.dtype)
    nn = np.empty_like(tn)
    _call(
        f"relm_oracle_lgan_pool_reduce_{_suffix(slots.dtype)}", LGAN_INDEX_NAMES,
        _ptr(slots), ctypes.c_int64(slots.shape[0]), ctypes.c_int64(emb), _ptr(s2r), _ptr(ar),
        ctypes.c_int64(ar.shape[0]), *graph, ctypes.c_int64(int(entity_dim_size)), ctypes.c_int(mean),
        _ptr(x1), _ptr(tn), _ptr(nn),
    )
    return x1, tn, nn


def lgan_pool_reduce_backward(grad_x, grad_tn, grad_nn, slot_to_relation_instance, relation_instance_arities,
                              rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, relation_count: int, mode: int):
    """mp_ops.cpp:3527-3572 (ATen formulas)."""

    mean = _lgan_mode(mode, "lgan_pool_reduce_backward")
    gx = _vals(grad_x)
    gtn = np.ascontiguousarray(_vals(grad_tn).astype(gx.dtype, copy=False))
    gnn = np.ascontiguousarray(_vals(grad_nn).astype(gx.dtype, copy=False))
    s2r = _idx(slot_to_relation_instance)
    ar = _idx(relation_instance_arities)
    ix, graph = _lgan_graph(rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
    emb = gx.shape[1]
    out = np.empty((s2r.shape[0], emb), dtype=gx.dtype)
    _call(
        f"relm_oracle_lgan_pool_reduce_backward_{_suffix(gx.dtype)}", LGAN_INDEX_NAMES,
        _ptr(gx), _ptr(gtn), _ptr(gnn), ctypes.c_int64(gtn.shape[0]), ctypes.c_int64(emb), _ptr(s2r),
        ctypes.c_int64(s2r.shape[0]), _ptr(ar), *graph, ctypes.c_int64(int(relation_count)), ctypes.c_int(mean),
        _ptr(out),
    )
    return out
