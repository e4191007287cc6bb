"""CPU formulas of the fan-out / fan-in ops and the index pack helpers.

These are the reference's ATen formulas (relmo ``src/relmo/ops/mp_pack.py``:
``fanout_scatter_python`` 19-30, ``fanin_reduce_python`` 33-63, pack helpers
66-292), used only for CPU tensors and for the pack ops when the library is
not loaded. CUDA tensors never reach this module from ``relmo_b200.ops.mp``.
"""

from __future__ import annotations

from .mp_constants import MODE_LOGSUMEXP, MODE_SUM
from .mp_runtime import torch


def _require_rank(op: str, name: str, t, rank: int) -> None:
    if t.dim() != rank:
        raise ValueError(f"{op} expects {name} to be rank-{rank}, got shape {tuple(t.shape)}.")


def _require_int64(op: str, name: str, t) -> None:
    if t.dtype != torch.int64:
        raise ValueError(f"{op} expects {name} to have dtype int64, got {t.dtype}.")


def _cat(parts):
    return parts[0] if len(parts) == 1 else torch.cat(list(parts), dim=0)


def _empty_index(device):
    return torch.empty(0, device=device, dtype=torch.int64)


def fanout_scatter_python(x_cat, src_global_idx, flat_dst, out_rows: int):
    out = x_cat.new_zeros((int(out_rows), int(x_cat.size(-1))))
    if src_global_idx.numel() == 0 or int(out_rows) == 0:
        return out
    out.index_copy_(0, flat_dst, x_cat.index_select(0, src_global_idx))
    return out


def fanin_reduce_python(rel_flat, flat_src, dst_idx, dim_size: int, mode: int):
    emb = int(rel_flat.size(-1))
    if mode == MODE_SUM:
        out = rel_flat.new_zeros((int(dim_size), emb))
        if flat_src.numel() == 0 or int(dim_size) == 0:
            return out
        out.index_add_(0, dst_idx, rel_flat.index_select(0, flat_src))
        return out
    if mode == MODE_LOGSUMEXP:
        out = rel_flat.new_full((int(dim_size), emb), float("-inf"))
        if flat_src.numel() == 0 or int(dim_size) == 0:
            return out
        values = rel_flat.index_select(0, flat_src)
        index = dst_idx.view(-1, 1).expand(-1, emb)
        amax = rel_flat.new_full((int(dim_size), emb), float("-inf"))
        amax.scatter_reduce_(0, index, values, reduce="amax", include_self=True)
        exps = (values - amax.index_select(0, dst_idx)).exp()
        exps_sum = rel_flat.new_zeros((int(dim_size), emb))
        exps_sum.scatter_add_(0, index, exps)
        return exps_sum.log() + amax
    raise ValueError(f"Unsupported fanin mode {mode!r}. Supported: 0=sum, 1=logsumexp.")


def fanout_pack_multi_python(x_parts, src_idx_parts, flat_dst_parts):
    op = "fanout_pack_multi"
    if not x_parts:
        raise ValueError(f"{op} requires at least one source tensor.")
    if not (len(x_parts) == len(src_idx_parts) == len(flat_dst_parts)):
        raise ValueError(f"{op} expects matching sequence lengths.")
    offset = 0
    xs, srcs, dsts = [], [], []
    for x, src, dst in zip(x_parts, src_idx_parts, flat_dst_parts, strict=True):
        _require_rank(op, "source tensor", x, 2)
        _require_rank(op, "src_idx", src, 1)
        _require_rank(op, "flat_dst", dst, 1)
        _require_int64(op, "src_idx", src)
        _require_int64(op, "flat_dst", dst)
        if src.numel() != dst.numel():
            raise ValueError(f"{op} expects src_idx and flat_dst lengths to match per source.")
        xs.append(x)
        srcs.append(src + int(offset))
        dsts.append(dst)
        offset += int(x.size(0))
    return _cat(xs), _cat(srcs), _cat(dsts)


def fanin_pack_multi_python(rel_parts, flat_src_parts, dst_idx_parts):
    op = "fanin_pack_multi"
    if not rel_parts:
        raise ValueError(f"{op} requires at least one relation tensor.")
    if not (len(rel_parts) == len(flat_src_parts) == len(dst_idx_parts)):
        raise ValueError(f"{op} expects matching sequence lengths.")
    offset = 0
    rels, srcs, dsts = [], [], []
    for rel, src, dst in zip(rel_parts, flat_src_parts, dst_idx_parts, strict=True):
        _require_rank(op, "relation tensor", rel, 2)
        _require_rank(op, "flat_src", src, 1)
        _require_rank(op, "dst_idx", dst, 1)
        _require_int64(op, "flat_src", src)
        _require_int64(op, "dst_idx", dst)
        if src.numel() != dst.numel():
            raise ValueError(f"{op} expects flat_src and dst_idx lengths to match per relation tensor.")
        rels.append(rel)
        srcs.append(src + int(offset))
        dsts.append(dst)
        offset += int(rel.size(0))
    return _cat(rels), _cat(srcs), _cat(dsts)


def fanout_pack_from_edges_python(
    x_parts, edge_src_parts, edge_dst_parts, src_part_ids, arity_parts, pos_parts, slot_offset_parts
):
    op = "fanout_pack_from_edges"
    if not x_parts:
        raise ValueError(f"{op} requires at least one source tensor.")
    n = len(edge_src_parts)
    if not (len(edge_dst_parts) == len(src_part_ids) == len(arity_parts) == len(pos_parts) == len(slot_offset_parts) == n):
        raise ValueError(f"{op} expects matching sequence lengths.")
    offsets, offset = [], 0
    for x in x_parts:
        _require_rank(op, "source tensor", x, 2)
        offsets.append(offset)
        offset += int(x.size(0))
    srcs, dsts = [], []
    for es, ed, part, arity, pos, slot in zip(
        edge_src_parts, edge_dst_parts, src_part_ids, arity_parts, pos_parts, slot_offset_parts, strict=True
    ):
        _require_rank(op, "edge_src", es, 1)
        _require_rank(op, "edge_dst", ed, 1)
        _require_int64(op, "edge_src", es)
        _require_int64(op, "edge_dst", ed)
        if es.numel() != ed.numel():
            raise ValueError(f"{op} expects edge src/dst lengths to match.")
        part = int(part)
        if part < 0 or part >= len(x_parts):
            raise ValueError(f"{op} src_part_ids out of range: {part!r}.")
        arity, pos = int(arity), int(pos)
        if arity <= 0:
            raise ValueError(f"{op} expects arity > 0.")
        if pos < 0 or pos >= arity:
            raise ValueError(f"{op} expects pos in [0, arity), got pos={pos} arity={arity}.")
        srcs.append(es + int(offsets[part]))
        dsts.append(int(slot) + ed * arity + pos)
    x_cat = _cat(x_parts)
    if not srcs:
        return x_cat, _empty_index(x_parts[0].device), _empty_index(x_parts[0].device)
    return x_cat, _cat(srcs), _cat(dsts)


def fanin_pack_from_edges_python(rel_parts, edge_src_parts, edge_dst_parts, rel_part_ids, arity_parts, pos_parts, mode):
    op = "fanin_pack_from_edges"
    if not rel_parts:
        raise ValueError(f"{op} requires at least one relation tensor.")
    n = len(edge_src_parts)
    if not (len(edge_dst_parts) == len(rel_part_ids) == len(arity_parts) == len(pos_parts) == n):
        raise ValueError(f"{op} expects matching sequence lengths.")
    mode = int(mode)
    if mode not in (0, 1):
        raise ValueError(f"{op} expects mode in {{0,1}}, got {mode!r}.")
    offsets, offset = [], 0
    for rel in rel_parts:
        _require_rank(op, "relation tensor", rel, 2)
        offsets.append(offset)
        offset += int(rel.size(0))
    srcs, dsts = [], []
    for es, ed, part, arity, pos in zip(edge_src_parts, edge_dst_parts, rel_part_ids, arity_parts, pos_parts, strict=True):
        _require_rank(op, "edge_src", es, 1)
        _require_rank(op, "edge_dst", ed, 1)
        _require_int64(op, "edge_src", es)
        _require_int64(op, "edge_dst", ed)
        if es.numel() != ed.numel():
            raise ValueError(f"{op} expects edge src/dst lengths to match.")
        part = int(part)
        if part < 0 or part >= len(rel_parts):
            raise ValueError(f"{op} rel_part_ids out of range: {part!r}.")
        local = es
        if mode != 1:
            arity, pos = int(arity), int(pos)
            if arity <= 0:
                raise ValueError(f"{op} expects arity > 0.")
            if pos < 0 or pos >= arity:
                raise ValueError(f"{op} expects pos in [0, arity), got pos={pos} arity={arity}.")
            local = es * arity + pos
        srcs.append(local + int(offsets[part]))
        dsts.append(ed)
    rel_cat = _cat(rel_parts)
    if not srcs:
        return rel_cat, _empty_index(rel_parts[0].device), _empty_index(rel_parts[0].device)
    return rel_cat, _cat(srcs), _cat(dsts)
