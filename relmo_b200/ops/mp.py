"""Public facade of the relational message-passing ops (mirrors ``relmo.ops.mp``).

Same functions, arguments and return values as relmo's ``src/relmo/ops/mp.py``
for the fan-out / fan-in path (``fanout_scatter`` 43-52, ``fanin_reduce`` 55-70,
the four pack helpers, ``available``, ``assert_runtime_compat``, ``__all__``
528-544). Each call runs where ``mp_dispatch.route`` sends it:

- CUDA tensors: the B200 kernels through ``torch.ops.relm_mp`` with the
  reference's autograd wrappers. There is no GPU fallback: if the library is
  missing or disabled the call raises.
- CPU tensors: the library's CPU kernels (the reference CPU library's loops and
  ATen formulas) when it loads, as relmo sends CPU tensors to its library;
  otherwise the reference's Python formulas (``mp_pack``), or an error under
  ``RELM_MP_FALLBACK=error``.
- fanin modes other than sum / logsumexp (mean) use the Python formulas on every
  device, as relmo's facade does (mp.py:64-65).

The LGAN indexed reductions (``_lgan_pool_reduce``, ``_lgan_relation_graph_step``,
mp.py:468-525, modes ``"sum"`` / ``"mean"``) follow the same routing through the
reference's autograd wrappers. The fused block / program ops of relmo
(``block_*``, ``program_*``, ``_lgan_build_pointwise_step``) are a different
model family and are not part of this package.
"""

from __future__ import annotations

from .mp_autograd import (
    _FaninReduceLogSumExpFunction,
    _FaninReduceSmoothedLogSumExpFunction,
    _FaninReduceSumFunction,
    _FanoutScatterFunction,
)
from .mp_constants import MODE_LOGSUMEXP, MODE_MEAN, MODE_SUM
from .mp_dispatch import CUSTOM, call, route
from .mp_lgan import (
    _LGANPoolReduceFunction,
    _LGANRelationGraphStepFunction,
    lgan_pool_reduce_python,
    lgan_relation_graph_step_python,
    resolve_lgan_mode,
)
from .mp_pack import (
    fanin_pack_from_edges_python,
    fanin_pack_multi_python,
    fanin_reduce_python,
    fanout_pack_from_edges_python,
    fanout_pack_multi_python,
    fanout_scatter_python,
)
from .mp_runtime import TORCH_IMPORT_ERROR, assert_runtime_compat, available, ops_namespace, require_torch, torch


def _first(parts):
    """The tensor whose device decides where a pack op runs (None for no parts)."""

    return parts[0] if len(parts) else None


def fanout_scatter(x_cat, src_global_idx, flat_dst, out_rows: int):
    """``out = zeros(out_rows, D); out[flat_dst[e]] = x_cat[src_global_idx[e]]``."""

    require_torch("fanout_scatter")
    if route("fanout_scatter", x_cat) == CUSTOM:
        return _FanoutScatterFunction.apply(x_cat, src_global_idx, flat_dst, int(out_rows))
    return fanout_scatter_python(x_cat, src_global_idx, flat_dst, int(out_rows))


def fanin_reduce(rel_flat, flat_src, dst_idx, dim_size: int, mode: int):
    """Reduce ``rel_flat[flat_src[e]]`` into row ``dst_idx[e]``: mode 0 sum,
    mode 1 logsumexp (-inf for rows without messages)."""

    require_torch("fanin_reduce")
    mode_int = int(mode)
    if mode_int not in (MODE_SUM, MODE_LOGSUMEXP):
        return fanin_reduce_python(rel_flat, flat_src, dst_idx, int(dim_size), mode_int)
    if route("fanin_reduce", rel_flat) == CUSTOM:
        if mode_int == MODE_SUM:
            return _FaninReduceSumFunction.apply(rel_flat, flat_src, dst_idx, int(dim_size))
        return _FaninReduceLogSumExpFunction.apply(rel_flat, flat_src, dst_idx, int(dim_size))
    return fanin_reduce_python(rel_flat, flat_src, dst_idx, int(dim_size), mode_int)


def smoothed_logsumexp_python(rel_flat, flat_src, dst_idx, dim_size: int, beta: float, eps: float):
    """relmo's LogSumExpAggregation.forward (models/aggr.py:103-123) on the
    gathered messages: the formula the CPU path runs without the library."""

    x = rel_flat.index_select(0, flat_src)
    m = torch.zeros((int(dim_size), x.size(-1)), device=x.device, dtype=x.dtype)
    m = m.index_reduce(0, dst_idx, x, "amax", include_self=False).detach()
    s = torch.full_like(m, eps).index_add(0, dst_idx, (beta * (x - m.index_select(0, dst_idx))).exp())
    return (1.0 / beta) * s.log() + m


def fanin_reduce_smoothed_logsumexp(rel_flat, flat_src, dst_idx, dim_size: int, beta: float = 12.0,
                                    eps: float = 1e-16):
    """The smoothed logsumexp relmo's models aggregate with (LogSumExpAggregation,
    models/aggr.py:96-123; beta = its maximum_smoothness): per column
    ``m + (1/beta) log(eps + sum exp(beta (x - m)))`` over the row's messages
    ``rel_flat[flat_src[e]]``, m the row max (no gradient through it); rows
    without messages get ``(1/beta) log(eps)``. One planned kernel pass forward
    and one backward (gradient ``exp(beta (x - out))``), instead of relmo's
    four ATen passes. Not part of relmo's op facade."""

    require_torch("fanin_reduce_smoothed_logsumexp")
    if route("fanin_reduce_smoothed_logsumexp", rel_flat) == CUSTOM:
        if rel_flat.dtype in (torch.bfloat16, torch.float16):
            # The backward weight exp(beta (x - out)) would carry the rounding
            # of a 2-byte `out` times beta (12: ~25% at bf16's 2^-9); run the op
            # in fp32 so the gradient sees the fp32 output, and round the
            # result for the caller.
            out = _FaninReduceSmoothedLogSumExpFunction.apply(
                rel_flat.float(), flat_src, dst_idx, int(dim_size), float(beta), float(eps)
            )
            return out.to(rel_flat.dtype)
        return _FaninReduceSmoothedLogSumExpFunction.apply(
            rel_flat, flat_src, dst_idx, int(dim_size), float(beta), float(eps)
        )
    return smoothed_logsumexp_python(rel_flat, flat_src, dst_idx, int(dim_size), float(beta), float(eps))


def fanout_pack_multi(x_parts, src_idx_parts, flat_dst_parts):
    require_torch("fanout_pack_multi")
    return call(
        "fanout_pack_multi", x_parts, src_idx_parts, flat_dst_parts, tensor=_first(x_parts),
        python=fanout_pack_multi_python,
    )


def fanin_pack_multi(rel_parts, flat_src_parts, dst_idx_parts):
    require_torch("fanin_pack_multi")
    return call(
        "fanin_pack_multi", rel_parts, flat_src_parts, dst_idx_parts, tensor=_first(rel_parts),
        python=fanin_pack_multi_python,
    )


def fanout_pack_from_edges(x_parts, edge_src_parts, edge_dst_parts, src_part_ids, arity_parts, pos_parts, slot_offset_parts):
    require_torch("fanout_pack_from_edges")
    return call(
        "fanout_pack_from_edges",
        x_parts,
        edge_src_parts,
        edge_dst_parts,
        [int(v) for v in src_part_ids],
        [int(v) for v in arity_parts],
        [int(v) for v in pos_parts],
        [int(v) for v in slot_offset_parts],
        tensor=_first(x_parts),
        python=fanout_pack_from_edges_python,
    )


def fanin_pack_from_edges(rel_parts, edge_src_parts, edge_dst_parts, rel_part_ids, arity_parts, pos_parts, mode: int):
    require_torch("fanin_pack_from_edges")
    return call(
        "fanin_pack_from_edges",
        rel_parts,
        edge_src_parts,
        edge_dst_parts,
        [int(v) for v in rel_part_ids],
        [int(v) for v in arity_parts],
        [int(v) for v in pos_parts],
        int(mode),
        tensor=_first(rel_parts),
        python=fanin_pack_from_edges_python,
    )


def _lgan_pool_reduce(slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel,
                      tn_ent, nn_rel, nn_ent, *, entity_dim_size: int, mode: str):
    """Pool slot messages to relation instances (mean over each instance's
    arity), then run the RR / TN / NN indexed reductions; returns
    ``(relation_pair_x, tn_msgs, nn_msgs)``."""

    require_torch("_lgan_pool_reduce")
    mode_int = resolve_lgan_mode("_lgan_pool_reduce", mode)
    args = (slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel, tn_ent,
            nn_rel, nn_ent, int(entity_dim_size), int(mode_int))
    if route("lgan_pool_reduce", slot_messages) == CUSTOM:
        return _LGANPoolReduceFunction.apply(*args)
    return lgan_pool_reduce_python(*args)


def _lgan_relation_graph_step(relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, *,
                              entity_dim_size: int, mode: str):
    """RR / TN / NN propagation on pooled relation-instance embeddings; returns
    ``(relation_pair_x + rr_msgs, tn_msgs, nn_msgs)``."""

    require_torch("_lgan_relation_graph_step")
    mode_int = resolve_lgan_mode("_lgan_relation_graph_step", mode)
    args = (relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, int(entity_dim_size), int(mode_int))
    if route("lgan_relation_graph_step", relation_pair_x) == CUSTOM:
        return _LGANRelationGraphStepFunction.apply(*args)
    return lgan_relation_graph_step_python(*args)


def clear_plan_cache() -> None:
    """Drop every cached index plan (they are rebuilt on the next call)."""

    ops_namespace()  # loads the library (raises when it is unusable)
    torch.ops.relm_mp_b200.clear_plan_cache()


def plan_cache_stats() -> dict[str, int]:
    """Entries, hits, builds, bytes and capacity of the index-plan cache."""

    ops_namespace()  # loads the library (raises when it is unusable)
    entries, hits, builds, nbytes, capacity = torch.ops.relm_mp_b200.plan_cache_stats()
    return {"entries": entries, "hits": hits, "builds": builds, "bytes": nbytes, "capacity": capacity}


def set_plan_cache_capacity(capacity: int) -> None:
    ops_namespace()  # loads the library (raises when it is unusable)
    torch.ops.relm_mp_b200.set_plan_cache_capacity(int(capacity))


__all__ = [
    "fanout_scatter",
    "fanin_reduce",
    "fanin_reduce_smoothed_logsumexp",
    "fanout_pack_multi",
    "fanin_pack_multi",
    "fanout_pack_from_edges",
    "fanin_pack_from_edges",
    "available",
    "assert_runtime_compat",
    "clear_plan_cache",
    "plan_cache_stats",
    "set_plan_cache_capacity",
    "MODE_SUM",
    "MODE_LOGSUMEXP",
    "MODE_MEAN",
]
