"""LGAN indexed reductions: CPU formulas and autograd wrappers.

Mirrors relmo's LGAN op path for the ``sum`` / ``mean`` modes:

- ``indexed_sum_or_mean`` (``src/relmo/ops/mp_common.py:88-118``) and the two
  Python formulas ``lgan_pool_reduce_python`` / ``lgan_relation_graph_step_python``
  (``mp_fallbacks.py:28-126``), used for CPU tensors;
- ``_LGANPoolReduceFunction`` / ``_LGANRelationGraphStepFunction``
  (``mp_autograd.py:194-535``): same saved tensors, same backward ops
  (``lgan_pool_reduce_backward`` / ``lgan_relation_graph_step_backward``, with
  zero tensors standing in for output gradients that are ``None``), gradient
  for the first input only.

CUDA tensors always run the B200 ops (``torch.ops.relm_mp.lgan_*``); there is
no GPU fallback to the Python formulas.
"""

from __future__ import annotations

from .mp_constants import MODE_MEAN, MODE_SUM
from .mp_runtime import ops_namespace, torch


def resolve_lgan_mode(op_name: str, mode: str) -> int:
    """``"sum"`` -> 0, ``"mean"`` -> 2 (mp.py:394-400)."""

    mode_key = str(mode).strip().lower()
    if mode_key == "sum":
        return MODE_SUM
    if mode_key == "mean":
        return MODE_MEAN
    raise ValueError(f"{op_name} supports only mode='sum' or mode='mean'.")


def _require_rank(op_name: str, name: str, tensor, rank: int) -> None:
    if tensor.dim() != rank:
        raise ValueError(f"{op_name} expects {name} to be rank-{rank}, got shape {tuple(tensor.shape)}.")


def indexed_sum_or_mean(source_embeddings, source_index, target_index, dim_size: int, mode: int, *, op_name: str):
    """``out[target[e]] += source[source_index[e]]``, divided by
    ``max(count of target, 1)`` in mean mode."""

    if mode not in (MODE_SUM, MODE_MEAN):
        raise ValueError(f"{op_name} supports only sum and mean modes.")
    out = source_embeddings.new_zeros((int(dim_size), int(source_embeddings.size(-1))))
    if int(source_index.numel()) == 0 or int(dim_size) == 0:
        return out
    out.index_add_(0, target_index, source_embeddings.index_select(0, source_index))
    if mode == MODE_MEAN:
        counts = out.new_zeros((int(dim_size), 1))
        counts.index_add_(
            0, target_index, torch.ones((int(target_index.numel()), 1), device=out.device, dtype=out.dtype)
        )
        out = out / counts.clamp_min_(1.0)
    return out


def lgan_relation_graph_step_python(relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                                    entity_dim_size: int, mode: int):
    op_name = "lgan_relation_graph_step"
    _require_rank(op_name, "relation_pair_x", relation_pair_x, 2)
    rr_msgs = indexed_sum_or_mean(relation_pair_x, rr_src, rr_dst, int(relation_pair_x.size(0)), mode,
                                  op_name=op_name)
    relation_pair_x = relation_pair_x + rr_msgs
    tn_msgs = indexed_sum_or_mean(relation_pair_x, tn_rel, tn_ent, int(entity_dim_size), mode, op_name=op_name)
    nn_msgs = indexed_sum_or_mean(relation_pair_x, nn_rel, nn_ent, int(entity_dim_size), mode, op_name=op_name)
    return relation_pair_x, tn_msgs, nn_msgs


def lgan_pool_reduce_python(slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst,
                            tn_rel, tn_ent, nn_rel, nn_ent, entity_dim_size: int, mode: int):
    op_name = "lgan_pool_reduce"
    _require_rank(op_name, "slot_messages", slot_messages, 2)
    relation_count = int(relation_instance_arities.numel())
    relation_pair_x = slot_messages.new_zeros((relation_count, int(slot_messages.size(-1))))
    if int(slot_messages.numel()) > 0:
        relation_pair_x.index_add_(0, slot_to_relation_instance, slot_messages)
        counts = relation_instance_arities.to(device=slot_messages.device, dtype=slot_messages.dtype)
        relation_pair_x = relation_pair_x / counts.view(-1, 1).clamp_min_(1.0)
    return lgan_relation_graph_step_python(relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent,
                                           entity_dim_size, mode)


def _zeros_if_none(grad, rows: int, like):
    if grad is not None:
        return grad.contiguous()
    return torch.zeros((int(rows), int(like.size(-1))), device=like.device, dtype=like.dtype)


if torch is not None:

    class _LGANPoolReduceFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst,
                    tn_rel, tn_ent, nn_rel, nn_ent, entity_dim_size: int, mode: int):
            ctx.entity_dim_size = int(entity_dim_size)
            ctx.mode = int(mode)
            ctx.save_for_backward(slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src,
                                  rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
            return ops_namespace().lgan_pool_reduce(
                slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel,
                tn_ent, nn_rel, nn_ent, int(entity_dim_size), int(mode)
            )

        @staticmethod
        def backward(ctx, grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs):
            (slot_messages, slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel, tn_ent,
             nn_rel, nn_ent) = ctx.saved_tensors
            if (grad_relation_pair_x is None and grad_tn_msgs is None and grad_nn_msgs is None) or not (
                ctx.needs_input_grad[0]
            ):
                return (None,) * 11
            relation_count = int(relation_instance_arities.numel())
            grad_slots = ops_namespace().lgan_pool_reduce_backward(
                _zeros_if_none(grad_relation_pair_x, relation_count, slot_messages),
                _zeros_if_none(grad_tn_msgs, ctx.entity_dim_size, slot_messages),
                _zeros_if_none(grad_nn_msgs, ctx.entity_dim_size, slot_messages),
                slot_to_relation_instance, relation_instance_arities, rr_src, rr_dst, tn_rel, tn_ent, nn_rel,
                nn_ent, relation_count, int(ctx.mode)
            )
            return (grad_slots,) + (None,) * 10

    class _LGANRelationGraphStepFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, entity_dim_size: int,
                    mode: int):
            ctx.entity_dim_size = int(entity_dim_size)
            ctx.mode = int(mode)
            ctx.save_for_backward(relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent)
            return ops_namespace().lgan_relation_graph_step(
                relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, int(entity_dim_size), int(mode)
            )

        @staticmethod
        def backward(ctx, grad_relation_pair_x, grad_tn_msgs, grad_nn_msgs):
            relation_pair_x, rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent = ctx.saved_tensors
            if (grad_relation_pair_x is None and grad_tn_msgs is None and grad_nn_msgs is None) or not (
                ctx.needs_input_grad[0]
            ):
                return (None,) * 9
            relation_count = int(relation_pair_x.size(0))
            grad_x = ops_namespace().lgan_relation_graph_step_backward(
                _zeros_if_none(grad_relation_pair_x, relation_count, relation_pair_x),
                _zeros_if_none(grad_tn_msgs, ctx.entity_dim_size, relation_pair_x),
                _zeros_if_none(grad_nn_msgs, ctx.entity_dim_size, relation_pair_x),
                rr_src, rr_dst, tn_rel, tn_ent, nn_rel, nn_ent, relation_count, int(ctx.mode)
            )
            return (grad_x,) + (None,) * 8
