"""Autograd wrappers of the hot ops (relmo ``src/relmo/ops/mp_autograd.py:110-191``).

Same saved tensors and backward ops as the reference:

- ``_FanoutScatterFunction``: saves (src_global_idx, flat_dst), ``x_rows``;
  backward = ``fanout_scatter_backward``.
- ``_FaninReduceSumFunction``: saves (flat_src, dst_idx), ``rel_rows``;
  backward = ``fanin_reduce_sum_backward``.
- ``_FaninReduceLogSumExpFunction``: saves (rel_flat, flat_src, dst_idx, out);
  backward = ``fanin_reduce_logsumexp_backward``.

Backward returns ``(grad, None, None, None)``; no double backward, as in the
reference. The index tensors saved here are the ones the forward saw, so the
library's plan cache serves the backward without a second sort.
"""

from __future__ import annotations

from .mp_constants import MODE_LOGSUMEXP, MODE_SUM
from .mp_runtime import ops_namespace, torch

if torch is not None:

    class _FanoutScatterFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x_cat, src_global_idx, flat_dst, out_rows: int):
            ctx.save_for_backward(src_global_idx, flat_dst)
            ctx.x_rows = int(x_cat.size(0))
            return ops_namespace().fanout_scatter(x_cat, src_global_idx, flat_dst, int(out_rows))

        @staticmethod
        def backward(ctx, grad_out):
            src_global_idx, flat_dst = ctx.saved_tensors
            grad_x = ops_namespace().fanout_scatter_backward(
                grad_out.contiguous(), src_global_idx, flat_dst, int(ctx.x_rows)
            )
            return grad_x, None, None, None

    class _FaninReduceSumFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, rel_flat, flat_src, dst_idx, dim_size: int):
            ctx.save_for_backward(flat_src, dst_idx)
            ctx.rel_rows = int(rel_flat.size(0))
            return ops_namespace().fanin_reduce(rel_flat, flat_src, dst_idx, int(dim_size), MODE_SUM)

        @staticmethod
        def backward(ctx, grad_out):
            flat_src, dst_idx = ctx.saved_tensors
            grad_rel = ops_namespace().fanin_reduce_sum_backward(
                grad_out.contiguous(), flat_src, dst_idx, int(ctx.rel_rows)
            )
            return grad_rel, None, None, None

    class _FaninReduceLogSumExpFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, rel_flat, flat_src, dst_idx, dim_size: int):
            ctx.rel_rows = int(rel_flat.size(0))
            out = ops_namespace().fanin_reduce(rel_flat, flat_src, dst_idx, int(dim_size), MODE_LOGSUMEXP)
            ctx.save_for_backward(rel_flat, flat_src, dst_idx, out)
            return out

        @staticmethod
        def backward(ctx, grad_out):
            rel_flat, flat_src, dst_idx, out = ctx.saved_tensors
            grad_rel = ops_namespace().fanin_reduce_logsumexp_backward(
                grad_out.contiguous(), rel_flat, flat_src, dst_idx, out, int(ctx.rel_rows)
            )
            return grad_rel, None, None, None

    class _FaninReduceSmoothedLogSumExpFunction(torch.autograd.Function):
        """The smoothed logsumexp of relmo's models (LogSumExpAggregation,
        relmo/models/aggr.py:96-123) as one op pair; not a reference op. Saves
        (rel_flat, flat_src, dst_idx, out) like the plain logsumexp."""

        @staticmethod
        def forward(ctx, rel_flat, flat_src, dst_idx, dim_size: int, beta: float, eps: float):
            ctx.rel_rows = int(rel_flat.size(0))
            ctx.beta = float(beta)
            out = torch.ops.relm_mp_b200.fanin_reduce_smoothed_logsumexp(
                rel_flat, flat_src, dst_idx, int(dim_size), float(beta), float(eps)
            )
            ctx.save_for_backward(rel_flat, flat_src, dst_idx, out)
            return out

        @staticmethod
        def backward(ctx, grad_out):
            rel_flat, flat_src, dst_idx, out = ctx.saved_tensors
            grad_rel = torch.ops.relm_mp_b200.fanin_reduce_smoothed_logsumexp_backward(
                grad_out.contiguous(), rel_flat, flat_src, dst_idx, out, int(ctx.rel_rows), ctx.beta
            )
            return grad_rel, None, None, None, None, None
