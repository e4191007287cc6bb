"""Relational message-passing layers: the model call sites of the fan-out /
fan-in ops, without torch_geometric.

Two lanes, as in relmo's ``models/hetero_mp``:

* ``CentralFusedLayer`` - ``CentralFusedLayerMP.forward`` (fused.py:121-406):
  one fan-out of object embeddings into ``max_arity`` slots per atom, one call
  of the shared central module on ``[condition | slot mask | arguments]``, one
  fan-in of the slot messages back to the objects. The input assembly of
  fused.py:311-374 (arguments and context copied into one buffer) is not
  done at all when the central module is a residual MLP (what relmo's
  ``ArityMLPFactory`` builds): its first Linear is applied by column blocks,
  ``W [ctx | args] + b = (W_c ctx + b) + W_a args``, with the context term
  computed once per forward (the context does not change across layers) and
  the fan-out's own output as the argument block, so the fan-out shares the
  fan-in's plan and no input buffer is written or read
  (``CentralFusedLayer.fuse_inputs``, on by default; other central modules
  take the concatenation).
* ``BatchedRelationLayer`` - ``BatchedFanOutMP`` + ``BatchedFanInMP``
  (batched.py:41-1199) on the flattened slot handoff: one fan-out into the
  slots of all predicates (``arity`` slots per atom), one per-predicate update
  module on each predicate's ``[n_atoms, arity*D]`` block, one fan-in.

The routing (which object feeds which slot) is built once per forward from the
batch (``build_fused_routing`` / ``build_batched_routing``) and reused by every
layer; fan-out and fan-in get the same index tensors, so the op library builds
one plan per forward for both directions and reuses it in the backward.

``use_kernels`` selects the relm_mp ops (default on CUDA) or the reference's
torch formulas (``index_select`` / ``index_copy_`` / ``index_add_`` and the
smoothed logsumexp of ``models/aggr.py:96-123``) - the latter is what relmo runs
when its kernel flags are off, and what the model parity tests compare with.
Unlike relmo (``_ops_env.py``: fan-out off, logsumexp off, batched lanes
experimental), CUDA tensors always take the kernels here.

Smoothed logsumexp (relmo's ``LogSumExpAggregation``, beta = 12, detached max,
1e-16 added to every sum): ``(1/beta) log(1e-16 + sum exp(beta (x - m))) + m``
equals ``fanin_reduce(beta x, logsumexp) / beta`` up to the 1e-16 term, which is
below float resolution for any row with a message (the max term alone
contributes 1). Rows without messages get ``log(1e-16) / beta`` as in relmo.
The gradient is softmax(beta x) over the row in both.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from .nn import MLP, ResidualModule, SimpleMLP
from .ops import mp
from .ops.mp_constants import MODE_SUM
from .workloads import RelationalBatch

LSE_BETA = 12.0
LSE_EPS = 1e-16


def _kernels(ref: torch.Tensor, use_kernels: bool | None) -> bool:
    if use_kernels is None:
        return ref.is_cuda and ref.dtype.is_floating_point
    return bool(use_kernels)


# ---- fan-out / fan-in through the ops or the reference formulas ------------------------


def fanout(x: torch.Tensor, src: torch.Tensor, flat_dst: torch.Tensor, out_rows: int, use_kernels: bool) -> torch.Tensor:
    """out[flat_dst[e]] = x[src[e]], zeros elsewhere."""

    if use_kernels:
        return mp.fanout_scatter(x, src, flat_dst, int(out_rows))
    out = x.new_zeros((int(out_rows), x.size(1)))
    return out.index_copy(0, flat_dst, x.index_select(0, src))


def smoothed_logsumexp_reference(x: torch.Tensor, index: torch.Tensor, dim_size: int,
                                 beta: float = LSE_BETA) -> torch.Tensor:
    """relmo's LogSumExpAggregation.forward (models/aggr.py:103-123); the row max
    is taken with ``scatter_reduce`` instead of the beta ``index_reduce_`` (same
    values: a max is exact)."""

    m = torch.zeros((dim_size, x.size(-1)), device=x.device, dtype=x.dtype)
    m = m.scatter_reduce(0, index.view(-1, 1).expand_as(x), x, reduce="amax", include_self=False).detach()
    s = torch.full_like(m, LSE_EPS)
    s = s.index_add(0, index, (beta * (x - m.index_select(0, index))).exp())
    return (1.0 / beta) * s.log() + m


def fanin(msgs: torch.Tensor, flat_src: torch.Tensor, dst: torch.Tensor, dim_size: int, aggr: str,
          use_kernels: bool) -> torch.Tensor:
    """Aggregate message rows ``msgs[flat_src[e]]`` into ``dst[e]``: "sum" or the
    smoothed "logsumexp" (one kernel pass each way on the kernel path, rows
    without messages included)."""

    if aggr == "sum":
        if use_kernels:
            return mp.fanin_reduce(msgs, flat_src, dst, int(dim_size), MODE_SUM)
        out = msgs.new_zeros((int(dim_size), msgs.size(1)))
        return out.index_add(0, dst, msgs.index_select(0, flat_src))
    if aggr == "logsumexp":
        if not use_kernels:
            return smoothed_logsumexp_reference(msgs.index_select(0, flat_src), dst, int(dim_size))
        return mp.fanin_reduce_smoothed_logsumexp(msgs, flat_src, dst, int(dim_size), LSE_BETA, LSE_EPS)
    raise ValueError(f"aggregation must be 'sum' or 'logsumexp', got {aggr!r}")


# ---- routing ------------------------------------------------------------------------------


@dataclass
class FusedRouting:
    """Routing of the centralized fused layer (fused.py:133-232)."""

    order: list                 # predicates with atoms and arity > 0, sorted
    offsets: dict               # first atom row of each predicate
    total_atoms: int            # R
    obj: torch.Tensor           # object of each (atom, pos) edge
    slot: torch.Tensor          # flat slot (atom_row * max_arity + pos) of each edge
    cond_index: torch.Tensor    # condition-embedding row of each atom row
    slot_mask: torch.Tensor     # [R, max_arity] 1 for pos < arity
    pred_meta: list = field(default_factory=list)  # (pred, start, n, arity)


def build_fused_routing(batch: RelationalBatch, relation_arities: dict, condition_index: dict, max_arity: int,
                        dtype: torch.dtype) -> FusedRouting:
    order = sorted(p for p, a in batch.relations.items()
                   if p in relation_arities and int(relation_arities[p]) > 0 and a.size(0) > 0)
    offsets, total = {}, 0
    for p in order:
        offsets[p] = total
        total += int(batch.relations[p].size(0))
    device = batch.object_state.device
    empty_idx = torch.empty(0, dtype=torch.int64, device=device)
    meta = [(p, offsets[p], int(batch.relations[p].size(0)), int(batch.relations[p].size(1))) for p in order]
    if not order:
        return FusedRouting(order, offsets, 0, empty_idx, empty_idx, empty_idx,
                            torch.zeros((0, max_arity), device=device, dtype=dtype), meta)
    # (atom, pos) edges of every predicate through the fan-out pack op (one
    # device pass for all parts): object = args[atom, pos], slot =
    # (offset_p + atom) * max_arity + pos.
    max_n = max(n for _, _, n, _ in meta)
    atoms = torch.arange(max_n, device=device, dtype=torch.int64)
    src_parts, dst_parts, pos_parts, slot_parts = [], [], [], []
    for p, off, n, k in meta:
        args = batch.relations[p]
        for pos in range(k):
            src_parts.append(args[:, pos])
            dst_parts.append(atoms[:n])
            pos_parts.append(pos)
            slot_parts.append(off * max_arity)
    nparts = len(src_parts)
    _, obj, slot = _pack_from_edges([empty_idx.view(0, 1).float()], src_parts, dst_parts, [0] * nparts,
                                    [max_arity] * nparts, pos_parts, slot_parts)
    # per atom row: its predicate's condition row and slot mask
    counts = torch.tensor([n for _, _, n, _ in meta], device=device)
    pred_of_row = torch.repeat_interleave(torch.arange(len(meta), device=device), counts, output_size=total)
    cond_table = torch.tensor([int(condition_index[p]) for p in order], device=device, dtype=torch.int64)
    mask_table = (torch.arange(max_arity).view(1, -1) < torch.tensor([k for *_, k in meta]).view(-1, 1))
    mask_table = mask_table.to(device=device, dtype=dtype)
    return FusedRouting(order, offsets, total, obj, slot, cond_table[pred_of_row], mask_table[pred_of_row], meta)


def _pack_from_edges(x_parts, edge_src, edge_dst, part_ids, arity, pos, slot_offsets):
    """The fan-out pack op (relm_mp_pack_index on CUDA) or, without the library,
    the reference's formula."""

    if mp.available():
        return torch.ops.relm_mp.fanout_pack_from_edges(x_parts, edge_src, edge_dst, part_ids, arity, pos, slot_offsets)
    from .ops import mp_pack

    return mp_pack.fanout_pack_from_edges_python(x_parts, edge_src, edge_dst, part_ids, arity, pos, slot_offsets)


@dataclass
class BatchedRouting:
    """Routing of the decentralized batched lane: slots of predicate p are
    ``[start_p, start_p + n_p * k_p)``, atom-major, so each predicate's block is a
    contiguous ``[n_p, k_p * D]`` view and the slot index is ``arange``."""

    pred_meta: list             # (pred, slot_start, n_atoms, arity)
    total_slots: int
    obj: torch.Tensor           # object of each slot
    slot: torch.Tensor          # arange(total_slots)


def build_batched_routing(batch: RelationalBatch, relation_arities: dict) -> BatchedRouting:
    device = batch.object_state.device
    meta, objs, start = [], [], 0
    for p in sorted(relation_arities):
        if p not in batch.relations or int(relation_arities[p]) == 0:
            continue
        args = batch.relations[p]
        n, k = int(args.size(0)), int(args.size(1))
        if n == 0:
            continue
        meta.append((p, start, n, k))
        objs.append(args.reshape(-1))
        start += n * k
    obj = torch.cat(objs) if objs else torch.empty(0, dtype=torch.int64, device=device)
    slot = torch.arange(start, dtype=torch.int64, device=device)
    return BatchedRouting(meta, start, obj, slot)


# ---- layers ---------------------------------------------------------------------------------


class CentralFusedLayer(nn.Module):
    """Fused centralized relational layer: fan-out -> central module -> fan-in.
    Returns (atom messages per predicate, object messages)."""

    def __init__(self, *, central_module: nn.Module, condition_embedding: nn.Embedding, max_arity: int,
                 embedding_size: int, condition_position: str = "pre", include_slot_mask: bool = True,
                 aggr: str = "logsumexp", use_kernels: bool | None = None, fuse_inputs: bool = True):
        super().__init__()
        if condition_position not in ("pre", "post"):
            raise ValueError(f"condition_position must be 'pre' or 'post', got {condition_position!r}.")
        self.fuse_inputs = bool(fuse_inputs)
        self.central_module = central_module
        self.condition_embedding = condition_embedding
        self.max_arity = int(max_arity)
        self.embedding_size = int(embedding_size)
        self.condition_position = condition_position
        self.include_slot_mask = bool(include_slot_mask)
        self.aggr = aggr
        self.use_kernels = use_kernels

    def context(self, routing: FusedRouting):
        """The [R, cond_dim (+ max_arity)] condition (and slot-mask) columns of
        the central module's input, built once per forward (the reference
        caches it for the whole forward); with the split first layer also its
        term ``W_c ctx + b``, the same in every layer."""

        cond = self.condition_embedding.weight.index_select(0, routing.cond_index)
        if self.include_slot_mask:
            mask = routing.slot_mask.to(cond.dtype)
            cond = torch.cat([cond, mask], dim=1) if self.condition_position == "pre" else torch.cat([mask, cond], dim=1)
        split = self._split_layers() if self.fuse_inputs else None
        if split is None:
            return cond
        lin0, _ = split
        A, d, C = self.max_arity, self.embedding_size, int(cond.size(1))
        w_ctx = lin0.weight[:, :C] if self.condition_position == "pre" else lin0.weight[:, A * d :]
        return SplitContext(cond, F.linear(cond.to(w_ctx.dtype), w_ctx, lin0.bias))

    def _split_layers(self):
        """(first Linear, later layers) when the central module is
        ``ResidualModule(MLP | SimpleMLP)`` over ``[context | arguments]``
        ("pre"; ``[arguments | context]`` "post") whose residual is the argument
        block; else None."""

        res = self.central_module
        A, d = self.max_arity, self.embedding_size
        if not isinstance(res, ResidualModule) or res.truncated_dim != A * d:
            return None
        if bool(res.truncate_right) != (self.condition_position == "post"):
            return None
        inner = res.module
        layers = list(inner.net) if isinstance(inner, MLP) else list(inner.mlp) if isinstance(inner, SimpleMLP) else None
        if not layers or not isinstance(layers[0], nn.Linear) or layers[0].in_features <= A * d:
            return None
        return layers[0], layers[1:]

    def forward(self, x: torch.Tensor, routing: FusedRouting, context):
        kern = _kernels(x, self.use_kernels)
        n_obj, d = x.size(0), self.embedding_size
        R = routing.total_atoms
        if R == 0:
            return {}, x.new_zeros((n_obj, d))
        args_flat = fanout(x, routing.obj, routing.slot, R * self.max_arity, kern)
        args_feat = args_flat.reshape(R, self.max_arity * d)
        if isinstance(context, SplitContext):
            all_outputs = self._split_forward(args_feat, context)
        else:
            ctx = context.to(args_feat.dtype)
            all_inputs = torch.cat([ctx, args_feat], dim=1) if self.condition_position == "pre" else torch.cat(
                [args_feat, ctx], dim=1)
            all_outputs = self.central_module(all_inputs)
        atom_msgs = {p: all_outputs[s : s + n, : k * d] for p, s, n, k in routing.pred_meta}
        out_flat = all_outputs.reshape(R * self.max_arity, d)
        msgs = fanin(out_flat, routing.slot, routing.obj, n_obj, self.aggr, kern)
        return atom_msgs, msgs

    def _split_forward(self, args_feat: torch.Tensor, context: "SplitContext") -> torch.Tensor:
        """The residual MLP on [context | arguments] without the concatenation:
        args + rest(W_a args + (W_c ctx + b))."""

        lin0, rest = self._split_layers()
        A, d = self.max_arity, self.embedding_size
        C = lin0.in_features - A * d
        w_args = lin0.weight[:, C:] if self.condition_position == "pre" else lin0.weight[:, : A * d]
        term = context.term
        if torch.is_autocast_enabled(args_feat.device.type):
            h = F.linear(args_feat, w_args) + term
        else:
            h = torch.addmm(term.to(args_feat.dtype), args_feat, w_args.t())
        for layer in rest:
            h = layer(h)
        return args_feat + h


@dataclass
class SplitContext:
    """Context of a forward whose central module takes its first layer by
    column blocks: the context columns and their layer term ``W_c ctx + b``."""

    columns: torch.Tensor
    term: torch.Tensor


class BatchedRelationLayer(nn.Module):
    """Decentralized relational layer on the flattened slot handoff: fan-out to
    all slots, one update module per predicate, fan-in of all slots."""

    def __init__(self, update_modules: dict, *, embedding_size: int, aggr: str = "sum",
                 use_kernels: bool | None = None):
        super().__init__()
        self.update_modules = nn.ModuleDict(update_modules)
        self.embedding_size = int(embedding_size)
        self.aggr = aggr
        self.use_kernels = use_kernels

    def forward(self, x: torch.Tensor, routing: BatchedRouting):
        kern = _kernels(x, self.use_kernels)
        d = self.embedding_size
        if routing.total_slots == 0:
            return {}, x.new_zeros((x.size(0), d))
        x_in = x
        if torch.is_autocast_enabled(x.device.type) and x.is_cuda:
            x_in = x.to(torch.get_autocast_dtype(x.device.type))  # low-precision messages
        slots = fanout(x_in, routing.obj, routing.slot, routing.total_slots, kern)
        # split, not slices: the backward of a split is one cat of the block
        # gradients, a slice's backward zero-fills the whole slot tensor per block
        blocks = slots.split([n * k for _, _, n, k in routing.pred_meta])
        outs, atom_msgs = [], {}
        for (p, start, n, k), block in zip(routing.pred_meta, blocks):
            y = self.update_modules[p](block.reshape(n, k * d))
            atom_msgs[p] = y
            outs.append(y.reshape(n * k, d))
        dtype = torch.promote_types(outs[0].dtype, outs[-1].dtype)
        msgs = torch.cat([o.to(dtype) for o in outs], dim=0) if len(outs) > 1 else outs[0]
        out = fanin(msgs, routing.slot, routing.obj, x.size(0), self.aggr, kern)
        return atom_msgs, out
