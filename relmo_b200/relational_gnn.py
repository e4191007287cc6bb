"""RelationalGNN and CentralizedRelationalGNN over the B200 fan-out / fan-in ops.

Restatements of relmo's model drivers (``models/relational_gnn.py``) for the
two lanes that call the ops, without torch_geometric:

* ``RelationalGNN`` with ``rel_layer_mode="batched_cached"`` (relational_gnn.py:
  124-535): one update module per predicate (``ArityMLPFactory`` default:
  residual MLP over the predicate's argument embeddings), a
  ``BatchedRelationLayer`` per layer, then ``x = x + updater([x, m])``.
* ``CentralizedRelationalGNN`` with ``central_layer_mode="fused"``
  (relational_gnn.py:552-846): one shared central module conditioned on a
  per-predicate embedding of ``int(sqrt(D))`` columns, a ``CentralFusedLayer``
  per layer, then the same update. The default central module is
  ``_build_default_central_module`` (757-787): residual ``FiLMConcatMLP``
  ("film") or ``SimpleMLP`` ("concat") with one hidden layer of max(in, out)
  units, over the slot mask too. ``arity_mlp_central_module`` builds what the
  reference's model benchmark passes instead (``ArityMLPFactory`` with
  condition features, benchmark_relational_models.py:258-277).

Object embeddings start at zero (``initialize_embeddings``, no random init;
here in the parameters' dtype, so a float64 model runs end to end);
the updater is ``SimpleMLP(2D, 2D, D)``; activation "mish". ``forward(batch)``
returns ``(object embeddings [num_objects, D], object_state)``.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .hetero_mp import (
    BatchedRelationLayer,
    CentralFusedLayer,
    build_batched_routing,
    build_fused_routing,
)
from .nn import MLP, FiLMConcatMLP, ResidualModule, SimpleMLP, arity_relation_module
from .workloads import RelationalBatch


def _check_aggr(aggregation: str | None) -> str:
    aggr = (aggregation or "logsumexp").lower()
    if aggr not in ("sum", "logsumexp"):
        raise ValueError(f"aggregation must be 'sum' or 'logsumexp', got {aggregation!r}")
    return aggr


class RelationalGNN(nn.Module):
    def __init__(self, embedding_size: int, num_layers: int, aggregation: str | None, relations: dict, *,
                 relation_layers: int = 1, activation: str = "mish", ignore_zero_arity_relations: bool = True,
                 use_kernels: bool | None = None):
        super().__init__()
        self.embedding_size = int(embedding_size)
        self.num_layers = int(num_layers)
        self.relations = dict(relations)
        self.aggr = _check_aggr(aggregation)
        arities = {p: int(a) for p, a in self.relations.items() if int(a) > 0 or not ignore_zero_arity_relations}
        self.relation_arities = {p: a for p, a in arities.items() if a > 0}
        modules = {p: arity_relation_module(self.embedding_size, a, relation_layers, activation)
                   for p, a in self.relation_arities.items()}
        self.relation_layer = BatchedRelationLayer(modules, embedding_size=self.embedding_size, aggr=self.aggr,
                                                   use_kernels=use_kernels)
        self.embedding_updater = SimpleMLP(2 * self.embedding_size, 2 * self.embedding_size, self.embedding_size,
                                           activation)

    def forward(self, batch: RelationalBatch):
        x = torch.zeros((batch.num_objects, self.embedding_size), device=batch.object_state.device,
                        dtype=self.embedding_updater.mlp[0].weight.dtype)
        routing = build_batched_routing(batch, self.relation_arities)
        for _ in range(self.num_layers):
            _, m = self.relation_layer(x, routing)
            x = x + self.embedding_updater(torch.cat([x, m.to(x.dtype) if m.dtype != x.dtype else m], dim=1))
        return x, batch.object_state


def arity_mlp_central_module(feature_size: int, max_arity: int, condition_dim: int, layers: int = 1,
                             condition_position: str = "pre", act: str = "mish") -> nn.Module:
    """``ArityMLPFactory(feature_size, in_condition_features=condition_dim,
    residual=True, layers=layers)(max_arity)`` (models/mlp.py:186-239): residual
    MLP from [condition | arguments] to the arguments, hidden width max_arity*D."""

    width = int(feature_size) * int(max_arity)
    mlp = MLP(in_features=width + int(condition_dim), num_cells=[width] * int(layers), out_features=width, act=act)
    return ResidualModule(mlp, truncated_dim=width, truncate_right=condition_position == "post")


class CentralizedRelationalGNN(nn.Module):
    def __init__(self, embedding_size: int, num_layers: int, aggregation: str | None, relations: dict, *,
                 relation_condition_dim: int | None = None, condition_position: str = "pre",
                 central_module: nn.Module | None = None, central_residual: bool = True,
                 central_conditioning: str = "film", central_slot_mask: bool = True, activation: str = "mish",
                 use_kernels: bool | None = None):
        super().__init__()
        if central_conditioning not in ("concat", "film"):
            raise ValueError(f"central_conditioning must be 'concat' or 'film', got {central_conditioning!r}.")
        self.embedding_size = int(embedding_size)
        self.num_layers = int(num_layers)
        self.relations = dict(relations)
        self.aggr = _check_aggr(aggregation)
        cond_dim = int(relation_condition_dim) if relation_condition_dim else max(1, int(math.sqrt(embedding_size)))
        self.relation_condition_dim = cond_dim
        self.relation_condition_index = {p: i for i, p in enumerate(self.relations)}
        self.relation_condition_embedding = nn.Embedding(len(self.relations), cond_dim)
        self.max_relation_arity = max(self.relations.values(), default=0)
        self.relation_arities = {p: int(a) for p, a in self.relations.items() if int(a) > 0}
        mask_dim = self.max_relation_arity if central_slot_mask else 0
        feature_in = self.max_relation_arity * self.embedding_size + mask_dim
        out_size = self.max_relation_arity * self.embedding_size
        hidden = max(feature_in + cond_dim, out_size)
        if central_module is None:
            if central_conditioning == "film":
                mlp = FiLMConcatMLP(in_dim=feature_in, cond_dim=cond_dim, hidden_dims=[hidden], out_dim=out_size,
                                    condition_position=condition_position, act=activation)
            else:
                mlp = SimpleMLP(feature_in + cond_dim, hidden, out_size, activation)
            central_module = (ResidualModule(mlp, truncated_dim=out_size,
                                             truncate_right=condition_position == "post")
                              if central_residual else mlp)
        self.central_module = central_module
        self.central_layer = CentralFusedLayer(
            central_module=self.central_module, condition_embedding=self.relation_condition_embedding,
            max_arity=self.max_relation_arity, embedding_size=self.embedding_size,
            condition_position=condition_position, include_slot_mask=central_slot_mask, aggr=self.aggr,
            use_kernels=use_kernels,
        )
        self.embedding_updater = SimpleMLP(2 * self.embedding_size, 2 * self.embedding_size, self.embedding_size,
                                           activation)

    def forward(self, batch: RelationalBatch):
        x = torch.zeros((batch.num_objects, self.embedding_size), device=batch.object_state.device,
                        dtype=self.embedding_updater.mlp[0].weight.dtype)
        routing = build_fused_routing(batch, self.relation_arities, self.relation_condition_index,
                                      self.max_relation_arity, x.dtype)
        context = self.central_layer.context(routing)
        for _ in range(self.num_layers):
            _, m = self.central_layer(x, routing, context)
            x = x + self.embedding_updater(torch.cat([x, m.to(x.dtype) if m.dtype != x.dtype else m], dim=1))
        return x, batch.object_state


def train_loss(out) -> torch.Tensor:
    """The reference model benchmark's loss (benchmark_relational_models.py:287-295):
    mean square of the object embeddings."""

    x = out[0] if isinstance(out, tuple) else out
    return x.float().square().mean()
