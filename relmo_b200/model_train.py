"""RelationalGNN train steps over the fan-out / fan-in ops (the model-level
workloads of the path).

Model construction follows relmo's model benchmark
(``scripts/benchmark_relational_models.py:237-277``):

* decentralized: ``RelationalGNN`` whose per-predicate modules are
  ``ArityMLPFactory(feature_size=D, residual=True, layers=2)``;
* centralized: ``CentralizedRelationalGNN`` with ``relation_condition_dim =
  int(sqrt(D))``, central module ``ArityMLPFactory(feature_size=D,
  in_condition_features=cond_dim, residual=True, layers=1)`` and no slot mask.

One train step is forward, loss (mean square of the object embeddings,
benchmark_relational_models.py:287-295), backward and an AdamW update. A global
batch larger than fits at once is split into equal micro-batches whose losses
are averaged (gradient accumulation); under data parallelism each rank takes an
equal share of the states and DDP averages the gradients with one all-reduce per
bucket after the last micro-batch (``no_sync`` before it), so the update equals
the single-process full-batch update.
"""

from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass

import torch
from torch import nn

from .relational_gnn import CentralizedRelationalGNN, RelationalGNN, arity_mlp_central_module, train_loss
from .workloads import CFG3_ARITIES, CFG4_ARITIES, RelationalBatch, cfg3_batch, cfg4_batch


@dataclass(frozen=True)
class ModelConfig:
    name: str
    kind: str               # "centralized" | "decentralized"
    embedding_size: int
    num_layers: int
    aggregation: str
    arities: dict
    global_states: int
    autocast: torch.dtype | None

    def batch(self, seed: int = 0, device="cpu", states: int | None = None) -> RelationalBatch:
        n = self.global_states if states is None else int(states)
        return cfg3_batch(seed, device, n) if self.name == "cfg3" else cfg4_batch(seed, device, n)


CFG3 = ModelConfig("cfg3", "centralized", 32, 10, "logsumexp", CFG3_ARITIES, 256, None)
CFG4 = ModelConfig("cfg4", "decentralized", 128, 30, "sum", CFG4_ARITIES, 4096, torch.bfloat16)
CONFIGS = {"cfg3": CFG3, "cfg4": CFG4}


def build_model(kind: str, embedding_size: int, num_layers: int, aggregation: str, relations: dict, *,
                use_kernels: bool | None = None) -> nn.Module:
    if kind == "decentralized":
        return RelationalGNN(embedding_size, num_layers, aggregation, relations, relation_layers=2,
                             use_kernels=use_kernels)
    if kind == "centralized":
        cond = max(1, int(math.sqrt(int(embedding_size))))
        central = arity_mlp_central_module(embedding_size, max(relations.values(), default=0), cond, layers=1)
        return CentralizedRelationalGNN(embedding_size, num_layers, aggregation, relations,
                                        relation_condition_dim=cond, central_module=central,
                                        central_slot_mask=False, use_kernels=use_kernels)
    raise ValueError(f"Unknown model kind: {kind!r}")


def model_for(cfg: ModelConfig, *, seed: int = 0, device="cpu", use_kernels: bool | None = None) -> nn.Module:
    torch.manual_seed(int(seed))
    return build_model(cfg.kind, cfg.embedding_size, cfg.num_layers, cfg.aggregation, cfg.arities,
                       use_kernels=use_kernels).to(device)


def shard_states(num_states: int, rank: int, world: int) -> tuple[int, int]:
    """Equal contiguous share of the states for one rank."""

    if num_states % world:
        raise ValueError(f"{num_states} states do not split evenly over {world} ranks")
    per = num_states // world
    return rank * per, (rank + 1) * per


def micro_batches(batch: RelationalBatch, micro_states: int) -> list[RelationalBatch]:
    if micro_states <= 0 or micro_states >= batch.num_states:
        return [batch]
    if batch.num_states % micro_states:
        raise ValueError(f"{batch.num_states} states do not split into micro-batches of {micro_states}")
    return [batch.state_slice(lo, lo + micro_states) for lo in range(0, batch.num_states, micro_states)]


def train_step(model: nn.Module, optimizer: torch.optim.Optimizer, batches: list[RelationalBatch], *,
               autocast: torch.dtype | None = None) -> torch.Tensor:
    """One optimizer step over ``batches`` (micro-batches of one rank's share).
    ``model`` may be wrapped in DistributedDataParallel. Returns the step's loss
    as a device scalar (no host sync)."""

    optimizer.zero_grad(set_to_none=True)
    n = len(batches)
    device_type = batches[0].object_state.device.type
    total = None
    for i, b in enumerate(batches):
        sync = i == n - 1 or not hasattr(model, "no_sync")
        ctx = contextlib.nullcontext() if sync else model.no_sync()
        with ctx:
            amp = torch.autocast(device_type, dtype=autocast) if autocast is not None else contextlib.nullcontext()
            with amp:
                loss = train_loss(model(b)) / n
            loss.backward()
        total = loss.detach() if total is None else total + loss.detach()
    optimizer.step()
    return total


def make_optimizer(model: nn.Module) -> torch.optim.Optimizer:
    on_cuda = next(model.parameters()).is_cuda
    return torch.optim.AdamW(model.parameters(), lr=1e-3, fused=on_cuda or None)
