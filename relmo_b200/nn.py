"""Dense building blocks of the relational models, restated without torch_geometric.

Same structure and parameter shapes as relmo's model blocks, so the relational
models around the fan-out / fan-in ops compute what relmo's do:

* ``MLP`` - relmo ``models/mlp.py:10-50``: Linear -> act -> ... -> Linear.
* ``SimpleMLP`` - ``models/mlp.py:55-82``: Linear(in, h) -> act -> ... -> Linear(h, out).
* ``ResidualModule`` - ``models/residual.py``: x (truncated left or right) + f(x).
* ``arity_relation_module`` - what ``ArityMLPFactory(feature_size=D,
  residual=True, layers=L)(k)`` builds (``models/mlp.py:151-245``):
  ResidualModule(MLP(kD -> [kD]*L -> kD)).
* ``FiLM``, ``FiLMBlock``, ``FiLMMLP``, ``FiLMConcatMLP`` - ``models/film.py:10-195``.

Activations are resolved by name ("mish", "relu", "gelu", "silu", "tanh"), the
names relmo passes to torch_geometric's ``activation_resolver``.

These blocks are dense contractions run by cuBLAS through torch; they are not
part of the accelerated fan-out / fan-in path. ``Linear`` is ``nn.Linear``
(same parameters, same results) whose backward, for bf16/fp16 gradients,
takes the bias gradient as a matrix-vector product with a ones vector:
torch's column-sum reduction of a tall [rows, out] bf16 gradient ran at well
under a tenth of HBM bandwidth and was a third of the GPU time of a
decentralized train step (cfg4: 2.14 -> 1.89 s per step).
"""

from __future__ import annotations

import itertools
from typing import Callable, Iterable

import torch
import torch.nn.functional as F
from torch import nn

_ACTIVATIONS: dict[str, Callable[[], nn.Module]] = {
    "mish": nn.Mish,
    "relu": nn.ReLU,
    "gelu": nn.GELU,
    "silu": nn.SiLU,
    "swish": nn.SiLU,
    "tanh": nn.Tanh,
    "elu": nn.ELU,
}


class _LinearFn(torch.autograd.Function):
    """y = x W^T + b with the bias gradient as ones^T @ grad (a GEMV)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        return F.linear(x, weight, bias)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, grad):
        x, weight = ctx.saved_tensors
        g2 = grad.reshape(-1, grad.size(-1))
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = torch.matmul(grad, weight.to(grad.dtype))
        if ctx.needs_input_grad[1]:
            gw = g2.t().mm(x.reshape(-1, x.size(-1)).to(g2.dtype))
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = torch.mv(g2.t(), torch.ones(g2.size(0), device=g2.device, dtype=g2.dtype))
        return gx, gw, gb


class Linear(nn.Linear):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # Only 2-byte gradients take the GEMV bias path: fp32 column sums are
        # fast in torch, and the Python autograd node costs launch time that
        # small fp32 models (launch-bound) notice.
        low = x.dtype in (torch.bfloat16, torch.float16) or torch.is_autocast_enabled(x.device.type)
        if low and self.bias is not None:
            return _LinearFn.apply(x, self.weight, self.bias)
        return F.linear(x, self.weight, self.bias)


def activation(name: str | nn.Module | Callable | None) -> nn.Module:
    if name is None:
        return nn.Identity()
    if isinstance(name, nn.Module):
        return name
    if isinstance(name, str):
        key = name.strip().lower()
        if key not in _ACTIVATIONS:
            raise ValueError(f"unknown activation {name!r}")
        return _ACTIVATIONS[key]()
    return name()


class MLP(nn.Module):
    def __init__(self, *, in_features: int, num_cells: Iterable[int], out_features: int, act: str = "mish",
                 bias_last_layer: bool = True):
        super().__init__()
        dims = [int(in_features), *[int(x) for x in num_cells], int(out_features)]
        layers: list[nn.Module] = []
        for idx, (din, dout) in enumerate(itertools.pairwise(dims)):
            last = idx == len(dims) - 2
            layers.append(Linear(din, dout, bias=bias_last_layer if last else True))
            if not last:
                layers.append(activation(act))
        self.net = nn.Sequential(*layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.net(x)


class SimpleMLP(nn.Module):
    def __init__(self, in_size: int, embedding_size: int | Iterable[int], out_size: int, act: str = "mish"):
        super().__init__()
        sizes = tuple(embedding_size) if isinstance(embedding_size, Iterable) else (int(embedding_size),)
        layers: list[nn.Module] = [Linear(in_size, sizes[0]), activation(act)]
        for a, b in itertools.pairwise(sizes):
            layers += [Linear(a, b), activation(act)]
        layers.append(Linear(sizes[-1], out_size))
        self.mlp = nn.Sequential(*layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.mlp(x)


class ResidualModule(nn.Module):
    def __init__(self, module: nn.Module, truncated_dim: int | None = None, truncate_right: bool | None = None):
        super().__init__()
        self.module = module
        self.truncated_dim = truncated_dim
        self.truncate_right = truncate_right

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.truncated_dim is None or x.size(-1) == self.truncated_dim:
            return x + self.module(x)
        if self.truncate_right:
            return x[..., : self.truncated_dim] + self.module(x)
        return x[..., -self.truncated_dim :] + self.module(x)


def arity_relation_module(feature_size: int, arity: int, layers: int = 1, act: str = "mish") -> nn.Module:
    """Per-predicate update module of the decentralized model for arity k:
    x + MLP(x) over the k concatenated argument embeddings."""

    width = int(feature_size) * int(arity)
    return ResidualModule(MLP(in_features=width, num_cells=[width] * int(layers), out_features=width, act=act),
                          truncated_dim=width, truncate_right=False)


class FiLM(nn.Module):
    """h' = gamma(c) * h + beta(c)."""

    def __init__(self, cond_dim: int, feat_dim: int):
        super().__init__()
        self.to_gamma = Linear(cond_dim, feat_dim)
        self.to_beta = Linear(cond_dim, feat_dim)

    def forward(self, h: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
        return self.to_gamma(c) * h + self.to_beta(c)


class FiLMBlock(nn.Module):
    """Linear -> FiLM -> activation."""

    def __init__(self, in_dim: int, out_dim: int, cond_dim: int, act: str = "mish"):
        super().__init__()
        self.lin = Linear(in_dim, out_dim)
        self.film = FiLM(cond_dim, out_dim)
        self.act = activation(act)

    def forward(self, x: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        return self.act(self.film(self.lin(x), cond))


class FiLMMLP(nn.Module):
    def __init__(self, in_dim: int, hidden_dims: list[int], out_dim: int, cond_dim: int, act: str = "mish"):
        super().__init__()
        self.blocks = nn.ModuleList()
        prev = in_dim
        for h in hidden_dims:
            self.blocks.append(FiLMBlock(prev, h, cond_dim, act))
            prev = h
        self.out = Linear(prev, out_dim)

    def forward(self, x: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        h = x
        for blk in self.blocks:
            h = blk(h, cond)
        return self.out(h)


class FiLMConcatMLP(nn.Module):
    """FiLM MLP over one concatenated input, [cond, x] ("pre") or [x, cond] ("post")."""

    def __init__(self, *, in_dim: int, cond_dim: int, hidden_dims: list[int], out_dim: int,
                 condition_position: str = "pre", act: str = "mish"):
        super().__init__()
        if condition_position not in ("pre", "post"):
            raise ValueError(f"condition_position must be 'pre' or 'post', got {condition_position!r}.")
        if cond_dim < 1:
            raise ValueError(f"cond_dim must be >= 1, got {cond_dim}")
        self.in_dim = int(in_dim)
        self.cond_dim = int(cond_dim)
        self.condition_position = condition_position
        self.film_mlp = FiLMMLP(self.in_dim, list(hidden_dims), int(out_dim), self.cond_dim, act)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.size(-1) != self.in_dim + self.cond_dim:
            raise ValueError(f"Expected input feature size {self.in_dim + self.cond_dim}, got {x.size(-1)}.")
        if self.condition_position == "pre":
            cond, feats = x[..., : self.cond_dim], x[..., self.cond_dim :]
        else:
            feats, cond = x[..., : self.in_dim], x[..., self.in_dim :]
        return self.film_mlp(feats, cond)
