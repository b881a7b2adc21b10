"""Activations and dense stacks shared by the model families.

Names and forms follow the reference's ``src/xnn/common/models/ops.py:334`` (activation factory:
``celu`` with alpha 0.1 as in ANI, ``ssp`` the shifted softplus of SchNet / PhysNet, ``softplus``
evaluated without the large-``x`` cut-off, ``scaled_tanh`` of RuNNer) and ``blocks.py:79,114``
(``MLP`` with its ``layers`` list, ``GatedMLP`` = ``mlp(x) * sigmoid(gate(x))``), so that state
dicts transplant between the two frameworks.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn.functional as F
from torch import Tensor, nn

_LOG2 = math.log(2.0)


def exact_softplus(x: Tensor) -> Tensor:
    """``log(1 + e^x)`` with a threshold above which the dropped tail is below rounding
    (40 in float64, 20 otherwise)."""
    return F.softplus(x, threshold=40.0 if x.dtype == torch.float64 else 20.0)


def shifted_softplus(x: Tensor) -> Tensor:
    """``ln(0.5 e^x + 0.5)``: zero at zero."""
    return exact_softplus(x) - _LOG2


class ShiftedSoftplus(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return shifted_softplus(x)


class Softplus(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return exact_softplus(x)


class GaussianActivation(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return torch.exp(-x * x)


class ScaledTanh(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return 1.59223 * torch.tanh(x)


class Square(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return x * x


_ACTIVATIONS = {
    "silu": nn.SiLU, "gelu": nn.GELU, "celu": lambda: nn.CELU(alpha=0.1), "gaussian": GaussianActivation,
    "tanh": nn.Tanh, "relu": nn.ReLU, "sigmoid": nn.Sigmoid, "ssp": ShiftedSoftplus, "softplus": Softplus,
    "scaled_tanh": ScaledTanh, "square": Square, "linear": nn.Identity,
}


def make_activation(activation) -> nn.Module:
    """A fresh activation module from its name (or the module itself)."""
    if isinstance(activation, nn.Module):
        return activation
    key = str(activation).lower()
    if key not in _ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r}; choose one of {sorted(_ACTIVATIONS)}")
    return _ACTIVATIONS[key]()


class MLP(nn.Module):
    """Dense layers with the activation between consecutive layers (and after the last with
    ``activate_last``)."""

    def __init__(self, sizes: Sequence[int], activation="gelu", activate_last: bool = False, bias: bool = True):
        super().__init__()
        sizes = [int(s) for s in sizes]
        if len(sizes) < 2:
            raise ValueError("an MLP needs an input and an output size")
        self.layers = nn.ModuleList(nn.Linear(a, b, bias=bias) for a, b in zip(sizes[:-1], sizes[1:]))
        self.act = make_activation(activation)
        self.activate_last = bool(activate_last)

    def forward(self, x: Tensor) -> Tensor:
        last = len(self.layers) - 1
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i < last or self.activate_last:
                x = self.act(x)
        return x


class GatedMLP(nn.Module):
    """``mlp(x) * sigmoid(gate(x))`` with two stacks of the same sizes."""

    def __init__(self, sizes: Sequence[int], activation="silu"):
        super().__init__()
        self.mlp = MLP(sizes, activation)
        self.gate = MLP(sizes, activation)

    def forward(self, x: Tensor) -> Tensor:
        return self.mlp(x) * torch.sigmoid(self.gate(x))


class GatedEquivariantBlock(nn.Module):
    """Scalars ``s (N, F_s)`` and vectors ``v (N, 3, F_v)`` -> gated outputs: the norms of a linear map
    of the vectors join the scalars in an MLP whose outputs are new scalars and gates of a second
    linear map of the vectors (PaiNN / TorchMD-Net readouts)."""

    def __init__(self, n_in_s: int, n_in_v: int, n_out_s: int, n_out_v: int, n_hidden=None,
                 scalar_activation: bool = True, n_norm=None, activation="silu"):
        super().__init__()
        n_hidden = n_in_s if n_hidden is None else int(n_hidden)
        n_norm = n_out_v if n_norm is None else int(n_norm)
        self.n_out_s, self.n_out_v, self.n_norm = n_out_s, n_out_v, n_norm
        self.lin_v = nn.Linear(n_in_v, n_norm + n_out_v, bias=False)
        self.net = nn.Sequential(nn.Linear(n_in_s + n_norm, n_hidden), make_activation(activation),
                                 nn.Linear(n_hidden, n_out_s + n_out_v))
        self.scalar_activation = scalar_activation
        self.act = make_activation(activation)

    def forward(self, s, v):
        v1, v2 = torch.split(self.lin_v(v), [self.n_norm, self.n_out_v], dim=-1)
        x = self.net(torch.cat([s, torch.linalg.norm(v1, dim=1)], -1))
        s_out, gate = x[:, :self.n_out_s], x[:, self.n_out_s:]
        return (self.act(s_out) if self.scalar_activation else s_out), gate.unsqueeze(1) * v2
