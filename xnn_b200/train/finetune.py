"""Fine-tuning: LoRA low-rank updates, multi-head models, parameter freezing.

Capabilities follow the reference's ``src/xnn/common/finetune`` (``inject_lora`` /
``merge_lora`` in ``lora.py:318``, ``MultiHead`` in ``heads.py:134``, ``freeze_parameters`` in
``freeze.py:10``); the mechanism here is different. A LoRA update is a weight
*parametrization* (``torch.nn.utils.parametrize``): reading ``module.weight`` returns
``W + (alpha / r) A B`` everywhere, so the fused CUDA paths, which read the weights directly,
train the adapted model without knowing about LoRA. An e3nn-layout linear (one flat weight
holding several ``mul_in x mul_out`` path blocks) gets one low-rank factor pair per path.
"""
from __future__ import annotations

import copy
import fnmatch
import math
from typing import Dict, Iterable, List, Optional, Sequence, Union

import torch
from torch import Tensor, nn
from torch.nn.utils import parametrize

from ..data.atomic_graph import AtomicGraph
from ..models.base import InteratomicPotential

DEFAULT_RANK = 4
DEFAULT_ALPHA = 1.0
DEFAULT_INIT_STD = 1e-3


# --------------------------------------------------------------------------- LoRA
class LoRAUpdate(nn.Module):
    """``W -> W + (alpha / rank) * delta`` with ``delta`` a product of two thin factors per
    block; ``blocks`` lists the ``(offset, rows, cols)`` of every block of the (flattened)
    weight, ``shape`` the weight's own shape."""

    def __init__(self, shape: torch.Size, blocks: List[tuple], rank: int, alpha: float, init_std: float,
                 dtype: torch.dtype, device):
        super().__init__()
        self.shape = tuple(shape)
        self.blocks = blocks
        self.rank, self.scale = int(rank), float(alpha) / float(rank)
        self.lora_in = nn.ParameterList()
        self.lora_out = nn.ParameterList()
        for _, rows, cols in blocks:
            r = min(self.rank, rows, cols)
            self.lora_in.append(nn.Parameter(torch.randn(rows, r, dtype=dtype, device=device) * init_std))
            self.lora_out.append(nn.Parameter(torch.zeros(r, cols, dtype=dtype, device=device)))

    def delta(self) -> Tensor:
        parts = [(a @ b).reshape(-1) for a, b in zip(self.lora_in, self.lora_out)]
        return (torch.cat(parts) * self.scale).reshape(self.shape)

    def forward(self, weight: Tensor) -> Tensor:
        return weight + self.delta().to(weight.dtype)


def _blocks_of(module: nn.Module) -> Optional[List[tuple]]:
    """Low-rank blocks of ``module.weight``, or ``None`` if LoRA does not apply."""
    w = getattr(module, "weight", None)
    if not isinstance(w, nn.Parameter) or w.numel() == 0:
        return None
    instr = getattr(module, "instructions", None)
    if w.dim() == 1 and instr is not None:                # e3nn-layout linear: one block per path
        out, off = [], 0
        for p in instr:
            shape = tuple(p.path_shape)
            if len(shape) != 2:
                return None
            out.append((off, shape[0], shape[1]))
            off += shape[0] * shape[1]
        return out if off == w.numel() else None
    if w.dim() == 2:
        return [(0, w.shape[0], w.shape[1])]
    return None


def inject_lora(model: nn.Module, rank: int = DEFAULT_RANK, alpha: float = DEFAULT_ALPHA,
                init_std: float = DEFAULT_INIT_STD, exclude: Sequence[str] = (), freeze: bool = True,
                trainable: Sequence[str] = ()) -> nn.Module:
    """Give every linear layer of ``model`` a LoRA update (in place); the model computes exactly
    what it did until the factors train. ``exclude``: ``fnmatch`` patterns of module names left
    alone; ``freeze`` freezes everything but the factors and the ``trainable`` patterns."""
    count = 0
    for name, mod in list(model.named_modules()):
        if any(fnmatch.fnmatchcase(name, pat) for pat in exclude) or parametrize.is_parametrized(mod, "weight"):
            continue
        if isinstance(mod, LoRAUpdate):
            continue
        blocks = _blocks_of(mod)
        if blocks is None:
            continue
        w = mod.weight
        parametrize.register_parametrization(mod, "weight", LoRAUpdate(w.shape, blocks, rank, alpha, init_std,
                                                                       w.dtype, w.device))
        count += 1
    if count == 0:
        raise ValueError(f"{type(model).__name__} has no linear layer LoRA can adapt")
    if freeze:
        for n, p in model.named_parameters():
            p.requires_grad = is_lora_name(n) or any(fnmatch.fnmatchcase(n, pat) for pat in trainable)
    return model


def is_lora_name(name: str) -> bool:
    parts = name.split(".")
    return "lora_in" in parts or "lora_out" in parts


def lora_parameters(model: nn.Module) -> Iterable[nn.Parameter]:
    for n, p in model.named_parameters():
        if is_lora_name(n):
            yield p


def has_lora(model: nn.Module) -> bool:
    return any(isinstance(m, LoRAUpdate) for m in model.modules())


def merge_lora(model: nn.Module) -> nn.Module:
    """Fold every LoRA update into its weight (in place): a plain model again."""
    for mod in list(model.modules()):
        if parametrize.is_parametrized(mod, "weight") and any(
                isinstance(p, LoRAUpdate) for p in mod.parametrizations["weight"]):
            parametrize.remove_parametrizations(mod, "weight", leave_parametrized=True)
    return model


# --------------------------------------------------------------------------- freezing
def freeze_parameters(model: nn.Module, freeze: Sequence[str] = (), trainable: Sequence[str] = ()) -> int:
    """Freeze the parameters whose names match ``freeze`` (``fnmatch``) unless they match
    ``trainable``; returns how many parameters stay trainable."""
    for n, p in model.named_parameters():
        if any(fnmatch.fnmatchcase(n, pat) for pat in freeze) and not any(
                fnmatch.fnmatchcase(n, pat) for pat in trainable):
            p.requires_grad = False
    return count_parameters(model, trainable_only=True)


def count_parameters(model: nn.Module, trainable_only: bool = False) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad or not trainable_only)


# --------------------------------------------------------------------------- multi-head
def head_module_names(model: nn.Module) -> tuple:
    names = tuple(getattr(model, "head_modules", ()) or ())
    if not names:
        raise TypeError(f"{type(model).__name__} declares no head_modules; it cannot carry several heads")
    return names


class _HeadCopy(nn.Module):
    """Copies of a model's head modules (parameters and buffers of one extra head)."""

    def __init__(self, model: nn.Module, names: Sequence[str]):
        super().__init__()
        self.names = list(names)
        self.mods = nn.ModuleDict({n.replace(".", "__"): copy.deepcopy(model.get_submodule(n)) for n in names})

    def overrides(self) -> Dict[str, Tensor]:
        out: Dict[str, Tensor] = {}
        for n in self.names:
            mod = self.mods[n.replace(".", "__")]
            for k, v in list(mod.named_parameters()) + list(mod.named_buffers()):
                out[f"{n}.{k}"] = v
        return out


class MultiHead(InteratomicPotential):
    """Several readout heads over one shared trunk; structure ``b`` uses head ``data.head[b]``.

    Head 0 is the wrapped model's own readout; the others are copies of its ``head_modules``.
    A batch that mixes heads runs the trunk once per head present, on that head's structures."""

    def __init__(self, model: InteratomicPotential, heads: Sequence[str]):
        super().__init__()
        heads = [str(h) for h in heads]
        if not heads or len(set(heads)) != len(heads):
            raise ValueError(f"heads must be distinct names, got {heads}")
        self.model = model
        self.heads = heads
        self.head_module_names = head_module_names(model)
        self.cutoff = getattr(model, "cutoff", None)
        self.node_feature_dim = getattr(model, "node_feature_dim", None)
        self.extra_heads = nn.ModuleList([_HeadCopy(model, self.head_module_names) for _ in heads[1:]])

    def receptive_field(self):
        rf = getattr(self.model, "receptive_field", None)
        return rf() if callable(rf) else None

    def index(self, head: Union[int, str]) -> int:
        if isinstance(head, str):
            if head not in self.heads:
                raise KeyError(f"unknown head {head!r}; this model has {self.heads}")
            return self.heads.index(head)
        if not 0 <= int(head) < len(self.heads):
            raise KeyError(f"head index {head} out of range for {self.heads}")
        return int(head)

    def _run(self, head: int, data: AtomicGraph) -> Dict[str, Tensor]:
        if head == 0:
            return self.model(data)
        return torch.func.functional_call(self.model, self.extra_heads[head - 1].overrides(), (data,))

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        if data.head is None or len(self.heads) == 1:
            return self._run(0, data)
        present = [int(h) for h in torch.unique(data.head).tolist()]
        if max(present) >= len(self.heads):
            raise IndexError(f"a structure asks for head {max(present)}; this model has {self.heads}")
        if len(present) == 1:
            return self._run(present[0], data)
        node_head = data.head[data.batch]
        outs, g_idx, n_idx = [], [], []
        for h in present:
            keep = data.head == h
            outs.append(self._run(h, data.subset(keep)))
            g_idx.append(keep.nonzero().squeeze(-1))
            n_idx.append((node_head == h).nonzero().squeeze(-1))
        g_order, n_order = torch.cat(g_idx), torch.cat(n_idx)
        inv_g = torch.empty_like(g_order)
        inv_g[g_order] = torch.arange(g_order.numel(), device=g_order.device)
        inv_n = torch.empty_like(n_order)
        inv_n[n_order] = torch.arange(n_order.numel(), device=n_order.device)
        merged: Dict[str, Tensor] = {}
        for key in outs[0]:
            vals = [o.get(key) for o in outs]
            if any(v is None or not torch.is_tensor(v) for v in vals):
                continue
            if vals[0].dim() == 0:
                merged[key] = torch.stack(vals).sum()
                continue
            cat = torch.cat(vals, 0)
            if cat.shape[0] == data.num_nodes and key != "energy":
                merged[key] = cat[inv_n]
            elif cat.shape[0] == data.num_graphs:
                merged[key] = cat[inv_g]
        return merged

    def select(self, head: Union[int, str]) -> InteratomicPotential:
        """A standalone copy of the model with ``head``'s parameters (for deployment)."""
        h = self.index(head)
        m = copy.deepcopy(self.model)
        if h > 0:
            with torch.no_grad():
                for k, v in self.extra_heads[h - 1].overrides().items():
                    owner, _, leaf = k.rpartition(".")
                    getattr(m.get_submodule(owner), leaf).copy_(v)
        return m
