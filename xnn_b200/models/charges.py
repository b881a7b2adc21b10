"""Charge equilibration without coupling between the charges (closed form per structure).

The minimum of ``sum_i chi_i q_i + q_i^2 / (2 J_i)`` at a fixed net charge ``Q`` of every
structure is ``q_i = (lambda - chi_i) / J_i`` with ``lambda = (Q + sum chi_j / J_j) / sum 1 / J_j``;
the sum of inverse hardnesses is bounded below by ``1e-12`` (reference
``src/xnn/common/models/charge_solve.py:333``).
"""
from __future__ import annotations

import torch
from torch import Tensor

from ..ops.scatter import scatter_sum


def closed_form_charges(chi: Tensor, inverse_hardness: Tensor, total_charge: Tensor, batch: Tensor,
                        num_graphs: int) -> Tensor:
    sums = scatter_sum(torch.stack([inverse_hardness, chi * inverse_hardness], -1), batch, num_graphs)
    lam = (total_charge.to(chi.dtype) + sums[:, 1]) / sums[:, 0].clamp(min=1e-12)
    return (lam.index_select(0, batch) - chi) * inverse_hardness
