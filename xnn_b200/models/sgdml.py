"""(s)GDML (Chmiela et al., Sci. Adv. 3, e1603015, 2017; Nat. Commun. 9, 3887, 2018): kernel
ridge regression in the gradient domain on inverse-distance descriptors, with the symmetric
variant summing the kernel over the molecule's permutation group.

The energy of a structure with descriptor ``x`` is
``c + std * sum_{j,q} [g(|x - P_q x_j|) (x - P_q x_j) . P_q w_j + k(|x - P_q x_j|) e_j]``
(``g = -k'/r`` of the Matern kernel); forces are its negative position gradient. The closed-form
fit solves ``(H + lam I) alpha = -y / std`` for the force(-and-energy) kernel matrix
``H_ij = sum_q J_i^T (g I + t d d^T) P_q J_j`` (``J`` the descriptor Jacobians, ``d`` the
descriptor difference) and stores ``w_j = J_j alpha_j``. Buffers, fit options and the model-file
reader follow the reference (``src/xnn/krnn/models/sgdml.py:133-410``,
``common/sgdml_fit.py``, ``common/sgdml_io.py``).
"""
from __future__ import annotations

import math
import os
from typing import Dict, Optional, Sequence

import numpy as np
import torch
from torch import Tensor

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS
from ..krnn.descriptor import InverseDistances
from ..krnn.kernels import Matern, safe_norm
from .base import InteratomicPotential
from .registry import register_model

_SIZED = ("train_desc", "train_weights", "energy_coef", "perms", "perm_index", "lattice")
CHUNK = 1 << 22


def kernel_energy(x: Tensor, xp: Tensor, wp: Tensor, ec: Tensor, kernel: Matern) -> Tensor:
    """``sum_{j,q} g (x - xp_jq) . wp_jq + k e_j`` per row of ``x`` ``(B, D)``; ``xp``, ``wp`` ``(M, Q, D)``."""
    b, (m, q, d) = x.shape[0], xp.shape
    e = x.new_zeros(b)
    step = max(1, CHUNK // max(1, b * q * d))
    for s in range(0, m, step):
        diff = x[:, None, :] - xp[s:s + step].reshape(1, -1, d)
        r = safe_norm(diff)
        e = e + (kernel.g(r) * (diff * wp[s:s + step].reshape(1, -1, d)).sum(-1)).sum(-1)
        if ec.numel():
            e = e + kernel.k(r) @ ec[s:s + step].repeat_interleave(q)
    return e


@register_model("sgdml")
class SGDML(InteratomicPotential):
    head_modules = ("train_weights", "energy_coef", "c")
    _default_symmetries = True

    def __init__(self, species: Sequence, sigma: float = 10.0, kernel_order: int = 2, use_symmetries: bool = True,
                 cutoff: float = 1.0):
        super().__init__()
        self.species = [ATOMIC_NUMBERS[z] if isinstance(z, str) else int(z) for z in species]
        self.n_atoms = len(self.species)
        if self.n_atoms < 2:
            raise ValueError("a GDML model needs at least two atoms")
        self.sigma, self.kernel_order = float(sigma), int(kernel_order)
        self.kernel = Matern(self.sigma, self.kernel_order)
        self.use_symmetries = bool(use_symmetries)
        self.cutoff = float(cutoff)
        self.descriptor = InverseDistances(self.n_atoms)
        d = self.descriptor.dim
        f64 = torch.float64
        self.register_buffer("_species", torch.tensor(self.species, dtype=torch.long), persistent=False)
        self.register_buffer("train_desc", torch.zeros(0, d, dtype=f64))
        self.register_buffer("train_weights", torch.zeros(0, d, dtype=f64))
        self.register_buffer("energy_coef", torch.zeros(0, dtype=f64))
        self.register_buffer("perms", torch.arange(self.n_atoms).unsqueeze(0))
        self.register_buffer("perm_index", torch.arange(d).unsqueeze(0))
        self.register_buffer("std", torch.ones((), dtype=f64))
        self.register_buffer("c", torch.zeros((), dtype=f64))
        self.register_buffer("lattice", torch.zeros(0, 3, dtype=f64))
        self.register_buffer("length_scale", torch.tensor(self.sigma, dtype=f64))
        self.fit_options: Dict[str, object] = {}
        self.fit_info: Dict[str, object] = {}

    def set_kernel(self, sigma: float, kernel_order: Optional[int] = None) -> None:
        self.sigma = float(sigma)
        if kernel_order is not None:
            self.kernel_order = int(kernel_order)
        self.kernel = Matern(self.sigma, self.kernel_order)
        self.length_scale.fill_(self.sigma)

    def set_permutations(self, perms) -> None:
        p = torch.as_tensor(np.asarray(perms), dtype=torch.long).reshape(-1, self.n_atoms)
        self.perms = p.to(self.perms.device)
        self.perm_index = self.descriptor.permutation_index(p.tolist()).to(self.perms.device)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        for name in _SIZED:
            if prefix + name in state_dict:
                setattr(self, name, torch.empty_like(state_dict[prefix + name]))
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        if prefix + "length_scale" in state_dict:
            self.set_kernel(float(self.length_scale))

    def _apply(self, fn, recurse=True):
        kept = {k: v for k, v in self.named_buffers(recurse=False) if v.is_floating_point()}
        out = super()._apply(fn, recurse)
        for k, old in kept.items():      # the coefficients cancel to many digits: they stay float64
            setattr(self, k, old.to(device=getattr(self, k).device, dtype=torch.float64))
        return out

    def receptive_field(self) -> Optional[float]:
        return None

    def geometry(self, data: AtomicGraph):
        b = data.num_graphs
        if not bool((data.n_atoms == self.n_atoms).all()):
            raise ValueError(f"the model is built for {self.n_atoms} atoms; got {data.n_atoms.tolist()}")
        if not torch.equal(data.atomic_numbers.reshape(b, self.n_atoms), self._species.expand(b, self.n_atoms)):
            raise ValueError("the atoms are not the elements of the model in its order")
        pos = data.pos.reshape(b, self.n_atoms, 3).to(torch.float64)
        cell = None
        if data.cell is not None and data.pbc is not None and bool(data.pbc.any()):
            cell = data.cell.reshape(b, 3, 3).to(torch.float64)
        elif self.lattice.numel():
            cell = self.lattice.expand(b, 3, 3)
        return pos, cell

    def permuted_training_set(self):
        return self.train_desc[:, self.perm_index], self.train_weights[:, self.perm_index]

    def energy_of_descriptors(self, x: Tensor) -> Tensor:
        xp, wp = self.permuted_training_set()
        return self.c + self.std * kernel_energy(x, xp, wp, self.energy_coef, self.kernel)

    def forward(self, data: AtomicGraph) -> dict:
        pos, cell = self.geometry(data)
        e = self.energy_of_descriptors(self.descriptor(pos, cell))
        node = (e / self.n_atoms).index_select(0, data.batch)
        return {"node_energy": node.to(data.model_dtype), "energy": self.aggregate_energy(node, data)}

    # ------------------------------------------------------------------ fitting
    def fit(self, graphs, **kwargs) -> "SGDML":
        return fit_sgdml(self, graphs, **kwargs)

    def fit_closed_form(self, train, validation=None) -> "SGDML":
        return self.fit(train, validation=validation, **self.fit_options)

    @classmethod
    def from_config(cls, cfg) -> "SGDML":
        e = dict(cfg.extra or {})
        if e.get("model_file"):
            return load_sgdml_model(e["model_file"], cutoff=float(cfg.cutoff))
        sigma = e.get("sigma", [float(s) for s in range(10, 101, 10)])
        sigmas = [float(s) for s in sigma] if isinstance(sigma, (list, tuple)) else [float(sigma)]
        model = cls(e["species"], sigma=sigmas[0], kernel_order=int(e.get("kernel_order", 2)),
                    use_symmetries=bool(e.get("use_symmetries", cls._default_symmetries)), cutoff=float(cfg.cutoff))
        model.fit_options = {"sigma": sigmas if len(sigmas) > 1 else sigmas[0], "lam": float(e.get("lam", 1e-10)),
                             "energy_constraint": bool(e.get("energy_constraint", False)),
                             "use_energy": bool(e.get("use_energy", True))}
        return model


@register_model("gdml")
class GDML(SGDML):
    _default_symmetries = False

    def __init__(self, species: Sequence, sigma: float = 10.0, kernel_order: int = 2, use_symmetries: bool = False,
                 cutoff: float = 1.0):
        super().__init__(species, sigma, kernel_order, use_symmetries, cutoff)


def kernel_matrix(model: SGDML, x: Tensor, u: Tensor, energy_constraint: bool = False) -> Tensor:
    """The force(-energy) kernel matrix of the training set, negated (see module notes)."""
    m, d = x.shape
    n, n3 = model.n_atoms, 3 * model.n_atoms
    a, b = model.descriptor.pairs
    pidx = model.perm_index
    q = pidx.shape[0]
    ap, bp = a[pidx], b[pidx]                                   # (Q, D): atoms of the moved entries
    xp, up = x[:, pidx], u[:, pidx]                             # (M, Q, D), (M, Q, D, 3)
    off = m * n3
    K = x.new_zeros(off + (m if energy_constraint else 0), off + (m if energy_constraint else 0))
    combos = [(a[None, :].expand(q, d), ap, 1.0), (a[None, :].expand(q, d), bp, -1.0),
              (b[None, :].expand(q, d), ap, -1.0), (b[None, :].expand(q, d), bp, 1.0)]
    slot = (torch.arange(q, device=x.device)[:, None] * n)
    for i in range(m):
        diff = x[i][None, None, :] - xp                         # (M, Q, D)
        r = safe_norm(diff)
        g, t = model.kernel.g_and_t(r)
        # g J_i^T P_q J_j: outer products of the pair gradients, summed onto (atom of i, atom of j)
        outer = (g[:, :, None, None, None] * u[i][None, None, :, :, None] * up[:, :, :, None, :]).reshape(m, q * d, 9)
        pairs = x.new_zeros(m, n * n, 9)
        for ai, aj, sg in combos:
            pairs.index_add_(1, (ai * n + aj).reshape(-1), sg * outer)
        term = pairs.reshape(m, n, n, 3, 3).permute(0, 1, 3, 2, 4).reshape(m, n3, n3)
        # t (J_i^T d)(d^T P_q J_j)
        wv = diff[..., None] * u[i][None, None]                 # (M, Q, D, 3)
        w = x.new_zeros(m, q, n, 3).index_add(2, a, wv).index_add(2, b, -wv).reshape(m, q, n3)
        vv = (diff[..., None] * up).reshape(m, q * d, 3)
        v = (x.new_zeros(m, q * n, 3).index_add(1, (slot + ap).reshape(-1), vv)
             .index_add(1, (slot + bp).reshape(-1), -vv).reshape(m, q, n3))
        block = -(term + torch.einsum("mq,mqa,mqb->mab", t, w, v))
        rows = slice(i * n3, (i + 1) * n3)
        K[rows, :off] = block.permute(1, 0, 2).reshape(n3, off)
        if energy_constraint:
            K[rows, off:] = (g[..., None] * w).sum(1).t()
            K[off + i, :off] = (-(g[..., None] * v).sum(1)).reshape(-1)
            K[off + i, off:] = -model.kernel.k(r).sum(1)
    return K


def _solve(K: Tensor, y: Tensor, lam: float) -> Tensor:
    A = -K
    A.diagonal().add_(lam)
    chol, info = torch.linalg.cholesky_ex(A)
    if int(info) == 0:
        return -torch.cholesky_solve(y.unsqueeze(1), chol).squeeze(1)
    return -torch.linalg.solve(A, y)


def _stack(model: SGDML, graphs):
    pos, cells, energies, forces = [], [], [], []
    for g in graphs:
        p, c = model.geometry(g)
        pos.append(p.detach())
        if c is not None:
            cells.append(c.detach())
        energies.append(None if g.energy is None else g.energy.reshape(-1).to(torch.float64))
        if g.forces is None:
            raise ValueError("every training structure needs force labels")
        forces.append(g.forces.reshape(-1, model.n_atoms, 3).to(torch.float64))
    e = torch.cat(energies) if all(v is not None for v in energies) else None
    return torch.cat(pos), (torch.cat(cells) if cells else None), e, torch.cat(forces)


def _fit_one(model: SGDML, x: Tensor, u: Tensor, forces: Tensor, energies: Optional[Tensor], lam: float,
             use_energy: bool, energy_constraint: bool) -> None:
    m, n3 = x.shape[0], 3 * model.n_atoms
    y = forces.reshape(-1)
    mean_e = None
    if energy_constraint:
        if energies is None:
            raise ValueError("energy_constraint needs energy labels")
        mean_e = energies.mean()
        y = torch.cat([y, -energies + mean_e])
    std = y.std(unbiased=False)
    alpha = _solve(kernel_matrix(model, x, u, energy_constraint), y / std, lam)
    model.fit_info = {"solver": "analytic"}
    a, b = model.descriptor.pairs
    al = alpha[:m * n3].reshape(m, model.n_atoms, 3)
    model.train_desc = x.clone()
    model.train_weights = (u * (al[:, a] - al[:, b])).sum(-1)
    model.energy_coef = alpha[m * n3:].clone() if energy_constraint else x.new_zeros(0)
    model.std = std.clone()
    model.c = x.new_zeros(())
    if energy_constraint:
        model.c = mean_e.clone()
    elif use_energy and energies is not None:
        with torch.no_grad():
            model.c = (energies - model.energy_of_descriptors(x)).mean()


def force_rmse(model: SGDML, graphs) -> float:
    total, count = 0.0, 0
    for g in graphs:
        pos, cell = model.geometry(g)
        pos = pos.detach().requires_grad_(True)
        f = -torch.autograd.grad(model.energy_of_descriptors(model.descriptor(pos, cell)).sum(), pos)[0]
        ref = g.forces.reshape(f.shape).to(torch.float64)
        total += float(((f - ref) ** 2).sum())
        count += ref.numel()
    return math.sqrt(total / count)


def fit_sgdml(model: SGDML, graphs, sigma=None, lam: float = 1e-10, perms=None, use_energy: bool = True,
              energy_constraint: bool = False, validation=None, max_symmetry_samples: int = 1000,
              generator: Optional[torch.Generator] = None) -> SGDML:
    """Closed-form fit (with a choice of ``sigma`` by validation force error when several are given)."""
    model.double()
    pos, cell, energies, forces = _stack(model, graphs)
    if perms is None:
        if model.use_symmetries:
            from ..krnn.permutations import find_permutations
            sel = pos
            if pos.shape[0] > max_symmetry_samples:
                sel = pos[torch.randperm(pos.shape[0], generator=generator)[:max_symmetry_samples]]
            perms = find_permutations(sel.cpu().numpy(), model._species.cpu().numpy(),
                                      None if cell is None else cell[0].cpu().numpy())
        else:
            perms = torch.arange(model.n_atoms).unsqueeze(0)
    model.set_permutations(perms)
    if cell is not None:
        model.lattice = cell[0].clone()
    x, u = model.descriptor(pos, cell), model.descriptor.pair_gradients(pos, cell)
    sigmas = [model.sigma] if sigma is None else ([float(sigma)] if isinstance(sigma, (int, float))
                                                  else [float(s) for s in sigma])
    if len(sigmas) > 1 and not validation:
        raise ValueError("choosing among several sigma needs validation structures")
    best = (math.inf, None)
    for s in sigmas:
        model.set_kernel(s)
        _fit_one(model, x, u, forces, energies, lam, use_energy, energy_constraint)
        if len(sigmas) == 1:
            return model
        err = force_rmse(model, validation)
        if err < best[0]:
            best = (err, {"sigma": s, "state": {k: v.clone() for k, v in model.state_dict().items()}})
    model.set_kernel(best[1]["sigma"])
    model.load_state_dict(best[1]["state"])
    return model


def load_sgdml_model(path, cutoff: float = 1.0) -> SGDML:
    """A trained model from an sGDML ``.npz`` model file (float64, eval mode)."""
    with np.load(os.fspath(path), allow_pickle=True) as f:
        m = {k: f[k] for k in f.files}
    perms = np.asarray(m["perms"], dtype=np.int64)
    model = SGDML([int(z) for z in m["z"]], sigma=float(m["sig"]), use_symmetries=perms.shape[0] > 1, cutoff=cutoff)
    model.set_permutations(perms)
    model.train_desc = torch.as_tensor(np.asarray(m["R_desc"]).T.copy(), dtype=torch.float64)
    model.train_weights = torch.as_tensor(np.asarray(m["R_d_desc_alpha"]), dtype=torch.float64)
    if "alphas_E" in m:
        model.energy_coef = torch.as_tensor(np.asarray(m["alphas_E"]).ravel(), dtype=torch.float64)
    model.std = torch.tensor(float(m["std"]) if "std" in m else 1.0, dtype=torch.float64)
    model.c = torch.tensor(float(m["c"]), dtype=torch.float64)
    if "lattice" in m:
        model.lattice = torch.as_tensor(np.asarray(m["lattice"]).T.copy(), dtype=torch.float64)
    return model.double().eval()
