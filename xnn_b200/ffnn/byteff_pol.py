"""ByteFF-Pol: the polarizable member of the ByteFF family, for molecules and clusters.

The same graph transformer and bonded head as :class:`~xnn_b200.ffnn.byteff.ByteFF` (two-well bonds
and angles by default) with a polarizable nonbonded head (:class:`PolarizableHead`): charges from
bond charge increments and, from a predicted effective atomic volume ``V`` scaling free-atom
values (``C6 ~ V^2``, ``alpha ~ V^(4/3)``, ``R ~ V^(4/21)``), the dispersion, polarizability and size
of every atom, plus Born-Mayer and charge-transfer constants. Pair terms (kcal/mol) over every pair
beyond 1,3 of a structure (1,4 pairs scaled):

* repulsion ``a eps exp[lam (1 - r / r0)] + (s12 / r)^12``; dispersion ``-C6 / (s r0^6 + r^6)``;
  charge transfer ``-eps_ct r^-4 exp[-(lam_ct r / r0)^3]`` beyond 1,5; electrostatics ``k q_i q_j / r``
  (geometric means of ``eps, lam, C6, eps_ct, lam_ct``, arithmetic mean of ``r0``);
* polarization: induced point dipoles ``mu`` with ``A mu = E``, ``A`` the inverse polarizabilities
  and the Thole-damped dipole tensor between every two atoms (``u = a r^3 / sqrt(damp_i damp_j)``),
  ``E`` the damped field of the charges (zero from 1,2 and 1,3 neighbours, scaled at 1,4 and 1,5);
  ``E_pol = -k / 2 mu . E``. The dense solve is differentiable, so forces include the dipoles'
  response.

Weights load from the reference's state dicts (same module layout). Parity: the reference's
``ByteFFPol`` (``src/xnn/hybnn/models/byteff.py:1362``, isolated structures); the periodic (Ewald)
evaluation of cells is not built here.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .byteff import BondChargeIncrements, ByteFF, _fourier, _mlp, _torsion_cos
from .geometry import pair_vectors
from .opls import KCAL_TO_EV

_BOHR = 1.0 / 1.88973
_HARTREE = 627.509474
#: free-atom volume (bohr^3), polarizability (bohr^3), C6 (hartree bohr^6) and van der Waals radius
#: (bohr) per element, the Tkatchenko-Scheffler values (Phys. Rev. Lett. 102, 073005 (2009)) with the
#: released ByteFF-Pol models' volumes and ion-like entries (Li, Na, K)
FREE_ATOMS = {
    1: (7.9, 4.5, 6.5, 3.1), 3: (89.0, 1.38, 1.46, 2.65), 5: (47.1, 21.0, 99.5, 3.89),
    6: (35.7, 12.0, 46.6, 3.59), 7: (27.0, 7.4, 24.2, 3.34), 8: (22.7, 5.4, 15.6, 3.19),
    9: (18.6, 3.8, 9.5, 3.04), 11: (114.3, 2.67, 6.38, 2.91), 14: (99.5, 37.0, 305.0, 4.2),
    15: (95.7, 25.0, 185.0, 4.01), 16: (77.0, 19.6, 134.0, 3.86), 17: (66.7, 15.0, 94.6, 3.71),
    19: (219.4, 11.1, 64.3, 3.55), 35: (97.0, 20.0, 162.0, 3.93), 53: (152.2, 35.0, 385.0, 4.17),
}
N_ELEMENTS = 86


def free_atom_column(k: int) -> list:
    """Column ``k`` (0 volume, 1 polarizability, 2 C6, 3 radius) per element row ``Z - 1``, in
    Angstrom and kcal/mol."""
    unit = (_BOHR ** 3, _BOHR ** 3, _BOHR ** 6 * _HARTREE, _BOHR)[k]
    return [FREE_ATOMS.get(z, (0.0,) * 4)[k] * unit for z in range(1, N_ELEMENTS + 1)]


class PolarizableHead(nn.Module):
    """Charges and the repulsion, dispersion, polarization and charge-transfer parameters per atom."""

    def __init__(self, node_dim: int, edge_dim: int, pre=(256, 256, 3), out=(256, 3), charge_bound: float = 4.0,
                 lithium_volume: float = 13.0, lithium_alpha: Optional[float] = 1.0e-6,
                 lithium_damping: float = 0.2, damping_floor: float = 1.0e-6, lambda_scale: float = 5.0,
                 c6_scale: float = 1000.0, activation: str = "gelu"):
        super().__init__()
        self.lithium_volume, self.lithium_alpha = float(lithium_volume), lithium_alpha
        self.lithium_damping, self.damping_floor = float(lithium_damping), float(damping_floor)
        self.lambda_scale, self.c6_scale = float(lambda_scale), float(c6_scale)
        self.charge = BondChargeIncrements(node_dim, edge_dim, pre, out, charge_bound, activation)
        self.volume = _mlp(node_dim, out[0], 1, out[1], activation)
        self.lam = _mlp(node_dim, out[0], 1, out[1], activation)
        self.eps = _mlp(node_dim, out[0], 1, out[1], activation)
        self.ct_eps = _mlp(node_dim, out[0], 1, out[1], activation)
        self.ct_lam = _mlp(node_dim, out[0], 1, out[1], activation)
        self.register_buffer("volume_ref", torch.tensor(free_atom_column(0)), persistent=False)
        self.v_free = nn.Parameter(torch.tensor(free_atom_column(0)))
        self.alpha_free = nn.Parameter(torch.tensor(free_atom_column(1)))
        self.c6_free = nn.Parameter(torch.tensor(free_atom_column(2)) / self.c6_scale)
        self.r_free = nn.Parameter(torch.tensor(free_atom_column(3)))

    def forward(self, x: Tensor, e: Tensor, g: dict) -> Dict[str, Tensor]:
        z = g["element"]                                  # row Z - 1
        li = z == 2
        q = self.charge(x, e, g["bonds"], g["bond_edges"], g["formal"], g["atom_class"])
        head = lambda mlp: torch.exp(mlp(x).squeeze(-1))  # noqa: E731
        volume = head(self.volume) * self.volume_ref.to(x.dtype)[z]
        volume = torch.where(li, torch.full_like(volume, self.lithium_volume), volume)
        ratio = volume / self.v_free[z]
        alpha = (self.alpha_free[z] * ratio ** (4.0 / 3.0)).clamp_min(1.0e-6)
        if self.lithium_alpha is not None:
            alpha = torch.where(li, torch.full_like(alpha, float(self.lithium_alpha)), alpha)
        damp = torch.where(li, alpha.clamp_min(self.lithium_damping), alpha) if self.lithium_damping > 0 else alpha
        return {"charge": q, "volume": volume, "c6": (self.c6_free[z] * ratio ** 2 * self.c6_scale).clamp_min(1.0e-6),
                "r0": self.r_free[z] * ratio ** (4.0 / 21.0), "alpha": alpha, "damp": damp.clamp_min(self.damping_floor),
                "lam": head(self.lam) * self.lambda_scale, "eps": head(self.eps), "ct_eps": head(self.ct_eps),
                "ct_lam": head(self.ct_lam)}


@register_model("byteff_pol")
class ByteFFPol(ByteFF):
    """ByteFF-Pol bound to one system of molecules (every pair of a structure interacts); see the
    module notes. ``charge14``, ``vdw14``: 1,4 scale factors of the charges and of repulsion and
    dispersion; ``induction14``, ``induction15``: of the charges' polarizing field."""

    head = PolarizableHead
    nonbonded_defaults = dict(pre=(256, 256, 3), out=(256, 3))

    def __init__(self, graphs=None, species=None, *, graph: Optional[dict] = None, bonded: Optional[dict] = None,
                 nonbonded: Optional[dict] = None, members: int = 1,
                 supported_elements: Sequence[int] = (1, 3, 6, 7, 8, 9, 15, 16, 17),
                 coulomb_constant: float = 332.0637141491396, charge14: float = 0.5, vdw14: float = 0.5,
                 induction14: float = 0.5, induction15: float = 1.0, thole: float = 0.39,
                 dispersion_damping: float = 120.0, wall: float = 1.5, repulsion_prefactor: float = 6.0,
                 reference_positions=None):
        self.charge14, self.vdw14 = float(charge14), float(vdw14)
        self.induction14, self.induction15 = float(induction14), float(induction15)
        self.thole, self.dispersion_damping = float(thole), float(dispersion_damping)
        self.wall, self.repulsion_prefactor = float(wall), float(repulsion_prefactor)
        bonded = {**dict(pre=(256, 256, 3), out=(256, 4), tanh_output=20.0, form="two_well"), **(bonded or {})}
        super().__init__(graphs, species, graph=graph, bonded=bonded, nonbonded=nonbonded, members=members,
                         supported_elements=supported_elements, cutoff=None, coulomb_constant=coulomb_constant,
                         reference_positions=reference_positions)

    def _bind_pairs(self, n: int) -> None:
        super()._bind_pairs(n)
        dev = self._pairs12.device
        scale = 1.0 - torch.eye(n, dtype=torch.float64, device=dev)
        for p, v in ((self._pairs12, 0.0), (self._pairs13, 0.0), (self._pairs14, self.induction14),
                     (self._pairs15, self.induction15)):
            scale[p[0], p[1]] = v
            scale[p[1], p[0]] = v
        self.register_buffer("_field_scale", scale, persistent=False)
        is15 = torch.zeros(n, n, dtype=torch.bool, device=dev)
        is15[self._pairs15[0], self._pairs15[1]] = True
        is15 = is15 | is15.t()
        pl = self._pair_list
        self.register_buffer("_pair_is15", is15[pl[0], pl[1]], persistent=False)

    def _derive(self, p: dict) -> dict:
        nb = {k: p[k] for k in ("charge", "volume", "c6", "r0", "alpha", "damp", "lam", "eps", "ct_eps", "ct_lam")}
        out = super()._derive({k: v for k, v in p.items() if k not in nb})
        out.update(nb)
        return out

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        B = self._check(data)
        N, n = data.num_nodes, self.n_atoms
        plan = self._plan(B, data.pos.device)
        dt = data.model_dtype
        P = {k: v.to(dt) for k, v in self._params_cached().items()}
        A_ = {k: P[k][self._atom_src].repeat(B) for k in ("charge", "c6", "r0", "alpha", "damp", "lam", "eps",
                                                         "ct_eps", "ct_lam")}
        b, a, tp, ti, pr = (plan[k] for k in ("bonds", "angles", "propers", "impropers", "pairs"))
        vb = pair_vectors(data, b[0], b[1])
        e_bond = 0.5 * P["bond_k"][self._bonds_src].repeat(B) * (vb.norm(dim=1) - P["bond_x0"][self._bonds_src].repeat(B)) ** 2
        u, v = pair_vectors(data, a[1], a[0]), pair_vectors(data, a[1], a[2])
        theta = torch.atan2(torch.linalg.cross(u, v, dim=-1).norm(dim=-1), (u * v).sum(-1))
        e_angle = 0.5 * P["angle_k"][self._angles_src].repeat(B) * (theta - P["angle_x0"][self._angles_src].repeat(B)) ** 2

        def torsion_cos(t):
            return _torsion_cos(pair_vectors(data, t[0], t[1]), pair_vectors(data, t[1], t[2]),
                                pair_vectors(data, t[2], t[3]))
        e_tors = _fourier(torsion_cos(tp), P["proper_k"][self._propers_src].repeat(B, 1))
        e_impr = P["improper_k"][self._impropers_src].repeat(B, 1)[:, 0] * (1.0 - (2.0 * torsion_cos(ti) ** 2 - 1.0))
        # pairs beyond 1,3: the 1,4 pairs first
        i, j = pr
        is14 = plan["is14"]
        is15 = self._pair_is15.repeat(B)
        one = torch.ones(i.shape[0], dtype=dt, device=i.device)
        vdw_s = torch.where(is14, torch.full_like(one, self.vdw14), one)
        qq_s = torch.where(is14, torch.full_like(one, self.charge14), one)
        ct_on = (~(is14 | is15)).to(dt)
        gm = lambda key: torch.sqrt(A_[key][i] * A_[key][j])  # noqa: E731
        r0 = 0.5 * (A_["r0"][i] + A_["r0"][j])
        r = pair_vectors(data, i, j).norm(dim=1)
        rep = vdw_s * (self.repulsion_prefactor * gm("eps") * torch.exp(gm("lam") * (1.0 - r / r0))
                       + ((self.wall / r) ** 12 if self.wall > 0 else 0.0))
        disp = -vdw_s * gm("c6") / (self.dispersion_damping * r0 ** 6 + r ** 6)
        ct = -ct_on * gm("ct_eps") / r ** 4 * torch.exp(-(gm("ct_lam") * r / r0) ** 3)
        q = A_["charge"]
        elec = self.coulomb_constant * qq_s * q[i] * q[j] / r
        # polarization of each structure (dense, every pair)
        x = data.pos.to(dt).view(B, n, 3)
        mu, field = self._dipoles(x, q.view(B, n), A_["alpha"].view(B, n), A_["damp"].view(B, n))
        e_pol = -0.5 * self.coulomb_constant * (mu * field).sum(-1).reshape(-1)

        def halves(e):
            return scatter_sum(0.5 * e, i, N) + scatter_sum(0.5 * e, j, N)
        node = {"e_bond": scatter_sum(0.5 * e_bond, b[0], N) + scatter_sum(0.5 * e_bond, b[1], N),
                "e_angle": scatter_sum(e_angle, a[1], N), "e_torsion": scatter_sum(e_tors, tp[1], N),
                "e_improper": scatter_sum(e_impr, ti[0], N), "e_repulsion": halves(rep), "e_dispersion": halves(disp),
                "e_electrostatics": halves(elec), "e_charge_transfer": halves(ct), "e_polarization": e_pol}
        total = sum(node.values()) * KCAL_TO_EV
        out = {"node_energy": total, "energy": self.aggregate_energy(total, data),
               "induced_dipoles": mu.reshape(-1, 3), "charges": q, "node_features": q.unsqueeze(1)}
        out.update({k: v.view(B, -1).to(torch.float64).sum(1) * KCAL_TO_EV for k, v in node.items()})
        return out

    def _dipoles(self, x: Tensor, q: Tensor, alpha: Tensor, damp: Tensor):
        """Induced dipoles ``(B, n, 3)`` and the charges' damped field ``(B, n, 3)``."""
        B, n, _ = x.shape
        d = x.unsqueeze(1) - x.unsqueeze(2)                        # d[b, i, j] = x_j - x_i
        eye = torch.eye(n, dtype=torch.bool, device=x.device)
        r2 = torch.where(eye, torch.ones((), dtype=x.dtype, device=x.device), (d * d).sum(-1))
        r = torch.sqrt(r2)
        off = (~eye).to(x.dtype)
        u = self.thole * r * r2 / torch.sqrt(damp.unsqueeze(-1) * damp.unsqueeze(-2))
        ex = torch.exp(-u)
        l3 = (1.0 - ex) * off
        l5 = (1.0 - (1.0 + u) * ex).clamp_min(1.0e-6) * off
        r3 = r * r2
        scale = self._field_scale.to(x.dtype)
        field = -((scale * l3 / r3 * q.unsqueeze(-2)).unsqueeze(-1) * d).sum(2)
        I3 = torch.eye(3, dtype=x.dtype, device=x.device)
        T = (l3 / r3).unsqueeze(-1).unsqueeze(-1) * I3 - (3.0 * l5 / (r3 * r2)).unsqueeze(-1).unsqueeze(-1) * (
            d.unsqueeze(-1) * d.unsqueeze(-2))
        A = T.transpose(2, 3).reshape(B, 3 * n, 3 * n) + torch.diag_embed((1.0 / alpha).repeat_interleave(3, dim=-1))
        mu = torch.linalg.solve(A, field.reshape(B, 3 * n, 1)).reshape(B, n, 3)
        return mu, field

    @classmethod
    def from_config(cls, cfg) -> "ByteFFPol":
        e = dict(cfg.extra or {})
        kw = {k: e[k] for k in ("graph", "bonded", "nonbonded", "members", "supported_elements", "coulomb_constant",
                                "charge14", "vdw14", "induction14", "induction15", "thole", "dispersion_damping",
                                "wall", "repulsion_prefactor") if e.get(k) is not None}
        model = cls(**kw)
        if e.get("atomic_numbers") is not None and e.get("bonds") is not None:
            model.bind(e["atomic_numbers"], e["bonds"], e.get("bond_orders"), e.get("formal_charges"))
        return model
