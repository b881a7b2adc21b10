"""ReaxFF reactive force field, evaluated as LAMMPS ``pair_style reaxff`` with ``fix qeq/reaxff``.

Bond orders follow from the interatomic distances of every pair within 5 A (sigma, pi and double-pi
parts, ``BO' = (1 + c) exp(p_bo1 (r / r_s)^p_bo2) - c + ...`` with the bond-order cutoff ``c``), are
corrected for over-coordination (``f1``) and 1-3 bond orders (``f4 f5``), and drive the
many-body terms; the equilibrated charges (EEM / QEq with shielded, tapered Coulomb) drive the
electrostatics. Energy terms, in eV per structure:

``e_bond`` (with the C-O triple-bond stabilisation), ``e_lone``, ``e_over``, ``e_under``,
``e_angle``, ``e_penalty``, ``e_three_conj`` (coalition), ``e_torsion``, ``e_four_conj``,
``e_hbond``, ``e_vdw`` (shielded Morse, optional inner wall), ``e_coulomb`` and ``e_self``
(``chi q + eta q^2`` of the charges).

The thresholds are LAMMPS's: bonds from an uncorrected order of ``c = 0.01 x`` the library's
``BO_cutoff``; angles and torsions over bonds above 0.001; hydrogen bonds over X-H bonds above
0.01 and H..Z distances within 7.5 A; nonbonded terms within the library's upper taper radius
(10 A) under the seventh-order taper. Forces differentiate the energy at fixed equilibrated
charges (as LAMMPS does). Parameters come from the MolSSI ``.frc`` form of the ReaxFF libraries.

Parity: the reference's ``ReaxFF`` under ``conventions="lammps"`` (``src/xnn/ffnn/models/reaxff.py:509``);
the ReaxFF-nn bond networks are not built here.
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS, SYMBOLS
from ..models.base import InteratomicPotential
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .frc import read_forcefield

#: LAMMPS's kcal/mol per eV in the charge self-energy, Coulomb constant (kcal A / (mol e^2)) in
#: the energy and (eV A / e^2) in the charge equilibration
SELF_KCAL = 23.02
C_ELE = 332.06371
QEQ_COULOMB = 14.4
#: LAMMPS's conversion of kcal/mol to eV (its real-to-metal units factor)
KCAL_TO_EV = 4.3364432032e-2
BOND_CUT = 5.0
THB_CUT = 0.001
THB_CUTSQ = 0.00001
HB_THRESHOLD = 0.01
HB_CUT = 7.5
MIN_SINE = 1e-10

DATA = Path(__file__).resolve().parent / "data" / "reaxff"


# ----------------------------------------------------------------------------- parameters
ATOM_KEYS = {  # frc column -> name
    "R0,alpha": "r_s", "Val": "valency", "m": "mass", "RvdW": "r_vdw", "Dij": "epsilon", "gamma": "gamma",
    "R0,pi": "r_pi", "Val,e": "valency_e", "alpha": "alpha", "gamma,w": "gamma_w", "Val,boc": "valency_boc",
    "Povun,5": "p_ovun5", "chi": "chi", "eta": "eta", "Phbond": "p_hbond", "R0,pi-pi": "r_pi_pi",
    "Plp,2": "p_lp2", "Pboc,4": "b_o_131", "Pboc,3": "b_o_132", "Pboc,5": "b_o_133", "Povun,2": "p_ovun2",
    "Pval,3": "p_val3", "Val,angle": "valency_val", "Pval,5": "p_val5", "Rcore,2": "rcore2", "Ecore,2": "ecore2",
    "Acore,2": "acore2",
}
BOND_KEYS = {
    "De,sigma": "De_s", "De,pi": "De_p", "De,pi-pi": "De_pp", "Pbe,1": "p_be1", "Pbe,2": "p_be2",
    "Pbo,5": "p_bo5", "13_boc": "v13cor", "Pbo,6": "p_bo6", "Povun,1": "p_ovun1", "Pbo,3": "p_bo3",
    "Pbo,4": "p_bo4", "Pbo_1": "p_bo1", "Pbo,1": "p_bo1", "Pbo,2": "p_bo2", "ovc": "ovc",
}
GENERAL_KEYS = {
    "Pboc,1": "p_boc1", "Pboc,2": "p_boc2", "Pcoa,2": "p_coa2", "Ptrip,4": "p_trip4", "Ptrip,3": "p_trip3",
    "kc2": "kc2", "Povun,6": "p_ovun6", "Ptrip,2": "p_trip2", "Povun,7": "p_ovun7", "Povun,8": "p_ovun8",
    "Ptrip,1": "p_trip1", "Rtaper,lower": "swa", "Rtaper,upper": "swb", "Pval,7": "p_val6",
    "Plp,1": "p_lp1", "Pval,9": "p_val9", "Pval,10": "p_val10", "Ppen,2": "p_pen2", "Ppen,3": "p_pen3",
    "Ppen,4": "p_pen4", "Ptor,2": "p_tor2", "Ptor,3": "p_tor3", "Ptor,4": "p_tor4", "Pcot,2": "p_cot2",
    "PvdW,1": "p_vdw1", "BO_cutoff": "bo_cut100", "Pcoa,4": "p_coa4", "Povun,4": "p_ovun4",
    "Povun,3": "p_ovun3", "Pval,8": "p_val8", "Pcoa,3": "p_coa3",
}


class ReaxFFLibrary:
    """A ReaxFF parameter library read from its MolSSI ``.frc`` form."""

    def __init__(self, path: Union[str, Path]):
        path = Path(path)
        if not path.exists() and (DATA / f"{path.name}").exists():
            path = DATA / path.name
        if not path.exists() and (DATA / f"{path}.frc").exists():
            path = DATA / f"{path}.frc"
        ff = read_forcefield(str(path))
        self.name = path.stem

        def rows(kind):
            for k, v in ff.sections.items():
                if k.startswith(kind):
                    yield from v.items()
        self.general: Dict[str, float] = {}
        for key, row in rows("reaxff_general_parameters"):
            name = GENERAL_KEYS.get(key[0])
            if name is not None:
                self.general[name] = float(row.values["Value"])
        self.atoms: Dict[str, Dict[str, float]] = {}
        for key, row in rows("reaxff_atomic_parameters"):
            d = self.atoms.setdefault(key[0], {})
            for col, val in row.values.items():
                if col in ATOM_KEYS:
                    d[ATOM_KEYS[col]] = float(val)
        self.bonds: Dict[Tuple[str, str], Dict[str, float]] = {}
        for key, row in rows("reaxff_bond_parameters"):
            d = self.bonds.setdefault(tuple(sorted(key)), {})
            for col, val in row.values.items():
                if col in BOND_KEYS:
                    d[BOND_KEYS[col]] = float(val)
        self.offdiag: Dict[Tuple[str, str], Dict[str, float]] = {}
        for key, row in rows("reaxff_off-diagonal_parameters"):
            v = row.values
            self.offdiag[tuple(sorted(key))] = {"D": float(v["Dij"]), "r_vdw": float(v["RvdW"]),
                                                "alpha": float(v["alpha"]), "r_s": float(v["R0,sigma"]),
                                                "r_p": float(v["R0,pi"]), "r_pp": float(v["R0,pi-pi"])}
        self.angles: Dict[Tuple[str, str, str], Dict[str, float]] = {}
        for key, row in rows("reaxff_angle_parameters"):
            v = row.values
            par = {"theta_00": float(v["Theta0"]), "p_val1": float(v["Pval,1"]), "p_val2": float(v["Pval,2"]),
                   "p_coa1": float(v["Pcoa,1"]), "p_val7": float(v["Pval,7"]), "p_pen1": float(v["Ppen,1"]),
                   "p_val4": float(v["Pval,4"])}
            a, b, c = key
            self.angles[(a, b, c)] = par
            self.angles[(c, b, a)] = par
        self.torsions: Dict[Tuple[str, str, str, str], Dict[str, float]] = {}
        for key, row in rows("reaxff_torsion_parameters"):
            v = row.values
            par = {"V1": float(v["V1"]), "V2": float(v["V2"]), "V3": float(v["V3"]),
                   "p_tor1": float(v["Ptor,1"]), "p_cot1": float(v["Pcot,1"])}
            self.torsions[tuple(key)] = par
            self.torsions[tuple(key[::-1])] = par
        self.hbonds: Dict[Tuple[str, str, str], Dict[str, float]] = {}
        for key, row in rows("reaxff_hydrogen-bond_parameters"):
            v = row.values
            self.hbonds[tuple(key)] = {"r0_hb": float(v["Rhb"]), "p_hb1": float(v["Ehb"]), "p_hb2": float(v["Thb"]),
                                       "p_hb3": float(v["Phb3"])}
        self.species = list(self.atoms)

    def torsion(self, a, b, c, d):
        for key in ((a, b, c, d), ("*", b, c, "*")):
            if key in self.torsions:
                return self.torsions[key]
        return None


# ----------------------------------------------------------------------------- helpers
def _taper(r: Tensor, swa: float, swb: float) -> Tensor:
    """LAMMPS's seventh-order taper between ``swa`` and ``swb`` (1 at ``swa``, 0 at ``swb``)."""
    d7 = (swb - swa) ** 7
    a2, a3, b2, b3 = swa * swa, swa ** 3, swb * swb, swb ** 3
    c = [(-35.0 * a3 * b2 * b2 + 21.0 * a2 * b3 * b2 - 7.0 * swa * b3 * b3 + b3 * b3 * swb) / d7,
         140.0 * a3 * b3 / d7, -210.0 * (a3 * b2 + a2 * b3) / d7, 140.0 * (a3 * swb + 3.0 * a2 * b2 + swa * b3) / d7,
         -35.0 * (a3 + 9.0 * a2 * swb + 9.0 * swa * b2 + b3) / d7, 84.0 * (a2 + 3.0 * swa * swb + b2) / d7,
         -70.0 * (swa + swb) / d7, 20.0 / d7]
    t = torch.full_like(r, c[7])
    for k in range(6, -1, -1):
        t = t * r + c[k]
    return t


def _cos_angle(u: Tensor, v: Tensor) -> Tensor:
    return (u * v).sum(-1) / (torch.linalg.norm(u, dim=-1) * torch.linalg.norm(v, dim=-1))


def _trunc(x: Tensor) -> Tensor:
    """C's integer conversion (towards zero) of a floating value."""
    return torch.trunc(x)


@register_model("reaxff")
class ReaxFF(InteratomicPotential):
    """ReaxFF (LAMMPS conventions) for the species of a ``.frc`` library; see the module notes.
    ``ffield``: a path or a shipped library name (e.g. ``"CHO_cho_2008"``)."""

    def __init__(self, ffield: Union[str, Path, ReaxFFLibrary] = "CHO_cho_2008", *,
                 species: Optional[Sequence] = None, qeq_tol: float = 1e-10, atomic_energies=None):
        super().__init__()
        lib = ffield if isinstance(ffield, ReaxFFLibrary) else ReaxFFLibrary(ffield)
        self.lib = lib
        names = list(lib.species) if species is None else [s if isinstance(s, str) else SYMBOLS[int(s)]
                                                          for s in species]
        self.names = names
        self.species = [ATOMIC_NUMBERS[s] for s in names]
        g = lib.general
        self.swa, self.swb = g.get("swa", 0.0), g.get("swb", 10.0)
        self.cutoff = float(self.swb)
        self.bo_cut = 0.01 * g.get("bo_cut100", 0.1)
        self.qeq_tol = float(qeq_tol)
        self.node_feature_dim = 1
        n = len(names)
        zmap = torch.full((120,), -1, dtype=torch.long)
        for k, z in enumerate(self.species):
            zmap[z] = k
        self.register_buffer("zmap", zmap)
        A = lambda key, default=0.0: torch.tensor([lib.atoms[s].get(key, default) for s in names],  # noqa: E731
                                                  dtype=torch.float64)
        for key in ("r_s", "valency", "mass", "r_vdw", "epsilon", "gamma", "r_pi", "valency_e", "alpha", "gamma_w",
                    "valency_boc", "p_ovun5", "chi", "eta", "p_hbond", "r_pi_pi", "p_lp2", "b_o_131", "b_o_132",
                    "b_o_133", "p_ovun2", "p_val3", "valency_val", "p_val5", "rcore2", "ecore2", "acore2"):
            self.register_buffer("a_" + key, A(key))
        self.a_eta.mul_(2.0)                                      # LAMMPS stores twice the file's eta
        self.register_buffer("a_nlp_opt", 0.5 * (self.a_valency_e - self.a_valency))
        self.register_buffer("a_heavy", (self.a_mass > 21.0))
        self.register_buffer("a_is_C", torch.tensor([s == "C" for s in names]))
        # two-body tables
        T = {k: torch.zeros(n, n, dtype=torch.float64) for k in (
            "r_s", "r_p", "r_pp", "p_boc3", "p_boc4", "p_boc5", "D", "alpha", "r_vdW", "gamma_w", "gamma", "rcore",
            "ecore", "acore", "De_s", "De_p", "De_pp", "p_be1", "p_be2", "p_bo1", "p_bo2", "p_bo3", "p_bo4", "p_bo5",
            "p_bo6", "p_ovun1", "v13cor", "ovc", "has_bond")}
        for i, si in enumerate(names):
            for j, sj in enumerate(names):
                ai, aj = lib.atoms[si], lib.atoms[sj]
                T["r_s"][i, j] = 0.5 * (ai["r_s"] + aj["r_s"])
                T["r_p"][i, j] = 0.5 * (ai["r_pi"] + aj["r_pi"])
                T["r_pp"][i, j] = 0.5 * (ai["r_pi_pi"] + aj["r_pi_pi"])
                T["p_boc3"][i, j] = math.sqrt(ai["b_o_132"] * aj["b_o_132"])
                T["p_boc4"][i, j] = math.sqrt(ai["b_o_131"] * aj["b_o_131"])
                T["p_boc5"][i, j] = math.sqrt(ai["b_o_133"] * aj["b_o_133"])
                T["D"][i, j] = math.sqrt(ai["epsilon"] * aj["epsilon"])
                T["alpha"][i, j] = math.sqrt(ai["alpha"] * aj["alpha"])
                T["r_vdW"][i, j] = 2.0 * math.sqrt(ai["r_vdw"] * aj["r_vdw"])
                T["gamma_w"][i, j] = math.sqrt(ai["gamma_w"] * aj["gamma_w"])
                T["gamma"][i, j] = (ai["gamma"] * aj["gamma"]) ** -1.5
                T["rcore"][i, j] = math.sqrt(ai.get("rcore2", 0.0) * aj.get("rcore2", 0.0))
                T["ecore"][i, j] = math.sqrt(ai.get("ecore2", 0.0) * aj.get("ecore2", 0.0))
                T["acore"][i, j] = math.sqrt(ai.get("acore2", 0.0) * aj.get("acore2", 0.0))
                od = lib.offdiag.get(tuple(sorted((si, sj))))
                if od is not None:
                    for key, tk, f in (("D", "D", 1.0), ("r_vdw", "r_vdW", 2.0), ("alpha", "alpha", 1.0),
                                       ("r_s", "r_s", 1.0), ("r_p", "r_p", 1.0), ("r_pp", "r_pp", 1.0)):
                        if od[key] > 0.0:
                            T[tk][i, j] = f * od[key]
                bp = lib.bonds.get(tuple(sorted((si, sj))))
                if bp is not None:
                    T["has_bond"][i, j] = 1.0
                    for key in ("De_s", "De_p", "De_pp", "p_be1", "p_be2", "p_bo1", "p_bo2", "p_bo3", "p_bo4", "p_bo5",
                                "p_bo6", "p_ovun1", "v13cor", "ovc"):
                        T[key][i, j] = bp.get(key, 0.0)
        for k, v in T.items():
            self.register_buffer("t_" + k, v)
        # van der Waals form (LAMMPS): shielding when any gamma_w > 0.5, inner wall when cores are set
        shield = bool((self.a_gamma_w > 0.5).any())
        core = bool(((self.a_rcore2 > 0.01) & (self.a_acore2 > 0.01)).any())
        self.vdw_shield, self.vdw_core = shield, core
        # three- and four-body tables (index by species triples / quadruples)
        ang = torch.zeros(n, n, n, 8, dtype=torch.float64)          # 7 parameters + present flag
        for i, si in enumerate(names):
            for j, sj in enumerate(names):
                for k, sk in enumerate(names):
                    p = lib.angles.get((si, sj, sk))
                    if p is not None:
                        ang[i, j, k] = torch.tensor([p["theta_00"], p["p_val1"], p["p_val2"], p["p_coa1"],
                                                     p["p_val7"], p["p_pen1"], p["p_val4"], 1.0])
        self.register_buffer("angle_par", ang)
        tor = torch.zeros(n, n, n, n, 6, dtype=torch.float64)
        for i, si in enumerate(names):
            for j, sj in enumerate(names):
                for k, sk in enumerate(names):
                    for l, sl in enumerate(names):
                        p = lib.torsion(si, sj, sk, sl)
                        if p is not None:
                            tor[i, j, k, l] = torch.tensor([p["V1"], p["V2"], p["V3"], p["p_tor1"], p["p_cot1"], 1.0])
        self.register_buffer("torsion_par", tor)
        hb = torch.zeros(n, n, n, 5, dtype=torch.float64)
        for (a, b, c), p in lib.hbonds.items():
            if a in names and b in names and c in names:
                hb[names.index(a), names.index(b), names.index(c)] = torch.tensor(
                    [p["r0_hb"], p["p_hb1"], p["p_hb2"], p["p_hb3"], 1.0])
        self.register_buffer("hbond_par", hb)
        self.atom_ref = nn.Embedding(120, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.atom_ref.weight.requires_grad_(False)
        if atomic_energies is not None:
            with torch.no_grad():
                for z, v in dict(atomic_energies).items():
                    self.atom_ref.weight[int(z), 0] = float(v)

    # ------------------------------------------------------------------ pairs
    def _pairs(self, data: AtomicGraph):
        """Each neighbour pair once (``src < dst``, or an image of itself with a positive shift):
        indices, shifts and vectors ``pos[dst] - pos[src] + shift @ cell``."""
        src, dst = data.edge_index
        vec = data.edge_vectors()
        if data.cell is not None and data.cell_shifts is not None and data.cell_shifts.numel():
            sh = data.cell_shifts
            pos = (sh[:, 0] > 0) | ((sh[:, 0] == 0) & ((sh[:, 1] > 0) | ((sh[:, 1] == 0) & (sh[:, 2] > 0))))
            keep = (src < dst) | ((src == dst) & pos)
            sh = sh[keep]
        else:
            keep = src < dst
            sh = None
        return src[keep], dst[keep], vec[keep], sh

    # ------------------------------------------------------------------ charges
    def _qeq(self, data: AtomicGraph, t: Tensor, i: Tensor, j: Tensor, r: Tensor) -> Tensor:
        """Charge equilibration: ``H s = -chi``, ``H u = -1``, ``q = s - (sum s / sum u) u`` per
        structure (``H`` diagonal ``eta``, off-diagonal the tapered shielded Coulomb in eV)."""
        n = t.shape[0]
        dev, dt = r.device, r.dtype
        gam = self.t_gamma.to(dt)[t[i], t[j]]
        Hij = QEQ_COULOMB * _taper(r, self.swa, self.swb) / (r * r * r + gam) ** (1.0 / 3.0)
        B = data.num_graphs
        q = torch.zeros(n, dtype=dt, device=dev)
        for b in range(B):
            sel = (data.batch == b).nonzero()[:, 0]
            m = sel.shape[0]
            loc = torch.full((n,), -1, dtype=torch.long, device=dev)
            loc[sel] = torch.arange(m, device=dev)
            pm = (loc[i] >= 0)
            H = torch.zeros(m, m, dtype=dt, device=dev)
            H.index_put_((loc[i[pm]], loc[j[pm]]), Hij[pm].detach(), accumulate=True)
            H = H + H.t()
            H = H + torch.diag(self.a_eta.to(dt)[t[sel]])
            rhs = torch.stack([-self.a_chi.to(dt)[t[sel]], -torch.ones(m, dtype=dt, device=dev)], 1)
            sol = torch.linalg.solve(H, rhs)
            s, u = sol[:, 0], sol[:, 1]
            tot = 0.0 if data.total_charge is None else float(data.total_charge[b])
            q[sel] = s - ((s.sum() - tot) / u.sum()) * u
        return q

    # ------------------------------------------------------------------ forward
    def forward(self, data: AtomicGraph) -> dict:
        dt = data.pos.dtype if data.pos.dtype == torch.float64 else torch.float32
        t = self.zmap[data.atomic_numbers]
        if bool((t < 0).any()):
            raise ValueError("an atom's element is not in this ReaxFF library's species")
        n = t.shape[0]
        dev = data.pos.device
        g = self.lib.general
        P = lambda name: getattr(self, name).to(dt)  # noqa: E731
        i, j, vec, sh = self._pairs(data)
        vec = vec.to(dt)
        r = torch.linalg.norm(vec, dim=-1)
        ti, tj = t[i], t[j]
        B = data.num_graphs
        batch = data.batch
        out: Dict[str, Tensor] = {}

        # ---------------------------------------------------------- uncorrected bond orders
        near = r < BOND_CUT
        bi, bj, bv, br = i[near], j[near], vec[near], r[near]
        bsh = sh[near] if sh is not None else None
        tti, ttj = t[bi], t[bj]
        rs_ok = (P("a_r_s")[tti] > 0) & (P("a_r_s")[ttj] > 0)
        rp_ok = (P("a_r_pi")[tti] > 0) & (P("a_r_pi")[ttj] > 0)
        rpp_ok = (P("a_r_pi_pi")[tti] > 0) & (P("a_r_pi_pi")[ttj] > 0)
        tb = lambda name: getattr(self, "t_" + name).to(dt)[tti, ttj]  # noqa: E731
        c = self.bo_cut
        safe = lambda x: torch.where(x > 0, x, torch.ones_like(x))  # noqa: E731
        bo_s = torch.where(rs_ok, (1.0 + c) * torch.exp(tb("p_bo1") * (br / safe(tb("r_s"))) ** tb("p_bo2")), 0.0)
        bo_pi = torch.where(rp_ok, torch.exp(tb("p_bo3") * (br / safe(tb("r_p"))) ** tb("p_bo4")), 0.0)
        bo_pp = torch.where(rpp_ok, torch.exp(tb("p_bo5") * (br / safe(tb("r_pp"))) ** tb("p_bo6")), 0.0)
        bo = bo_s + bo_pi + bo_pp
        keep = (bo >= c) & (tb("has_bond") > 0)
        bi, bj, bv, br = bi[keep], bj[keep], bv[keep], br[keep]
        bsh = bsh[keep] if bsh is not None else None
        tti, ttj = t[bi], t[bj]
        bo_s, bo_pi, bo_pp, bo = bo_s[keep] - c, bo_pi[keep], bo_pp[keep], bo[keep] - c
        nb = bi.shape[0]
        tot_p = scatter_sum(bo, bi, n) + scatter_sum(bo, bj, n)

        # ---------------------------------------------------------- corrected bond orders
        Dp = tot_p - P("a_valency")[t]
        Dp_boc = tot_p - P("a_valency_val")[t]
        val_i, val_j = P("a_valency")[tti], P("a_valency")[ttj]
        ovc = tb("ovc") >= 0.001
        v13 = tb("v13cor") >= 0.001
        p1, p2 = g["p_boc1"], g["p_boc2"]
        Dpi, Dpj = Dp[bi], Dp[bj]
        f2 = torch.exp(-p1 * Dpi) + torch.exp(-p1 * Dpj)
        f3 = -1.0 / p2 * torch.log(0.5 * (torch.exp(-p2 * Dpi) + torch.exp(-p2 * Dpj)))
        f1 = 0.5 * ((val_i + f2) / (val_i + f2 + f3) + (val_j + f2) / (val_j + f2 + f3))
        f1 = torch.where(ovc, f1, torch.ones_like(f1))
        pb3, pb4, pb5 = tb("p_boc3"), tb("p_boc4"), tb("p_boc5")
        f4 = 1.0 / (1.0 + torch.exp(-(pb4 * bo * bo - Dp_boc[bi]) * pb3 + pb5))
        f5 = 1.0 / (1.0 + torch.exp(-(pb4 * bo * bo - Dp_boc[bj]) * pb3 + pb5))
        f45 = torch.where(v13, f4 * f5, torch.ones_like(f4))
        corr = ovc | v13
        A0 = f1 * f45
        BO = torch.where(corr, bo * A0, bo)
        BOpi = torch.where(corr, bo_pi * A0 * f1, bo_pi)
        BOpp = torch.where(corr, bo_pp * A0 * f1, bo_pp)
        BOs = BO - (BOpi + BOpp)
        z0 = torch.zeros_like(BO)
        BO = torch.where(BO < 1e-10, z0, BO)
        BOs = torch.where(BOs < 1e-10, z0, BOs)
        BOpi = torch.where(BOpi < 1e-10, z0, BOpi)
        BOpp = torch.where(BOpp < 1e-10, z0, BOpp)
        tot = scatter_sum(BO, bi, n) + scatter_sum(BO, bj, n)

        # ---------------------------------------------------------- atom quantities
        Delta = tot - P("a_valency")[t]
        Delta_e = tot - P("a_valency_e")[t]
        Delta_boc = tot - P("a_valency_boc")[t]
        Delta_val = tot - P("a_valency_val")[t]
        vlpex = Delta_e - 2.0 * _trunc(Delta_e / 2.0)
        plp1 = g["p_lp1"]
        explp1 = torch.exp(-plp1 * (2.0 + vlpex) ** 2)
        nlp = explp1 - _trunc(Delta_e / 2.0)
        Delta_lp = P("a_nlp_opt")[t] - nlp
        Clp = 2.0 * plp1 * explp1 * (2.0 + vlpex)
        heavy = self.a_heavy[t]
        nlp_temp = torch.where(heavy, 0.5 * (P("a_valency_e")[t] - P("a_valency")[t]), nlp)
        Delta_lp_temp = P("a_nlp_opt")[t] - nlp_temp
        nbonds = scatter_sum(torch.ones_like(BO), bi, n) + scatter_sum(torch.ones_like(BO), bj, n)

        # ---------------------------------------------------------- bond energy
        pbe1, pbe2 = tb("p_be1"), tb("p_be2")
        pow_bos = torch.where(BOs > 0, BOs, torch.ones_like(BOs)) ** pbe2
        pow_bos = torch.where(BOs > 0, pow_bos, torch.zeros_like(BOs))
        e_b = -tb("De_s") * BOs * torch.exp(pbe1 * (1.0 - pow_bos)) - tb("De_p") * BOpi - tb("De_pp") * BOpp
        mi, mj = P("a_mass")[tti], P("a_mass")[ttj]
        co = ((mi == 12.0) & (mj == 15.999)) | ((mj == 12.0) & (mi == 15.999))
        trip = (BO >= 1.0) & co
        exphu = torch.exp(-g["p_trip2"] * (BO - 2.5) ** 2)
        exphua = torch.exp(-g["p_trip4"] * (tot[bi] - BO))
        exphub = torch.exp(-g["p_trip4"] * (tot[bj] - BO))
        exphuov = torch.exp(g["p_trip3"] * (Delta[bi] + Delta[bj]))
        e_trip = g["p_trip1"] * exphu / (1.0 + 25.0 * exphuov) * (exphua + exphub)
        e_b = e_b + torch.where(trip, e_trip, torch.zeros_like(e_trip))
        bond_graph = batch[bi]
        out["e_bond"] = scatter_sum(e_b, bond_graph, B)

        # ---------------------------------------------------------- lone pair, over / under
        e_lp = P("a_p_lp2")[t] * Delta_lp / (1.0 + torch.exp(-75.0 * Delta_lp))
        kc2 = g.get("kc2", 0.0)
        if kc2 > 0.001:
            both_c = self.a_is_C[tti] & self.a_is_C[ttj]
            e_c2 = torch.zeros_like(BO)
            for side in (bi, bj):
                Di = Delta[side]
                vov3 = BO - Di - 0.040 * Di ** 4
                e_c2 = e_c2 + torch.where(both_c & (vov3 > 3.0), kc2 * (vov3 - 3.0) ** 2, torch.zeros_like(vov3))
            e_c2_atom = scatter_sum(e_c2, bond_graph, B)
        else:
            e_c2_atom = torch.zeros(B, dtype=dt, device=dev)
        out["e_lone"] = scatter_sum(e_lp, batch, B) + e_c2_atom
        dfvl = torch.where(heavy, 0.0, 1.0).to(dt)
        pov1De = tb("p_ovun1") * tb("De_s") * BO
        sum1 = scatter_sum(pov1De, bi, n) + scatter_sum(pov1De, bj, n)
        pis = BOpi + BOpp
        sum2 = (scatter_sum((Delta[bj] - dfvl[bj] * Delta_lp_temp[bj]) * pis, bi, n)
                + scatter_sum((Delta[bi] - dfvl[bi] * Delta_lp_temp[bi]) * pis, bj, n))
        exp_ovun1 = g["p_ovun3"] * torch.exp(g["p_ovun4"] * sum2)
        Dlpcorr = Delta - dfvl * Delta_lp_temp / (1.0 + exp_ovun1)
        exp_ovun2 = torch.exp(P("a_p_ovun2")[t] * Dlpcorr)
        e_ov = sum1 * Dlpcorr / (Dlpcorr + P("a_valency")[t] + 1e-8) / (1.0 + exp_ovun2)
        exp_ovun6 = torch.exp(g["p_ovun6"] * Dlpcorr)
        exp_ovun8 = g["p_ovun7"] * torch.exp(g["p_ovun8"] * sum2)
        e_un = -P("a_p_ovun5")[t] * (1.0 - exp_ovun6) / (1.0 + 1.0 / exp_ovun2) / (1.0 + exp_ovun8)
        out["e_over"] = scatter_sum(e_ov, batch, B)
        out["e_under"] = scatter_sum(e_un, batch, B)

        # ---------------------------------------------------------- valence angles
        # incidence: each bond seen from both ends, with the vector from the centre
        cen = torch.cat([bi, bj])
        oth = torch.cat([bj, bi])
        bvec = torch.cat([bv, -bv])
        bid = torch.cat([torch.arange(nb, device=dev), torch.arange(nb, device=dev)])
        order = torch.argsort(cen, stable=True)
        cen, oth, bvec, bid = cen[order], oth[order], bvec[order], bid[order]
        deg = torch.bincount(cen, minlength=n)
        start = torch.cumsum(deg, 0) - deg
        # pairs (a, b) of incidences of one centre with a < b
        pa, pb = _pairs_within(deg, start)
        j3 = cen[pa]
        ia, ka = oth[pa], oth[pb]
        u1, u2 = bvec[pa], bvec[pb]
        cos_t = _cos_angle(u1, u2).clamp(-1.0, 1.0)
        theta = torch.acos(cos_t)
        BO1, BO2 = BO[bid[pa]], BO[bid[pb]]
        # SBO of the centre
        bo8 = BO ** 8                                     # prod_t exp(-BO_t^8) = exp(-sum_t BO_t^8)
        prod_sbo = torch.exp(-(scatter_sum(bo8, bi, n) + scatter_sum(bo8, bj, n)))
        sbop = scatter_sum(pis, bi, n) + scatter_sum(pis, bj, n)
        pval8 = g["p_val8"]
        vlpadj = torch.where(vlpex >= 0, torch.zeros_like(nlp), nlp)
        SBO = sbop + (1.0 - prod_sbo) * (-Delta_boc - pval8 * vlpadj)
        pv9 = g["p_val9"]
        SBO_c = SBO.clamp(1e-30, 2.0 - 1e-30)
        SBO2 = torch.where(SBO <= 0, torch.zeros_like(SBO),
                           torch.where(SBO <= 1, SBO_c ** pv9,
                                       torch.where(SBO < 2, 2.0 - (2.0 - SBO_c) ** pv9, torch.full_like(SBO, 2.0))))
        expval6 = torch.exp(g["p_val6"] * Delta_boc)
        ap = self.angle_par.to(dt)[t[ia], t[j3], t[ka]]
        BOA1, BOA2 = BO1 - THB_CUT, BO2 - THB_CUT
        use = ((BOA1 > 0) & (BOA2 > 0) & (BO1 > THB_CUT) & (BO2 > THB_CUT) & (BO1 * BO2 > THB_CUTSQ)
               & (ap[:, 7] > 0) & (ap[:, 1].abs() > 0.001))
        theta_00, p_val1, p_val2, p_coa1, p_val7, p_pen1, p_val4 = ap[:, :7].unbind(-1)
        pval3, pval5 = P("a_p_val3")[t[j3]], P("a_p_val5")[t[j3]]
        BOA1s, BOA2s = BOA1.clamp_min(1e-30), BOA2.clamp_min(1e-30)
        f7a = 1.0 - torch.exp(-pval3 * BOA1s ** p_val4)
        f7b = 1.0 - torch.exp(-pval3 * BOA2s ** p_val4)
        expval7 = torch.exp(-p_val7 * Delta_boc[j3])
        trm8 = 1.0 + expval6[j3] + expval7
        f8 = pval5 - (pval5 - 1.0) * (2.0 + expval6[j3]) / trm8
        theta0 = (180.0 - theta_00 * (1.0 - torch.exp(-g["p_val10"] * (2.0 - SBO2[j3])))) * math.pi / 180.0
        expv2 = torch.exp(-p_val2 * (theta0 - theta) ** 2)
        e12 = torch.where(p_val1 >= 0, p_val1 * (1.0 - expv2), -p_val1 * expv2)
        e_ang = f7a * f7b * f8 * e12
        exp_pen2a = torch.exp(-g["p_pen2"] * (BOA1 - 2.0) ** 2)
        exp_pen2b = torch.exp(-g["p_pen2"] * (BOA2 - 2.0) ** 2)
        exp_pen3 = torch.exp(-g["p_pen3"] * Delta[j3])
        exp_pen4 = torch.exp(g["p_pen4"] * Delta[j3])
        f9 = (2.0 + exp_pen3) / (1.0 + exp_pen3 + exp_pen4)
        e_pen = p_pen1 * f9 * exp_pen2a * exp_pen2b
        exp_coa2 = torch.exp(g["p_coa2"] * Delta_val[j3])
        e_coa = (p_coa1 / (1.0 + exp_coa2) * torch.exp(-g["p_coa3"] * (tot[ia] - BOA1) ** 2)
                 * torch.exp(-g["p_coa3"] * (tot[ka] - BOA2) ** 2) * torch.exp(-g["p_coa4"] * (BOA1 - 1.5) ** 2)
                 * torch.exp(-g["p_coa4"] * (BOA2 - 1.5) ** 2))
        zero3 = torch.zeros_like(e_ang)
        ag = batch[j3]
        out["e_angle"] = scatter_sum(torch.where(use, e_ang, zero3), ag, B)
        out["e_penalty"] = scatter_sum(torch.where(use, e_pen, zero3), ag, B)
        out["e_three_conj"] = scatter_sum(torch.where(use, e_coa, zero3), ag, B)

        # ---------------------------------------------------------- torsions
        e_tor, e_cot, tg = self._torsions(n, nb, bi, bj, bv, BO, BOpi, Delta_boc, cen, oth, bvec, bid, deg, start,
                                          t, dt, batch)
        out["e_torsion"] = scatter_sum(e_tor, tg, B)
        out["e_four_conj"] = scatter_sum(e_cot, tg, B)

        # ---------------------------------------------------------- hydrogen bonds
        out["e_hbond"] = self._hbonds(data, t, i, j, vec, r, bi, bj, bv, BO, B, dt)

        # ---------------------------------------------------------- nonbonded
        tap = _taper(r, self.swa, self.swb)
        inside = r < self.swb
        tp = lambda name: getattr(self, "t_" + name).to(dt)[ti, tj]  # noqa: E731
        if self.vdw_shield:
            pv = g["p_vdw1"]
            fn13 = (r ** pv + (1.0 / tp("gamma_w")) ** pv) ** (1.0 / pv)
        else:
            fn13 = r
        a_, rv = tp("alpha"), tp("r_vdW")
        e_vdw = tp("D") * (torch.exp(a_ * (1.0 - fn13 / rv)) - 2.0 * torch.exp(0.5 * a_ * (1.0 - fn13 / rv)))
        if self.vdw_core:
            rc = tp("rcore")
            e_vdw = e_vdw + tp("ecore") * torch.exp(tp("acore") * (1.0 - r / torch.where(rc > 0, rc, torch.ones_like(rc))))
        w = torch.ones_like(r)         # an atom's own image pair is kept once (one of +-shift)
        pg = batch[i]
        out["e_vdw"] = scatter_sum(torch.where(inside, w * tap * e_vdw, torch.zeros_like(r)), pg, B)
        with torch.no_grad():
            q = self._qeq(data, t, i, j, r)
        shield = (r ** 3 + tp("gamma")) ** (1.0 / 3.0)
        e_c = C_ELE * q[i] * q[j] * tap / shield
        out["e_coulomb"] = scatter_sum(torch.where(inside, w * e_c, torch.zeros_like(r)), pg, B)
        e_self = SELF_KCAL * (P("a_chi")[t] * q + 0.5 * P("a_eta")[t] * q * q)
        out["e_self"] = scatter_sum(e_self, batch, B)

        terms = {k: v * KCAL_TO_EV for k, v in out.items()}
        e_ref = self.atom_ref(data.atomic_numbers).squeeze(-1).to(dt)
        terms["e_ref"] = scatter_sum(e_ref, batch, B)
        energy = sum(terms.values())
        counts = torch.bincount(batch, minlength=B).to(dt)
        node = ((energy - terms["e_ref"]) / counts)[batch] + e_ref
        res = {"node_energy": node, "energy": energy, "charges": q, "node_features": q[:, None]}
        res.update(terms)
        return res

    # ------------------------------------------------------------------ four-body
    def _torsions(self, n, nb, bi, bj, bv, BO, BOpi, Delta_boc, cen, oth, bvec, bid, deg, start, t, dt, batch):
        g = self.lib.general
        dev = BO.device
        # central bond (j, k) = (bi, bj) once; i from j's other bonds, l from k's other bonds
        ok = BO > THB_CUT
        cb = ok.nonzero()[:, 0]
        jc, kc = bi[cb], bj[cb]
        # expand i over incidences of j, l over incidences of k
        ii, jj = _expand(deg[jc], start[jc])                   # incidence index, central-bond row
        ll, kk = _expand(deg[kc], start[kc])
        # keep incidences that are not the central bond itself and are above threshold
        ki = (bid[ii] != cb[jj]) & (BO[bid[ii]] > THB_CUT)
        kl = (bid[ll] != cb[kk]) & (BO[bid[ll]] > THB_CUT)
        ii, jj = ii[ki], jj[ki]
        ll, kk = ll[kl], kk[kl]
        # combine per central bond: all (i, l) pairs
        ci = torch.bincount(jj, minlength=cb.shape[0])
        cl = torch.bincount(kk, minlength=cb.shape[0])
        si = torch.cumsum(ci, 0) - ci
        sl = torch.cumsum(cl, 0) - cl
        # ii, ll are sorted by central bond already (expanded in order)
        cnt = ci * cl
        row = torch.repeat_interleave(torch.arange(cb.shape[0], device=dev), cnt)
        off = torch.arange(int(cnt.sum()), device=dev) - torch.repeat_interleave(torch.cumsum(cnt, 0) - cnt, cnt)
        a_idx = si[row] + torch.div(off, cl[row].clamp_min(1), rounding_mode="floor")
        b_idx = sl[row] + off % cl[row].clamp_min(1)
        inc_i, inc_l = ii[a_idx], ll[b_idx]
        c_row = cb[row]
        j4, k4 = bi[c_row], bj[c_row]
        i4, l4 = oth[inc_i], oth[inc_l]
        v_ji = bvec[inc_i]                     # x_i - x_j
        v_jk = bv[c_row]                       # x_k - x_j
        v_kl = bvec[inc_l]                     # x_l - x_k
        # distinct atoms: i and l differ unless they are the same image
        same = (i4 == l4) & ((v_ji - (v_jk + v_kl)).abs().sum(-1) < 1e-6)
        BOij, BOjk, BOkl = BO[bid[inc_i]], BO[c_row], BO[bid[inc_l]]
        tp = self.torsion_par.to(dt)[t[i4], t[j4], t[k4], t[l4]]
        use = (~same) & (tp[:, 5] > 0) & (BOij * BOjk * BOkl > THB_CUT)
        # angles at j (i-j-k) and at k (j-k-l)
        cos_ijk = _cos_angle(v_ji, v_jk).clamp(-1.0, 1.0)
        cos_jkl = _cos_angle(-v_jk, v_kl).clamp(-1.0, 1.0)
        sin_ijk = torch.sin(torch.acos(cos_ijk))
        sin_jkl = torch.sin(torch.acos(cos_jkl))
        rjk2 = (v_jk * v_jk).sum(-1)
        cos_un = -(v_ji * v_jk).sum(-1) * (v_jk * v_kl).sum(-1) + rjk2 * (v_ji * v_kl).sum(-1)
        sin_un = -torch.sqrt(rjk2) * (v_ji * torch.cross(v_jk, v_kl, dim=-1)).sum(-1)
        omega = torch.atan2(sin_un, cos_un)
        BOA_ij, BOA_jk, BOA_kl = BOij - THB_CUT, BOjk - THB_CUT, BOkl - THB_CUT
        Dj, Dk = Delta_boc[j4], Delta_boc[k4]
        e3 = torch.exp(-g["p_tor3"] * (Dj + Dk))
        e4 = torch.exp(g["p_tor4"] * (Dj + Dk))
        f11 = (2.0 + e3) / (1.0 + e3 + e4)
        V1, V2, V3, ptor1, pcot1 = tp[:, :5].unbind(-1)
        exp_tor1 = torch.exp(ptor1 * (2.0 - BOpi[c_row] - f11) ** 2)
        fn10 = ((1.0 - torch.exp(-g["p_tor2"] * BOA_ij)) * (1.0 - torch.exp(-g["p_tor2"] * BOA_jk))
                * (1.0 - torch.exp(-g["p_tor2"] * BOA_kl)))
        CV = 0.5 * (V1 * (1.0 + torch.cos(omega)) + V2 * exp_tor1 * (1.0 - torch.cos(2.0 * omega))
                    + V3 * (1.0 + torch.cos(3.0 * omega)))
        e_tor = fn10 * sin_ijk * sin_jkl * CV
        pc2 = g["p_cot2"]
        fn12 = (torch.exp(-pc2 * (BOA_ij - 1.5) ** 2) * torch.exp(-pc2 * (BOA_jk - 1.5) ** 2)
                * torch.exp(-pc2 * (BOA_kl - 1.5) ** 2))
        e_cot = pcot1 * fn12 * (1.0 + (torch.cos(omega) ** 2 - 1.0) * sin_ijk * sin_jkl)
        z = torch.zeros_like(e_tor)
        return torch.where(use, e_tor, z), torch.where(use, e_cot, z), batch[j4]

    # ------------------------------------------------------------------ hydrogen bonds
    def _hbonds(self, data, t, i, j, vec, r, bi, bj, bv, BO, B, dt):
        ph = self.a_p_hbond
        dev = r.device
        # X-H bonds with X an acceptor-capable atom and BO >= 0.01, oriented H -> X
        hb_b = BO >= HB_THRESHOLD
        h_first = (ph[t[bi]] == 1) & (ph[t[bj]] == 2) & hb_b
        h_second = (ph[t[bj]] == 1) & (ph[t[bi]] == 2) & hb_b
        H = torch.cat([bi[h_first], bj[h_second]])
        X = torch.cat([bj[h_first], bi[h_second]])
        v_hx = torch.cat([bv[h_first], -bv[h_second]])
        bo_hx = torch.cat([BO[h_first], BO[h_second]])
        if H.numel() == 0:
            return torch.zeros(B, dtype=dt, device=dev)
        # H..Z pairs within the hydrogen-bond cutoff (both orientations of the pair list)
        close = r < HB_CUT
        pi_, pj_, pv = i[close], j[close], vec[close]
        hz_h = torch.cat([pi_, pj_])
        hz_z = torch.cat([pj_, pi_])
        hz_v = torch.cat([pv, -pv])                            # x_Z - x_H
        keep = (ph[t[hz_h]] == 1) & (ph[t[hz_z]] == 2)
        hz_h, hz_z, hz_v = hz_h[keep], hz_z[keep], hz_v[keep]
        # join on the hydrogen: every X-H bond with every H..Z pair of the same H
        order = torch.argsort(H, stable=True)
        H, X, v_hx, bo_hx = H[order], X[order], v_hx[order], bo_hx[order]
        n = t.shape[0]
        cnt_b = torch.bincount(H, minlength=n)
        st_b = torch.cumsum(cnt_b, 0) - cnt_b
        rows_b = cnt_b[hz_h]
        pair_idx = torch.repeat_interleave(torch.arange(hz_h.shape[0], device=dev), rows_b)
        offs = torch.arange(int(rows_b.sum()), device=dev) - torch.repeat_interleave(torch.cumsum(rows_b, 0) - rows_b,
                                                                                   rows_b)
        b_idx = st_b[hz_h[pair_idx]] + offs
        Z, hz = hz_z[pair_idx], hz_v[pair_idx]
        Xb, vx, bo = X[b_idx], v_hx[b_idx], bo_hx[b_idx]
        distinct = ~((Z == Xb) & ((hz - vx).abs().sum(-1) < 1e-6))
        par = self.hbond_par.to(dt)[t[Xb], t[hz_h[pair_idx]], t[Z]]
        use = (distinct & (par[:, 4] > 0) & (par[:, 0] > 0)).nonzero()[:, 0]
        par, hz, vx, bo, Z, pair_idx = par[use], hz[use], vx[use], bo[use], Z[use], pair_idx[use]
        r0, p1, p2, p3 = par[:, 0], par[:, 1], par[:, 2], par[:, 3]
        rhz = torch.linalg.norm(hz, dim=-1)
        cos_t = _cos_angle(vx, hz).clamp(-1.0, 1.0)
        theta = torch.acos(cos_t)
        s4 = torch.sin(theta / 2.0) ** 4
        r0s = torch.where(r0 > 0, r0, torch.ones_like(r0))
        e = p1 * (1.0 - torch.exp(-p2 * bo)) * torch.exp(-p3 * (r0s / rhz + rhz / r0s - 2.0)) * s4
        return scatter_sum(e, data.batch[hz_h[pair_idx]], B)

    @classmethod
    def from_config(cls, cfg) -> "ReaxFF":
        e = dict(cfg.extra or {})
        return cls(e.get("ffield", "CHO_cho_2008"), species=e.get("species"))


def _pairs_within(deg: Tensor, start: Tensor) -> Tuple[Tensor, Tensor]:
    """All ``(a, b)``, ``a < b``, of incidence positions within each centre's segment."""
    dev = deg.device
    npairs = deg * (deg - 1) // 2
    cen = torch.repeat_interleave(torch.arange(deg.shape[0], device=dev), npairs)
    off = torch.arange(int(npairs.sum()), device=dev) - torch.repeat_interleave(torch.cumsum(npairs, 0) - npairs,
                                                                              npairs)
    d = deg[cen].to(torch.float64)
    # row a of the upper triangle: pairs before row a = a (2d - a - 1) / 2
    a = torch.floor(((2 * d - 1) - torch.sqrt((2 * d - 1) ** 2 - 8 * off.to(torch.float64))) / 2).long()
    before = a * (2 * deg[cen] - a - 1) // 2
    b = a + 1 + (off - before)
    return start[cen] + a, start[cen] + b


def _expand(cnt: Tensor, st: Tensor) -> Tuple[Tensor, Tensor]:
    """Positions ``st[r] .. st[r] + cnt[r] - 1`` for every row ``r`` and the row of each."""
    dev = cnt.device
    rows = torch.repeat_interleave(torch.arange(cnt.shape[0], device=dev), cnt)
    off = torch.arange(int(cnt.sum()), device=dev) - torch.repeat_interleave(torch.cumsum(cnt, 0) - cnt, cnt)
    return st[rows] + off, rows
