"""DREIDING (Mayo, Olafson & Goddard, J. Phys. Chem. 94, 8897 (1990)): a rule-generated force field.
Every valence term is generated from per-type generators and global constants: bonds
``1/2 n K1 (R - R0_I - R0_J + 0.01)^2`` (or Morse), harmonic-cosine angles with ``theta0`` of the
centre (``K (1 + cos)`` at linear centres), torsions ``1/2 V {1 - cos[n(phi - phi0)]}`` whose
``(V, n, phi0)`` follow from the central atoms' hybridisations and bond order (rules a-j; the
barrier of a bond split over its dihedrals), umbrella inversions at listed planar centres (three
axis choices, 1/3 each), 12-6 ``D0 [rho^-12 - 2 rho^-6]`` or exponential-6 van der Waals, Coulomb
with 332.0637, and the explicit 12-10 hydrogen bond on ``H__HB`` donor triplets.

The generators' library (``dreiding``, ``dreiding/X6`` in ``dreiding.frc``), the rule table and
engine, the trainable generator groups and the outputs follow the reference
(``src/xnn/ffnn/models/dreidinglib.py``, ``dreiding.py``).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence, Union

import torch
from torch import Tensor, nn
from torch.nn import Parameter, ParameterDict

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS
from ..models.fast import resolve_use_fast
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .frc import read_forcefield
from .geometry import TINY, batch_index, dihedral_cos, geometric_mean, pair_vectors, quintic_switch
from .opls import DEG, KCAL_TO_EV, FixedTopologyPotential, _groups, _listy
from .topology import MolecularTopology, read_topology

KE = 332.0637 * KCAL_TO_EV
DELTA, BOND_K1, BOND_D1, ANGLE_K = 0.01, 700.0, 70.0, 100.0
HBOND_D0, HBOND_R0 = 9.0, 2.75
# rule -> (barrier per bond [kcal/mol], periodicity, phi0 [deg]); rule g (sp1, monovalent or metal
# centre) has no term
TORSION_RULES = {"a": (2.0, 3, 180.0), "b": (1.0, 6, 0.0), "c": (45.0, 2, 180.0), "d": (25.0, 2, 180.0),
                 "e": (5.0, 2, 180.0), "f": (10.0, 2, 180.0), "h": (2.0, 2, 90.0), "i": (2.0, 2, 180.0),
                 "j": (2.0, 3, 180.0)}
RULE_IDS = tuple(TORSION_RULES)
OXYGEN_COLUMN = frozenset({"O", "S", "Se", "Te", "Po"})
HB_ACCEPTOR_ELEMENTS = frozenset({"N", "O", "F"})
HB_DONOR_TYPES = frozenset({"H__HB"})
GROUPS = ("radius", "theta0", "bond_k", "bond_d", "angle_k", "torsion_v", "oop_k", "oop_psi0", "vdw_r0", "vdw_d0",
          "x6_zeta", "hbond_d0", "hbond_r0")


def hybridization(type_name: str) -> str:
    """``1``/``2``/``3``/``R`` from the third character of the label, ``0`` for none."""
    return type_name[2] if len(type_name) > 2 and type_name[2] in "123R" else "0"


def element_of(type_name: str) -> str:
    two, one = type_name[:2], type_name[:1]
    return two if two in ATOMIC_NUMBERS else (one if one in ATOMIC_NUMBERS else "")


@dataclass
class DreidingLibrary:
    """Generators in the paper's units (kcal/mol, Å, degrees)."""
    atom_types: dict = field(default_factory=dict)
    radius: dict = field(default_factory=dict)
    theta0: dict = field(default_factory=dict)
    vdw_r0: dict = field(default_factory=dict)
    vdw_d0: dict = field(default_factory=dict)
    x6_zeta: dict = field(default_factory=dict)
    oop: dict = field(default_factory=dict)
    form: str = "lj"
    combination: str = "arithmetic"
    delta: float = DELTA
    bond_k1: float = BOND_K1
    bond_d1: float = BOND_D1
    angle_k: float = ANGLE_K
    torsion_v: dict = field(default_factory=lambda: {r: v for r, (v, _, _) in TORSION_RULES.items()})
    hbond_d0: float = HBOND_D0
    hbond_r0: float = HBOND_R0
    hb_donor_types: set = field(default_factory=lambda: set(HB_DONOR_TYPES))
    templates: dict = field(default_factory=dict)
    fragments: dict = field(default_factory=dict)
    name: str = "dreiding"

    def hybrid(self, t: str) -> str:
        return hybridization(t)

    def element(self, t: str) -> str:
        e = self.atom_types.get(t)
        return str(e["element"]) if e and e.get("element") else element_of(t)

    def oxygen_column(self, t: str) -> bool:
        return self.element(t) in OXYGEN_COLUMN

    def is_acceptor(self, t: str) -> bool:
        return self.element(t) in HB_ACCEPTOR_ELEMENTS

    def save(self, path: Union[str, Path]) -> Path:
        data = {"format": "xnn-dreiding-1", **{k: getattr(self, k) for k in (
            "name", "form", "combination", "delta", "bond_k1", "bond_d1", "angle_k", "torsion_v", "hbond_d0",
            "hbond_r0", "atom_types", "radius", "theta0", "vdw_r0", "vdw_d0", "x6_zeta", "templates", "fragments")},
            "hb_donor_types": sorted(self.hb_donor_types), "oop": {k: list(v) for k, v in self.oop.items()}}
        Path(path).write_text(json.dumps(data, indent=2) + "\n")
        return Path(path)


def torsion_rule(lib: DreidingLibrary, ti: str, tj: str, tk: str, tl: str, order: float = 1.0) -> Optional[str]:
    """The rule of dihedral ``I-J-K-L`` (``order`` of the ``J-K`` bond), ``None`` for rule g."""
    hj, hk = lib.hybrid(tj), lib.hybrid(tk)
    if hj in ("0", "1") or hk in ("0", "1"):
        return None
    sp2 = ("2", "R")
    if hj in sp2 and hk in sp2:
        if order >= 1.75:
            return "c"
        if abs(order - 1.5) < 0.25:
            return "d"
        return "f" if hj == "R" and hk == "R" else "e"
    if hj == "3" and hk == "3":
        return "h" if lib.oxygen_column(tj) and lib.oxygen_column(tk) else "a"
    t2, t3, outer = (tj, tk, ti) if hj in sp2 else (tk, tj, tl)
    if lib.oxygen_column(t3) and not lib.oxygen_column(t2):
        return "i"
    return "b" if lib.hybrid(outer) in sp2 else "j"


def read_dreiding(spec: Union[str, Path] = "dreiding") -> DreidingLibrary:
    """A library from ``"dreiding"``, ``"dreiding/X6"``, a ``.frc`` path or a native JSON."""
    p = Path(str(spec))
    if p.suffix.lower() == ".json" and p.is_file():
        d = json.loads(p.read_text())
        lib = DreidingLibrary()
        for k, v in d.items():
            if k == "oop":
                v = {c: tuple(x) for c, x in v.items()}
            elif k == "hb_donor_types":
                v = set(v)
            if k != "format":
                setattr(lib, k, v)
        return lib
    ff = read_forcefield(str(spec))
    if ff.ff_form != "dreiding":
        raise ValueError(f"force field {ff.name!r} has ff_form {ff.ff_form!r}, not 'dreiding'")
    lib = DreidingLibrary(name=ff.name, templates=dict(ff.templates), fragments=dict(ff.fragments))

    def ensure(t):
        lib.atom_types.setdefault(t, {"element": element_of(t), "mass": 0.0, "connections": 0, "comment": ""})
    for key, row in ff.rows("atom_types").items():
        v = row.values
        lib.atom_types[key[0]] = {"element": str(v.get("El", "")) or element_of(key[0]), "mass": float(v.get("Mass", 0.0)),
                                  "connections": int(v.get("connections", 0)), "comment": str(v.get("Comment", ""))}
    for key, row in ff.rows("dreiding_atomic_parameters").items():
        ensure(key[0])
        lib.radius[key[0]], lib.theta0[key[0]] = float(row.values["Radius"]), float(row.values["Theta0"])
    if "buckingham" in ff.sections:
        lib.form = "x6"
        for key, row in ff.rows("buckingham").items():
            ensure(key[0])
            lib.vdw_r0[key[0]], lib.vdw_d0[key[0]] = float(row.values["rho"]), float(row.values["eps"])
            lib.x6_zeta[key[0]] = float(row.values["S"])
    else:
        lib.form, lib.combination = "lj", ff.combination("nonbond(12-6)")
        for key, row in ff.rows("nonbond(12-6)").items():
            ensure(key[0])
            lib.vdw_r0[key[0]] = float(row.values["sigma"]) * 2.0 ** (1.0 / 6.0)
            lib.vdw_d0[key[0]] = float(row.values["eps"])
    for key, row in ff.rows("dreiding_out_of_plane").items():
        ensure(key[1])
        lib.oop[key[1]] = (float(row.values["K2"]), float(row.values["Psi0"]))
    return lib


class DreidingForceField(nn.Module):
    """The trainable generators (eV, Å, rad): per-type ``radius``, ``theta0``, ``oop_k``,
    ``oop_psi0``, ``vdw_r0``, ``vdw_d0``, ``x6_zeta``; global ``bond_k``, ``bond_d``, ``angle_k``,
    ``torsion_v`` (per rule), ``hbond_d0``, ``hbond_r0``."""

    def __init__(self, library: Union[DreidingLibrary, str, Path] = "dreiding", trainable=()):
        super().__init__()
        lib = library if isinstance(library, DreidingLibrary) else read_dreiding(library)
        dt = torch.get_default_dtype()
        train = _groups(trainable, GROUPS)
        self.lib, self.name, self.form, self.combination = lib, lib.name, lib.form, str(lib.combination)
        self.delta = float(lib.delta)
        self.templates, self.fragments = dict(lib.templates), dict(lib.fragments)
        self.type_names = list(lib.atom_types)
        self._type_index = {n: i for i, n in enumerate(self.type_names)}
        self.hybrids = [lib.hybrid(n) for n in self.type_names]
        self.register_buffer("type_z", torch.tensor([ATOMIC_NUMBERS.get(lib.element(n), 0) for n in self.type_names],
                                                    dtype=torch.long))
        self.register_buffer("type_mass", torch.tensor([float(lib.atom_types[n].get("mass", 0.0))
                                                        for n in self.type_names], dtype=dt))
        self.register_buffer("type_acceptor", torch.tensor([lib.is_acceptor(n) for n in self.type_names]))
        self.donor_types = {n for n in self.type_names if n in lib.hb_donor_types}
        self._has_radius = {n for n in self.type_names if n in lib.radius}
        self._has_vdw = {n for n in self.type_names if n in lib.vdw_r0}
        self.oop_types = set(lib.oop)
        self.params = ParameterDict()

        def per_type(table, default, scale=1.0):
            return [float(table.get(n, default)) * scale for n in self.type_names]

        def make(name, vals):
            self.params[name] = Parameter(torch.tensor(vals, dtype=dt), requires_grad=name in train)
        make("radius", per_type(lib.radius, 0.0))
        make("theta0", per_type(lib.theta0, 180.0, DEG))
        make("bond_k", float(lib.bond_k1) * KCAL_TO_EV)
        make("bond_d", float(lib.bond_d1) * KCAL_TO_EV)
        make("angle_k", float(lib.angle_k) * KCAL_TO_EV)
        make("torsion_v", [float(lib.torsion_v.get(r, TORSION_RULES[r][0])) * KCAL_TO_EV for r in RULE_IDS])
        make("oop_k", [float(lib.oop.get(n, (0.0, 0.0))[0]) * KCAL_TO_EV for n in self.type_names])
        make("oop_psi0", [float(lib.oop.get(n, (0.0, 0.0))[1]) * DEG for n in self.type_names])
        make("vdw_r0", per_type(lib.vdw_r0, 0.0))
        make("vdw_d0", per_type(lib.vdw_d0, 0.0, KCAL_TO_EV))
        make("x6_zeta", per_type(lib.x6_zeta, 12.0))
        make("hbond_d0", float(lib.hbond_d0) * KCAL_TO_EV)
        make("hbond_r0", float(lib.hbond_r0))
        # 1/2 V {1 - cos[n (phi - phi0)]} = 1/2 V {1 - s cos(n phi)}, s = cos(n phi0) = +-1
        signs = [math.cos(n * p0 * DEG) for _, n, p0 in TORSION_RULES.values()]
        if any(abs(abs(s) - 1.0) > 1e-9 for s in signs):
            raise ValueError("every torsion rule needs n phi0 a multiple of 180 degrees")
        self.register_buffer("rule_n", torch.tensor([n for _, n, _ in TORSION_RULES.values()], dtype=torch.long))
        self.register_buffer("rule_sign", torch.tensor([round(s) for s in signs], dtype=dt))

    def type_index(self, name: str) -> int:
        if name not in self._type_index:
            raise KeyError(f"atom type {name!r} is not in library {self.name!r}")
        return self._type_index[name]

    def check_generators(self, name: str) -> None:
        if name not in self._has_radius:
            raise KeyError(f"atom type {name!r} has no bond radius / angle in library {self.name!r}")
        if name not in self._has_vdw:
            raise KeyError(f"atom type {name!r} has no van der Waals parameters in library {self.name!r}")


@register_model("dreiding")
class Dreiding(FixedTopologyPotential):
    """DREIDING bound to one topology (with bond orders). Outputs ``e_bond``, ``e_angle``,
    ``e_torsion``, ``e_inversion``, ``e_vdw``, ``e_coulomb``, ``e_hbond``."""

    def __init__(self, ffield="dreiding", topology=None, *, cutoff: float = 10.0, switch_width: float = 0.0,
                 charges: Optional[Sequence[float]] = None, bond_style: str = "harmonic", angle_style: str = "cosine",
                 hbond: bool = True, hbond_cutoff: Optional[float] = None, hbond_angle: float = 90.0, trainable=(),
                 keep_intermediates: bool = False, use_fast="auto"):
        super().__init__()
        if topology is None:
            raise ValueError("Dreiding needs a topology (a MolecularTopology or a topology JSON path)")
        groups = set(GROUPS) | {"charge"} if isinstance(trainable, str) and trainable.lower() == "all" else \
            ({trainable} if isinstance(trainable, str) else set(trainable))
        self._train_charge = "charge" in groups
        self.ff = ffield if isinstance(ffield, DreidingForceField) else DreidingForceField(ffield, groups - {"charge"})
        if bond_style not in ("harmonic", "morse"):
            raise ValueError(f"bond_style must be 'harmonic' or 'morse', got {bond_style!r}")
        if angle_style not in ("cosine", "harmonic"):
            raise ValueError(f"angle_style must be 'cosine' or 'harmonic', got {angle_style!r}")
        self.bond_style, self.angle_style = bond_style, angle_style
        self.cutoff, self.switch_width = float(cutoff), float(switch_width)
        if not 0.0 <= self.switch_width < self.cutoff:
            raise ValueError("switch_width must satisfy 0 <= switch_width < cutoff")
        self.use_hbond = bool(hbond)
        self.hbond_cutoff = self.cutoff if hbond_cutoff is None else float(hbond_cutoff)
        if self.hbond_cutoff > self.cutoff + 1e-9:
            raise ValueError("hbond_cutoff must not exceed cutoff: the hydrogen bonds come from the neighbor list")
        self.hbond_cos = math.cos(float(hbond_angle) * DEG)
        self.keep_intermediates, self.intermediates = bool(keep_intermediates), {}
        self.node_feature_dim = 1
        self.use_fast = resolve_use_fast(use_fast)
        self._bind(topology if isinstance(topology, MolecularTopology) else read_topology(topology), charges)
        self.species = sorted({int(z) for z in self.top_z.tolist()})

    def _bind(self, top: MolecularTopology, charges) -> None:
        self.topology, ff, lib = top, self.ff, self.ff.lib
        n, dt = top.n_atoms, torch.get_default_dtype()
        missing = []
        for name in dict.fromkeys(top.types):
            try:
                ff.type_index(name)
                ff.check_generators(name)
            except KeyError as err:
                missing.append(str(err.args[0]))
        if missing:
            raise KeyError("the topology needs parameters the library does not provide:\n  " + "\n  ".join(missing))
        t = [ff.type_index(nm) for nm in top.types]
        orders = list(top.bond_orders) or [1.0] * len(top.bonds)
        self._buf("top_type", t, 1)
        self.register_buffer("top_z", ff.type_z[self.top_type].clone())
        self._buf("bond_index", top.bonds, 2)
        self.register_buffer("bond_order", torch.tensor(orders, dtype=dt).reshape(-1))
        self._buf("angle_index", top.angles, 3)
        self.register_buffer("angle_linear", torch.tensor(
            [abs(lib.theta0.get(top.types[j], 180.0) - 180.0) < 1e-8 for _, j, _ in top.angles], dtype=torch.bool))
        shared: dict = {}
        for _, j, k, _ in top.dihedrals:
            shared[(min(j, k), max(j, k))] = shared.get((min(j, k), max(j, k)), 0) + 1
        order_of = dict(zip(top.bonds, orders))
        rid = {r: m for m, r in enumerate(RULE_IDS)}
        d_idx, d_rule, d_w = [], [], []
        for i, j, k, l in top.dihedrals:
            key = (min(j, k), max(j, k))
            rule = torsion_rule(lib, top.types[i], top.types[j], top.types[k], top.types[l], order_of.get(key, 1.0))
            if rule is not None:
                d_idx.append((i, j, k, l))
                d_rule.append(rid[rule])
                d_w.append(1.0 / shared[key])
        self._buf("dihedral_index", d_idx, 4)
        self._buf("dihedral_rule", d_rule, 1)
        self.register_buffer("dihedral_weight", torch.tensor(d_w, dtype=dt).reshape(-1))
        nbr: dict = {}
        for i, j in top.bonds:
            nbr.setdefault(i, []).append(j)
            nbr.setdefault(j, []).append(i)
        inv = []
        for m, nb in sorted(nbr.items()):
            if len(nb) == 3 and top.types[m] in ff.oop_types:
                a, b, c = sorted(nb)
                inv += [(m, a, b, c), (m, b, c, a), (m, c, a, b)]
        self._buf("inversion_index", inv, 4)
        self._buf("excl_index", top.exclusions, 2)
        hyd: dict = {}
        for h in (i for i, nm in enumerate(top.types) if nm in ff.donor_types):
            if len(nbr.get(h, [])) != 1:
                raise ValueError(f"hydrogen-bond donor atom {h} ({top.types[h]}) must have exactly one bond, "
                                 f"found {len(nbr.get(h, []))}")
            hyd.setdefault(nbr[h][0], []).append(h)
        width = max((len(v) for v in hyd.values()), default=0)
        table = [[-1] * width for _ in range(n)]
        for d, hs in hyd.items():
            table[d][:len(hs)] = hs
        self.register_buffer("hbond_hydrogens", torch.tensor(table, dtype=torch.long).reshape(n, width),
                             persistent=False)
        self.register_buffer("hbond_acceptor", torch.tensor([bool(ff.type_acceptor[i]) for i in t],
                                                            dtype=torch.bool).reshape(n), persistent=False)
        q = torch.zeros(n, dtype=dt) if charges is None else torch.as_tensor([float(c) for c in charges], dtype=dt)
        if q.numel() != n:
            raise ValueError(f"got {q.numel()} charges for {n} atoms")
        self.has_coulomb = bool(q.abs().sum() > 0.0) or self._train_charge
        if self._train_charge:
            self.charge = Parameter(q)
        else:
            self.register_buffer("charge", q)

    @property
    def graph_capturable(self) -> bool:
        # the hydrogen-bond triplets are selected from the list by their distances (data-dependent shapes)
        return not (self.use_hbond and self.hbond_hydrogens.shape[1] > 0)

    def forward(self, data: AtomicGraph) -> dict:
        N, B, n = self._check_batch(data)
        P, ff = self.ff.params, self.ff
        t = self.top_type.repeat(B)
        q = self.charge.repeat(B)
        bi, ai = batch_index(self.bond_index, n, B), batch_index(self.angle_index, n, B)
        di, ii = batch_index(self.dihedral_index, n, B), batch_index(self.inversion_index, n, B)
        # bonds
        bo = self.bond_order.repeat(B)
        bv = pair_vectors(data, bi[0], bi[1])
        br = torch.sqrt((bv * bv).sum(1) + TINY)
        r0 = P["radius"][t[bi[0]]] + P["radius"][t[bi[1]]] - ff.delta
        k_n = bo * P["bond_k"]
        if self.bond_style == "morse":
            d_n = bo * P["bond_d"]
            e_bond = d_n * (torch.exp(-torch.sqrt(k_n / (2.0 * d_n + TINY)) * (br - r0)) - 1.0) ** 2
        else:
            e_bond = 0.5 * k_n * (br - r0) ** 2
        e_bond_node = scatter_sum(0.5 * e_bond, bi[0], N) + scatter_sum(0.5 * e_bond, bi[1], N)
        # angles
        u, v = pair_vectors(data, ai[1], ai[0]), pair_vectors(data, ai[1], ai[2])
        cos_th = (u * v).sum(1) / torch.sqrt((u * u).sum(1) * (v * v).sum(1) + TINY)
        th0, ka = P["theta0"][t[ai[1]]], P["angle_k"]
        if self.angle_style == "harmonic":
            bound = min(0.9999999999, 1.0 - 4.0 * torch.finfo(cos_th.dtype).eps)
            e_bent = 0.5 * ka * (torch.arccos(torch.clamp(cos_th, -bound, bound)) - th0) ** 2
        else:
            e_bent = 0.5 * (ka / torch.clamp(torch.sin(th0) ** 2, min=TINY)) * (cos_th - torch.cos(th0)) ** 2
        e_angle = torch.where(self.angle_linear.repeat(B), ka * (1.0 + cos_th), e_bent)
        e_angle_node = scatter_sum(e_angle, ai[1], N)
        # torsions: cos(n phi) for n = 2, 3, 6 by Chebyshev
        dr = self.dihedral_rule.repeat(B)
        c1 = dihedral_cos(data, di)
        t2, t3 = 2.0 * c1 * c1 - 1.0, c1 * (4.0 * c1 * c1 - 3.0)
        nd = ff.rule_n[dr]
        tn = torch.where(nd == 2, t2, torch.where(nd == 3, t3, 2.0 * t3 * t3 - 1.0))
        e_tors = self.dihedral_weight.repeat(B) * 0.5 * P["torsion_v"][dr] * (1.0 - ff.rule_sign[dr] * tn)
        e_tors_node = scatter_sum(e_tors, di[1], N)
        # inversions: angle of bond I-L with the plane I-J-K
        it = t[ii[0]]
        nrm = torch.cross(pair_vectors(data, ii[0], ii[1]), pair_vectors(data, ii[0], ii[2]), dim=1)
        nrm = nrm / torch.sqrt((nrm * nrm).sum(1, keepdim=True) + TINY)
        ril = pair_vectors(data, ii[0], ii[3])
        sin_psi = (nrm * ril / torch.sqrt((ril * ril).sum(1, keepdim=True) + TINY)).sum(1)
        cos_psi = torch.sqrt(torch.clamp(1.0 - sin_psi * sin_psi, min=TINY))
        k_i, psi0 = P["oop_k"][it], P["oop_psi0"][it]
        e_inv = torch.where(psi0.abs() < 1e-8, k_i * (1.0 - cos_psi),
                            0.5 * k_i / torch.clamp(torch.sin(psi0) ** 2, min=TINY) * (cos_psi - torch.cos(psi0)) ** 2) / 3.0
        e_inv_node = scatter_sum(e_inv, ii[0], N)
        # nonbonded (1-2, 1-3 excluded; 1-4 in full)
        src, dst, vec, r2, half, keep = self._pairs_once(data, self.excl_index, n)
        r = torch.sqrt(r2 + TINY)
        r0_t, d0_t = P["vdw_r0"][t], P["vdw_d0"][t]
        d0 = geometric_mean(d0_t[src], d0_t[dst])
        if ff.form == "x6":
            z_t = torch.clamp(P["x6_zeta"][t], min=6.0 + 1e-6)
            a_t = d0_t * (6.0 / (z_t - 6.0)) * torch.exp(z_t)
            b_t = d0_t * (z_t / (z_t - 6.0)) * torch.clamp(r0_t, min=TINY) ** 6
            c_t = z_t / torch.clamp(r0_t, min=TINY)
            vdw = (geometric_mean(a_t[src], a_t[dst]) * torch.exp(-0.5 * (c_t[src] + c_t[dst]) * r)
                   - geometric_mean(b_t[src], b_t[dst]) / (r2 ** 3 + TINY))
        else:
            r0_ij = geometric_mean(r0_t[src], r0_t[dst]) if ff.combination == "geometric" else 0.5 * (r0_t[src] + r0_t[dst])
            s6 = (r0_ij * r0_ij / (r2 + TINY)) ** 3
            vdw = d0 * (s6 * s6 - 2.0 * s6)
        coul = KE * q[src] * q[dst] / r if self.has_coulomb else torch.zeros_like(r)
        w = keep.to(r.dtype) * half * quintic_switch(r, self.cutoff, self.switch_width)
        hv, hc = 0.5 * w * vdw, 0.5 * w * coul
        e_vdw_node = scatter_sum(hv, src, N) + scatter_sum(hv, dst, N)
        e_c_node = scatter_sum(hc, src, N) + scatter_sum(hc, dst, N)
        # hydrogen bonds over the list's donor-acceptor pairs (either direction), once per donor H
        e_hb_node = torch.zeros_like(e_vdw_node)
        if self.use_hbond and self.hbond_hydrogens.shape[1] > 0:
            K = int(self.hbond_hydrogens.shape[1])
            starts = torch.arange(B, device=t.device) * n
            hyd = self.hbond_hydrogens.repeat(B, 1)
            hyd = torch.where(hyd >= 0, hyd + starts.repeat_interleave(n)[:, None], hyd)
            acc = self.hbond_acceptor.repeat(B)
            near = keep & (r.detach() < self.hbond_cutoff)
            fwd = ((hyd[src, 0] >= 0) & acc[dst] & near).nonzero()[:, 0]
            rev = ((hyd[dst, 0] >= 0) & acc[src] & near & (src != dst)).nonzero()[:, 0]
            donor, accept = torch.cat([src[fwd], dst[rev]]), torch.cat([dst[fwd], src[rev]])
            h_all = hyd[donor].reshape(-1)
            ok = h_all >= 0
            e_da = torch.arange(donor.shape[0], device=t.device).repeat_interleave(K)[ok]
            h = h_all[ok]
            vec_da = torch.cat([vec[fwd], -vec[rev]])[e_da]
            r_da = torch.cat([r[fwd], r[rev]])[e_da]
            v_hd = pair_vectors(data, h, donor[e_da])
            v_ha = v_hd + vec_da
            cos_dha = (v_hd * v_ha).sum(1) / torch.sqrt((v_hd * v_hd).sum(1) * (v_ha * v_ha).sum(1) + TINY)
            rho2 = (P["hbond_r0"] / r_da) ** 2
            rho10 = rho2 ** 5
            e_hb = P["hbond_d0"] * (5.0 * rho10 * rho2 - 6.0 * rho10) * cos_dha ** 4
            e_hb = e_hb * ((r_da < self.hbond_cutoff) & (cos_dha < self.hbond_cos)).to(e_hb.dtype)
            e_hb_node = scatter_sum(e_hb, h, N)
        node = e_bond_node + e_angle_node + e_tors_node + e_inv_node + e_vdw_node + e_c_node + e_hb_node
        if self.keep_intermediates:
            self.intermediates = dict(bond_r=br, bond_r0=r0, e_bond=e_bond, angle_cos=cos_th, e_angle=e_angle,
                                      dihedral_cos=c1, e_torsion=e_tors, inversion_sin=sin_psi, e_inversion=e_inv)
        agg = lambda x: self.aggregate_energy(x, data)  # noqa: E731
        return {"node_energy": node, "energy": agg(node), "charges": q, "node_features": q.unsqueeze(1),
                "e_bond": agg(e_bond_node), "e_angle": agg(e_angle_node), "e_torsion": agg(e_tors_node),
                "e_inversion": agg(e_inv_node), "e_vdw": agg(e_vdw_node), "e_coulomb": agg(e_c_node),
                "e_hbond": agg(e_hb_node)}

    @classmethod
    def from_config(cls, cfg) -> "Dreiding":
        e = dict(cfg.extra or {})
        if e.get("topology") is not None:
            top = read_topology(e["topology"])
        else:
            types, bonds = _listy(e.get("types")), _listy(e.get("bonds"))
            if types is None or bonds is None:
                raise ValueError("Dreiding needs a topology: set model.topology to a topology JSON path, or give "
                                 "model.types and model.bonds inline")
            top = MolecularTopology.from_bonds(types, bonds, bond_orders=_listy(e.get("bond_orders")))
        kw = {k: str(e[k]) for k in ("bond_style", "angle_style") if e.get(k) is not None}
        kw.update({k: float(e[k]) for k in ("hbond_cutoff", "hbond_angle") if e.get(k) is not None})
        if e.get("hbond") is not None:
            kw["hbond"] = bool(e["hbond"])
        return cls(e.get("ffield") or "dreiding", top, cutoff=float(cfg.cutoff),
                   switch_width=float(e.get("switch_width") or 0.0), charges=_listy(e.get("charges")),
                   trainable=_listy(e.get("trainable")) or (), **kw)
