"""The AMOEBA polarizable multipole force field bound to a molecular topology.

Energy terms (Ponder et al., J. Phys. Chem. B 114, 2549 (2010); Ren and Ponder 2003 for water),
each in eV per structure:

* ``e_bond``: ``K dr^2 (1 + c3 dr + c4 dr^2)``; ``e_angle``: ``K dt^2 (1 + c3 dt + ... + c6 dt^4)``
  with ``dt`` in degrees (in-plane angles at three-connected centres for ``anglep`` entries);
  ``e_strbnd``: ``(k1 dr1 + k2 dr2) dt``; ``e_urey``: ``K (s - s0)^2`` on the 1-3 distance;
  ``e_opbend``: Allinger out-of-plane angles, same sextic series; ``e_torsion``: ``sum_n V_n (1 +
  cos(n phi - delta_n))`` times the torsion unit;
* ``e_vdw``: Halgren's buffered 14-7 between the reduced sites (hydrogens moved towards their
  parent), cubic-mean radii and HHG depths, scaled by bond separation;
* ``e_multipole``: permanent charges, dipoles and quadrupoles given in local frames (z-then-x,
  bisector, z-bisect, 3-fold, z-only, with Tinker's chirality rule for a fourth frame atom), scaled
  by bond separation;
* ``e_polar``: mutual induction with Thole damping. With the direct-field scales ``d`` (by
  polarization group) and the energy-field scales ``p`` (by bond separation) the induced dipoles
  ``mu_d = A^-1 E_d`` and ``mu_p = A^-1 E_p`` (``A = alpha^-1 - T``, ``T`` scaled by the mutual
  factors) give ``E_pol = -1/2 mu_d . E_p``; the forces differentiate the stationary function
  ``L = -1/2 mu_p.E_d - 1/2 mu_d.E_p + 1/2 mu_p.A mu_d`` at fixed dipoles, so no derivative of
  the solve is needed (frame torques follow from the moments' dependence on the positions).

Molecules (no cell) sum every pair directly. Periodic water boxes (every intramolecular pair a 1-2
or 1-3 pair, one polarization group per molecule) take the smooth-PME electrostatics of
:class:`~xnn_b200.ffnn.multipoles.PolarizableMultipoles` with intramolecular mutual induction and
a cutoff on the van der Waals term (Tinker's quintic switch over its last 10 %).

Parity: the reference's ``Amoeba`` (``src/xnn/ffnn/models/amoeba.py:2107``); HIPPO, charge flux,
pi-torsions and torsion-torsion grids are not built here.
"""
from __future__ import annotations

import math
from collections import deque
from typing import Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .amoeba_params import AmoebaParameters, load_parameters
from .geometry import half_edges, quintic_switch
from .multipoles import DEBYE, KE, EwaldSetup, PolarizableMultipoles, pair_energy, thole_damp
from .opls import FixedTopologyPotential
from .topology import MolecularTopology

BOHR = 0.529177210903
KCAL_TO_EV = 1.0 / 23.060547830619
DEG = 180.0 / math.pi
FRAMES = {"none": 0, "z-only": 1, "z-then-x": 2, "bisector": 3, "z-bisect": 4, "3-fold": 5}


# ----------------------------------------------------------------------------- frames
def _unit(v: Tensor) -> Tensor:
    return v / torch.linalg.norm(v, dim=-1, keepdim=True).clamp_min(1e-12)


def local_frames(pos: Tensor, kind: Tensor, zi: Tensor, xi: Tensor, yi: Tensor) -> Tensor:
    """Rotation ``(n, 3, 3)`` whose rows are each atom's local x, y, z axes in the global frame."""
    uz = _unit(pos[zi] - pos)
    ux = _unit(pos[xi] - pos)
    uy = _unit(pos[yi] - pos)
    lab = torch.zeros_like(pos)
    lab[:, 0] = 1.0
    alt = torch.zeros_like(pos)
    alt[:, 1] = 1.0
    k = kind[:, None]
    z = torch.where(k == 3, _unit(uz + ux), torch.where(k == 5, _unit(uz + ux + uy), uz))
    z = torch.where(k == 0, torch.zeros_like(z) + torch.tensor([0.0, 0.0, 1.0], dtype=pos.dtype, device=pos.device), z)
    xref = torch.where(k == 4, _unit(ux + uy), ux)
    zonly = torch.where((uz[:, 0:1].abs() > 0.866), alt, lab)
    xref = torch.where(k == 1, zonly, xref)
    xref = torch.where(k == 0, lab, xref)
    x = _unit(xref - (xref * z).sum(-1, keepdim=True) * z)
    y = torch.cross(z, x, dim=-1)
    return torch.stack([x, y, z], 1)


def rotate_moments(R: Tensor, d: Tensor, Q: Tensor) -> Tuple[Tensor, Tensor]:
    """Local-frame dipoles ``(n, 3)`` and quadrupoles ``(n, 3, 3)`` into the global frame."""
    dg = (d[:, :, None] * R).sum(1)
    Qg = torch.einsum("nai,nab,nbj->nij", R, Q, R)
    return dg, Qg


def chirality_flip(pos: Tensor, i: Tensor, zi: Tensor, xi: Tensor, yi: Tensor, ysign: Tensor) -> Tensor:
    """Tinker's rule for z-then-x frames with a fourth (y) atom: the sign of the volume spanned
    from the x atom to the y atom, the atom and the z atom, against the sign the parameters give
    the y atom; a mismatch mirrors the frame's y axis. ``True`` where the moments flip."""
    a = pos[yi] - pos[xi]
    b = pos[i] - pos[xi]
    c = pos[zi] - pos[xi]
    vol = (a * torch.cross(b, c, dim=-1)).sum(-1)
    return ((vol < 0) & (ysign > 0)) | ((vol > 0) & (ysign < 0))


# ----------------------------------------------------------------------------- the model
def _bfs(n: int, nbr: List[List[int]], src: int, depth: int) -> Dict[int, int]:
    out = {src: 0}
    dq = deque([src])
    while dq:
        a = dq.popleft()
        if out[a] >= depth:
            continue
        for b in nbr[a]:
            if b not in out:
                out[b] = out[a] + 1
                dq.append(b)
    return out


@register_model("amoeba")
class Amoeba(FixedTopologyPotential):
    """AMOEBA on one molecular topology (types are Tinker atom types, as integers or strings);
    see the module notes. ``cutoff`` is the neighbour-list (and van der Waals) cutoff of periodic
    boxes; molecules sum every pair."""

    graph_capturable = False

    def __init__(self, ffield="amoeba-water-2003", topology: Optional[MolecularTopology] = None, *,
                 cutoff: float = 9.0, polarization: Optional[str] = None, polar_eps: float = 1e-8,
                 max_iter: int = 200, ewald: Optional[EwaldSetup] = None, atomic_energies=None):
        super().__init__()
        self.params: AmoebaParameters = load_parameters(ffield)
        if topology is None:
            raise ValueError("a topology is required (e.g. Amoeba.water(n_molecules))")
        self.cutoff = float(cutoff)
        mode = (polarization or str(self.params.get("polarization", "MUTUAL"))).lower()
        if mode not in ("mutual", "direct", "none"):
            raise ValueError(f"polarization must be mutual, direct or none, not {mode!r}")
        self.polarization = mode
        self.polar_eps = float(polar_eps)
        self.max_iter = int(max_iter)
        self.ewald = ewald
        self.atom_ref = nn.Embedding(120, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.atom_ref.weight.requires_grad_(False)
        self.node_feature_dim = 1
        self._bind(topology)
        if atomic_energies is not None:
            with torch.no_grad():
                for z, v in dict(atomic_energies).items():
                    self.atom_ref.weight[int(z), 0] = float(v)

    # ------------------------------------------------------------------ construction helpers
    @classmethod
    def water(cls, n_molecules: int = 1, ffield="amoeba-water-2003", **kw) -> "Amoeba":
        """AMOEBA water: molecules as consecutive O, H, H (Tinker types 1, 2, 2)."""
        top = MolecularTopology.from_bonds(["1", "2", "2"], [(0, 1), (0, 2)]).replicate(int(n_molecules))
        return cls(ffield, top, **kw)

    def _buf(self, name: str, rows, width: int, dtype=torch.long) -> None:
        if width > 1:
            t = torch.tensor(rows, dtype=dtype).reshape(-1, width)
            t = t.t().contiguous()
        else:
            t = torch.tensor(rows, dtype=dtype).reshape(-1)
        self.register_buffer(name, t)

    def _fbuf(self, name: str, rows, shape=None) -> None:
        t = torch.tensor(rows, dtype=torch.float64)
        self.register_buffer(name, t.reshape(shape) if shape is not None else t)

    def _bind(self, top: MolecularTopology) -> None:
        P = self.params
        self.topology = top
        n = top.n_atoms
        types = [int(t) for t in top.types]
        missing: List[str] = []
        for t in sorted(set(types)):
            if t not in P.types:
                missing.append(f"atom type {t}")
        if missing:
            raise KeyError("; ".join(missing))
        cls_ = [P.types[t][0] for t in types]
        Z = [P.types[t][2] for t in types]
        self._buf("top_type", types, 1)
        self._buf("top_z", Z, 1)
        nbr: List[List[int]] = [[] for _ in range(n)]
        for i, j in top.bonds:
            nbr[i].append(j)
            nbr[j].append(i)
        self._nbr = nbr

        # bonds
        b_rows, b_par = [], []
        for i, j in top.bonds:
            v = P.bond(cls_[i], cls_[j])
            if v is None:
                missing.append(f"bond {cls_[i]}-{cls_[j]}")
                continue
            b_rows.append((i, j))
            b_par.append(v)
        self._buf("bond_index", b_rows, 2)
        self._fbuf("bond_par", b_par, (-1, 2))
        bond_len = {(min(i, j), max(i, j)): v[1] for (i, j), v in zip(b_rows, b_par)}

        # angles, Urey-Bradley, stretch-bend
        a_rows, a_par, a_inplane, u_rows, u_par, s_rows, s_par = [], [], [], [], [], [], []
        for i, j, k in top.angles:
            v = P.angle(cls_[i], cls_[j], cls_[k])
            if v is None:
                missing.append(f"angle {cls_[i]}-{cls_[j]}-{cls_[k]}")
                continue
            K, th0s, inplane = v
            nh = sum(1 for m in nbr[j] if m not in (i, k) and Z[m] == 1)
            th0 = th0s[min(nh, len(th0s) - 1)]
            third = [m for m in nbr[j] if m not in (i, k)]
            use_ip = inplane and len(nbr[j]) == 3
            a_rows.append((i, j, k, third[0] if use_ip else j))
            a_par.append((K, th0))
            a_inplane.append(1 if use_ip else 0)
            ub = P.urey(cls_[i], cls_[j], cls_[k])
            if ub is not None:
                u_rows.append((i, k))
                u_par.append(ub)
            sb = P.stretch_bend(cls_[i], cls_[j], cls_[k])
            if sb is not None:
                r1 = bond_len.get((min(i, j), max(i, j)))
                r2 = bond_len.get((min(k, j), max(k, j)))
                if r1 is not None and r2 is not None:
                    s_rows.append((i, j, k, len(a_rows) - 1))
                    s_par.append((sb[0], sb[1], r1, r2))
        self._buf("angle_index", a_rows, 4)
        self._fbuf("angle_par", a_par, (-1, 2))
        self._buf("angle_inplane", a_inplane, 1, torch.bool)
        self._buf("urey_index", u_rows, 2)
        self._fbuf("urey_par", u_par, (-1, 2))
        self._buf("strbnd_index", s_rows, 4)
        self._fbuf("strbnd_par", s_par, (-1, 4))

        # out-of-plane bends at three-connected centres (one per bent neighbour)
        o_rows, o_par = [], []
        for b in range(n):
            if len(nbr[b]) != 3:
                continue
            for d in nbr[b]:
                a, c = [m for m in nbr[b] if m != d]
                K = P.out_of_plane(cls_[d], cls_[b], cls_[a], cls_[c])
                if K is not None and K != 0.0:
                    o_rows.append((a, b, c, d))
                    o_par.append(K)
        self._buf("opbend_index", o_rows, 4)
        self._fbuf("opbend_par", o_par)

        # torsions (three Fourier terms, padded)
        t_rows, t_par = [], []
        for i, j, k, l in top.dihedrals:
            v = P.torsion(cls_[i], cls_[j], cls_[k], cls_[l])
            if v is None:
                missing.append(f"torsion {cls_[i]}-{cls_[j]}-{cls_[k]}-{cls_[l]}")
                continue
            row = [0.0] * 9
            for m, (amp, phase, per) in enumerate(v[:3]):
                row[3 * m:3 * m + 3] = [amp, phase, float(per)]
            t_rows.append((i, j, k, l))
            t_par.append(row)
        self._buf("torsion_index", t_rows, 4)
        self._fbuf("torsion_par", t_par, (-1, 9))

        # van der Waals sites
        vd = []
        parent = []
        for a in range(n):
            if cls_[a] not in P.vdw:
                missing.append(f"vdw class {cls_[a]}")
                vd.append((1.0, 0.0, 1.0))
                parent.append(a)
                continue
            R, eps, red = P.vdw[cls_[a]]
            if str(P.get("radiussize", "DIAMETER")).upper() == "RADIUS":
                R = 2.0 * R
            if str(P.get("radiustype", "R-MIN")).upper() == "SIGMA":
                R = R * 2.0 ** (1.0 / 6.0)
            vd.append((R, eps, red))
            parent.append(nbr[a][0] if (red != 1.0 and len(nbr[a]) == 1) else a)
        self._fbuf("vdw_par", vd, (-1, 3))
        self._buf("vdw_parent", parent, 1)

        # multipoles and their frames
        kinds, fz, fx, fy, ysg, q, dl, Ql = [], [], [], [], [], [], [], []
        for a in range(n):
            found = self._frame_of(a, types, nbr)
            if found is None:
                missing.append(f"multipole frame of atom {a} (type {types[a]})")
                kinds.append(0), fz.append(a), fx.append(a), fy.append(a), ysg.append(0)
                q.append(0.0), dl.append((0.0, 0.0, 0.0)), Ql.append(((0.0,) * 3,) * 3)
                continue
            m, (za, xa, ya) = found
            kinds.append(FRAMES[m.frame])
            fz.append(za), fx.append(xa), fy.append(ya)
            ysg.append(0 if (m.frame != "z-then-x" or m.y == 0) else (1 if m.y > 0 else -1))
            q.append(m.q)
            dl.append(tuple(c * BOHR for c in m.d))
            Ql.append(tuple(tuple(c * BOHR * BOHR for c in row) for row in m.Q))
        self._buf("frame_kind", kinds, 1)
        self._buf("frame_z", fz, 1)
        self._buf("frame_x", fx, 1)
        self._buf("frame_y", fy, 1)
        self._buf("frame_ysign", ysg, 1)
        self._fbuf("mp_q", q)
        self._fbuf("mp_d", dl, (-1, 3))
        self._fbuf("mp_Q", Ql, (-1, 3, 3))

        # polarizabilities and polarization groups
        alpha, thole = [], []
        for a in range(n):
            v = P.polarize.get(types[a])
            alpha.append(v[0] if v else 0.0)
            thole.append(v[1] if v else 0.0)
        self._fbuf("pol_alpha", alpha)
        self._fbuf("pol_thole", thole)
        group = list(range(n))

        def find(a):
            while group[a] != a:
                group[a] = group[group[a]]
                a = group[a]
            return a
        for i, j in top.bonds:
            gi = P.polarize.get(types[i], (0, 0, ()))[2]
            gj = P.polarize.get(types[j], (0, 0, ()))[2]
            if types[j] in gi or types[i] in gj:
                group[find(i)] = find(j)
        groups = [find(a) for a in range(n)]
        self._groups = groups
        if missing:
            raise KeyError("the topology needs parameters the set does not provide: " + "; ".join(sorted(set(missing))))
        self._scaled_pairs(n, nbr, groups)

    def _frame_of(self, a: int, types: List[int], nbr: List[List[int]]):
        """The first multipole entry of atom ``a``'s type whose frame atoms exist: z among the
        bonded atoms, x and y among the bonded atoms, then among the atoms two bonds away."""
        defs = self.params.multipoles.get(types[a], [])
        for m in defs:
            if m.z == 0:
                return m, (a, a, a)
            zc = [b for b in nbr[a] if types[b] == abs(m.z)]
            for za in zc:
                if m.x == 0:
                    return m, (za, a, a)
                near = [b for b in nbr[a] if b != za] + [c for b in nbr[a] for c in nbr[b] if c not in (a, za)]
                xc = [b for b in near if types[b] == abs(m.x)]
                for xa in xc:
                    if m.y == 0:
                        return m, (za, xa, a)
                    yc = [b for b in near if types[b] == abs(m.y) and b != xa]
                    if yc:
                        return m, (za, xa, yc[0])
        return None

    def _scaled_pairs(self, n: int, nbr: List[List[int]], groups: List[int]) -> None:
        """Pairs within four bonds (or sharing / neighbouring polarization groups) with their
        scale factors: van der Waals, permanent multipoles, the energy field (p), the direct
        field (d) and the mutual coupling (u)."""
        P = self.params
        gid = {g: k for k, g in enumerate(sorted(set(groups)))}
        G = [gid[g] for g in groups]
        gnbr: List[set] = [set() for _ in gid]
        for i, j in self.topology.bonds:
            if G[i] != G[j]:
                gnbr[G[i]].add(G[j])
                gnbr[G[j]].add(G[i])
        gl = [sorted(s) for s in gnbr]
        gsep_cache: Dict[int, Dict[int, int]] = {}
        rows, fac = [], []
        for i in range(n):
            sep = _bfs(n, nbr, i, 4)
            gs = gsep_cache.setdefault(G[i], _bfs(len(gl), gl, G[i], 3))
            cand = set(k for k in sep if k > i)
            for k in cand:
                s = sep[k] + 1                                  # 2 = 1-2, ..., 5 = 1-5
                g = gs.get(G[k])
                gsep = None if g is None else g + 1             # 1 = same group
                f_v = P.scale("vdw", s) if s <= 5 else 1.0
                f_m = P.scale("mpole", s) if s <= 5 else 1.0
                f_p = P.scale("polar", s) if s <= 5 else 1.0
                if s <= 5 and G[i] == G[k]:
                    intra = P.scalars.get(f"polar-1{s}-intra")
                    if intra is not None:
                        f_p = float(intra)
                f_d = P.group_scale("direct", gsep) if gsep is not None else 1.0
                f_u = P.group_scale("mutual", gsep) if gsep is not None else 1.0
                if (f_v, f_m, f_p, f_d, f_u) != (1.0,) * 5:
                    rows.append((i, k))
                    fac.append((f_v, f_m, f_p, f_d, f_u))
        self._buf("scaled_index", rows, 2)
        self._fbuf("scaled_fac", fac, (-1, 5))
        self.molecule_ids = torch.tensor(self._components(n, nbr))

    @staticmethod
    def _components(n: int, nbr: List[List[int]]) -> List[int]:
        comp = [-1] * n
        c = 0
        for a in range(n):
            if comp[a] >= 0:
                continue
            for b in _bfs(n, nbr, a, n):
                comp[b] = c
            c += 1
        return comp

    # ------------------------------------------------------------------ valence terms (kcal/mol)
    def _valence(self, x: Tensor) -> Dict[str, Tensor]:
        P = self.params
        out = {}
        i, j = self.bond_index
        K, r0 = self.bond_par.to(x.dtype).unbind(-1)
        dr = torch.linalg.norm(x[:, j] - x[:, i], dim=-1) - r0
        c3, c4 = P.get("bond-cubic", 0.0), P.get("bond-quartic", 0.0)
        out["e_bond"] = (K * dr * dr * (1.0 + c3 * dr + c4 * dr * dr)).sum(-1)

        ia, ja, ka, la = self.angle_index
        K, th0 = self.angle_par.to(x.dtype).unbind(-1)
        xj = x[:, ja]
        # in-plane angle: the centre projected onto the plane of its three neighbours
        ip = self.angle_inplane
        if bool(ip.any()):
            a_, c_, d_ = x[:, ia], x[:, ka], x[:, la]
            nrm = torch.cross(a_ - d_, c_ - d_, dim=-1)
            nrm = nrm / (nrm * nrm).sum(-1, keepdim=True).clamp_min(1e-24).sqrt()
            proj = xj - ((xj - d_) * nrm).sum(-1, keepdim=True) * nrm
            xj = torch.where(ip[None, :, None], proj, xj)
        u, v = x[:, ia] - xj, x[:, ka] - xj
        cos = (u * v).sum(-1) / (torch.linalg.norm(u, dim=-1) * torch.linalg.norm(v, dim=-1))
        theta = torch.acos(cos.clamp(-1.0 + 1e-15, 1.0 - 1e-15)) * DEG
        dt = theta - th0
        poly = 1.0 + dt * (P.get("angle-cubic", 0.0) + dt * (P.get("angle-quartic", 0.0) + dt * (
            P.get("angle-pentic", 0.0) + dt * P.get("angle-sextic", 0.0))))
        out["e_angle"] = (K * (dt / DEG) ** 2 * poly).sum(-1)

        if self.strbnd_index.shape[1]:
            si, sj, sk, sa = self.strbnd_index
            k1, k2, r1, r2 = self.strbnd_par.to(x.dtype).unbind(-1)
            d1 = torch.linalg.norm(x[:, si] - x[:, sj], dim=-1) - r1
            d2 = torch.linalg.norm(x[:, sk] - x[:, sj], dim=-1) - r2
            out["e_strbnd"] = ((k1 * d1 + k2 * d2) * dt[:, sa] / DEG).sum(-1)
        else:
            out["e_strbnd"] = x.new_zeros(x.shape[0])

        ui, uk = self.urey_index
        K, s0 = self.urey_par.to(x.dtype).unbind(-1)
        ds = torch.linalg.norm(x[:, uk] - x[:, ui], dim=-1) - s0
        out["e_urey"] = (K * ds * ds).sum(-1)

        if self.opbend_index.shape[1]:
            oa, ob, oc, od = self.opbend_index
            K = self.opbend_par.to(x.dtype)
            # Allinger: angle between the b-d bond and the plane a-b-c
            nrm = torch.cross(x[:, oa] - x[:, ob], x[:, oc] - x[:, ob], dim=-1)
            bd = x[:, od] - x[:, ob]
            sin = (nrm * bd).sum(-1) / (torch.linalg.norm(nrm, dim=-1) * torch.linalg.norm(bd, dim=-1)).clamp_min(1e-24)
            chi = torch.asin(sin.clamp(-1.0, 1.0)) * DEG
            poly = 1.0 + chi * (P.get("opbend-cubic", 0.0) + chi * (P.get("opbend-quartic", 0.0) + chi * (
                P.get("opbend-pentic", 0.0) + chi * P.get("opbend-sextic", 0.0))))
            out["e_opbend"] = (K * (chi / DEG) ** 2 * poly).sum(-1)
        else:
            out["e_opbend"] = x.new_zeros(x.shape[0])

        if self.torsion_index.shape[1]:
            ti, tj, tk, tl = self.torsion_index
            b1, b2, b3 = x[:, tj] - x[:, ti], x[:, tk] - x[:, tj], x[:, tl] - x[:, tk]
            n1, n2 = torch.cross(b1, b2, dim=-1), torch.cross(b2, b3, dim=-1)
            m1 = torch.cross(n1, b2 / torch.linalg.norm(b2, dim=-1, keepdim=True), dim=-1)
            phi = torch.atan2((m1 * n2).sum(-1), (n1 * n2).sum(-1))
            par = self.torsion_par.to(x.dtype)
            e = x.new_zeros(phi.shape)
            for m in range(3):
                amp, ph, per = par[:, 3 * m], par[:, 3 * m + 1], par[:, 3 * m + 2]
                e = e + amp * (1.0 + torch.cos(per * phi - ph / DEG))
            out["e_torsion"] = P.get("torsionunit", 1.0) * e.sum(-1)
        else:
            out["e_torsion"] = x.new_zeros(x.shape[0])
        return out

    # ------------------------------------------------------------------ van der Waals
    @staticmethod
    def _buffered_14_7(r: Tensor, R: Tensor, eps: Tensor, delta: float, gamma: float) -> Tensor:
        rho = r / R
        rho7 = rho ** 7
        return eps * ((1.0 + delta) / (rho + delta)) ** 7 * ((1.0 + gamma) / (rho7 + gamma) - 2.0)

    def _vdw_mix(self, a: Tensor, b: Tensor, dtype) -> Tuple[Tensor, Tensor]:
        par = self.vdw_par.to(dtype)
        Ra, ea = par[a, 0], par[a, 1]
        Rb, eb = par[b, 0], par[b, 1]
        rule = str(self.params.get("radiusrule", "CUBIC-MEAN")).upper()
        if rule == "CUBIC-MEAN":
            R = (Ra ** 3 + Rb ** 3) / (Ra ** 2 + Rb ** 2)
        elif rule == "GEOMETRIC":
            R = torch.sqrt(Ra * Rb)
        else:
            R = 0.5 * (Ra + Rb)
        erule = str(self.params.get("epsilonrule", "HHG")).upper()
        if erule == "HHG":
            s = torch.sqrt(ea) + torch.sqrt(eb)
            eps = 4.0 * ea * eb / (s * s).clamp_min(1e-300)
        else:
            eps = torch.sqrt(ea * eb)
        return R, eps

    def _sites(self, x: Tensor) -> Tensor:
        red = self.vdw_par[:, 2].to(x.dtype)
        xp = x[..., self.vdw_parent, :]
        return xp + red[:, None] * (x - xp)

    def _vdw_cluster(self, x: Tensor) -> Tensor:
        n = x.shape[1]
        s = self._sites(x)
        i, k = torch.triu_indices(n, n, 1, device=x.device)
        scale = self._pair_scale(i, k, 0, n, x.dtype)
        keep = scale != 0
        i, k, scale = i[keep], k[keep], scale[keep]
        R, eps = self._vdw_mix(i, k, x.dtype)
        r = torch.linalg.norm(s[:, k] - s[:, i], dim=-1)
        e = self._buffered_14_7(r, R, eps, self.params.get("delta-halgren", 0.07),
                                self.params.get("gamma-halgren", 0.12))
        return (scale * e).sum(-1)

    def _pair_scale(self, i: Tensor, k: Tensor, col: int, n: int, dtype) -> Tensor:
        """Scale factor ``col`` (0 vdw, 1 mpole, 2 p, 3 d, 4 u) of pairs ``i < k`` of one structure."""
        out = torch.ones(i.shape, dtype=dtype, device=i.device)
        if self.scaled_index.shape[1] == 0:
            return out
        key = torch.minimum(i, k) * n + torch.maximum(i, k)
        si, sk = self.scaled_index
        skey = si * n + sk
        order = torch.argsort(skey)
        skey_s = skey[order]
        pos = torch.searchsorted(skey_s, key).clamp(max=skey_s.shape[0] - 1)
        hit = skey_s[pos] == key
        val = self.scaled_fac[order, col].to(dtype)[pos]
        return torch.where(hit, val, out)

    # ------------------------------------------------------------------ multipoles
    def moments(self, x: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
        """Global-frame charges, dipoles (e A) and traceless quadrupoles (e A^2) of one structure."""
        n = x.shape[0]
        ar = torch.arange(n, device=x.device)
        R = local_frames(x, self.frame_kind, self.frame_z, self.frame_x, self.frame_y)
        d = self.mp_d.to(x.dtype)
        Q = self.mp_Q.to(x.dtype)
        flip = (self.frame_ysign != 0) & chirality_flip(x, ar, self.frame_z, self.frame_x, self.frame_y,
                                                        self.frame_ysign)
        if bool(flip.any()):
            sy = torch.where(flip, -1.0, 1.0).to(x.dtype)
            d = torch.stack([d[:, 0], sy * d[:, 1], d[:, 2]], -1)
            m = torch.ones(n, 3, 3, dtype=x.dtype, device=x.device)
            m[:, 0, 1] = m[:, 1, 0] = sy
            m[:, 1, 2] = m[:, 2, 1] = sy
            Q = Q * m
        dg, Qg = rotate_moments(R, d, Q)
        return self.mp_q.to(x.dtype), dg, Qg

    def _pairs_all(self, n: int, device, dtype):
        i, k = torch.triu_indices(n, n, 1, device=device)
        sc = torch.stack([self._pair_scale(i, k, c, n, dtype) for c in range(5)], 0)
        return i, k, sc

    def _electrostatics_cluster(self, x: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
        """``(e_multipole, e_polar, induced dipoles)`` of one molecule or cluster (every pair)."""
        n = x.shape[0]
        q, d, Q = self.moments(x)
        i, k, sc = self._pairs_all(n, x.device, x.dtype)
        v = x[k] - x[i]
        r = torch.linalg.norm(v, dim=-1)
        r2 = r * r
        B = [1.0 / r, 1.0 / (r2 * r), 3.0 / (r2 * r2 * r), 15.0 / (r2 * r2 * r2 * r),
             105.0 / (r2 * r2 * r2 * r2 * r)]
        e_mp = KE * (sc[1] * pair_energy(v, q[i], d[i], Q[i], q[k], d[k], Q[k], B)).sum()
        if self.polarization == "none":
            return e_mp, x.new_zeros(()), x.new_zeros(n, 3)
        alpha = self.pol_alpha.to(x.dtype)
        polar = alpha > 0
        th = torch.minimum(self.pol_thole[i], self.pol_thole[k]).to(x.dtype)
        aa = (alpha[i] * alpha[k]).clamp_min(1e-30) ** (1.0 / 6.0)
        u = r / aa
        Bd = thole_damp(B, r, th * u * u * u)
        zero, z3 = x.new_zeros(i.shape[0]), x.new_zeros(i.shape[0], 3, 3)

        def perm_dipole(mu: Tensor, s: Tensor) -> Tensor:
            """Interaction energy (Coulomb units) of dipoles ``mu`` with the permanent moments."""
            return (s * (pair_energy(v, zero, mu[i], z3, q[k], d[k], Q[k], Bd)
                         + pair_energy(v, q[i], d[i], Q[i], zero, mu[k], z3, Bd))).sum()

        def dip_dip(a: Tensor, b: Tensor) -> Tensor:
            s = sc[4]
            return (s * (pair_energy(v, zero, a[i], z3, zero, b[k], z3, Bd)
                         + pair_energy(v, zero, b[i], z3, zero, a[k], z3, Bd))).sum()

        def fields(s: Tensor) -> Tensor:
            probe = x.new_zeros(n, 3, requires_grad=True)
            with torch.enable_grad():
                w = perm_dipole(probe, s.detach())
                (g,) = torch.autograd.grad(w, probe, create_graph=False)
            return -g

        with torch.no_grad():
            Ed = fields(sc[3]).detach()
            Ep = fields(sc[2]).detach()
        inv_a = torch.where(polar, 1.0 / alpha.clamp_min(1e-30), torch.zeros_like(alpha))
        if self.polarization == "direct":
            mu_d = alpha[:, None] * Ed
            mu_p = alpha[:, None] * Ep
        else:
            with torch.no_grad():
                vv, Bdd = v.detach(), [b.detach() for b in Bd]
                mu_d = self._solve(vv, i, k, sc[4], Bdd, alpha, Ed)
                mu_p = mu_d if torch.equal(sc[2], sc[3]) else self._solve(vv, i, k, sc[4], Bdd, alpha, Ep)
        mu_d, mu_p = mu_d.detach(), mu_p.detach()
        # the stationary function: -1/2 mu_p.E_d - 1/2 mu_d.E_p + 1/2 mu_p.A mu_d (Coulomb units)
        L = 0.5 * perm_dipole(mu_p, sc[3]) + 0.5 * perm_dipole(mu_d, sc[2])
        if self.polarization == "mutual":
            L = L + 0.5 * (inv_a[:, None] * mu_p * mu_d).sum() + 0.5 * dip_dip(mu_p, mu_d)
        else:
            L = L + 0.5 * (inv_a[:, None] * mu_p * mu_d).sum()
        return e_mp, KE * L, mu_d

    def _solve(self, v, i, k, s, Bd, alpha, E) -> Tensor:
        """``(alpha^-1 - T) mu = E`` by Jacobi-preconditioned conjugate gradients (pairwise ``T``)."""
        n = alpha.shape[0]
        b1, b2 = (s * Bd[1])[:, None], (s * Bd[2])[:, None]

        def T(m: Tensor) -> Tensor:
            mk, mi = m[k], m[i]
            fi = b2 * (mk * v).sum(-1, keepdim=True) * v - b1 * mk
            fk = b2 * (mi * v).sum(-1, keepdim=True) * v - b1 * mi
            return torch.zeros_like(m).index_add_(0, i, fi).index_add_(0, k, fk)

        polar = alpha > 0
        inv_a = torch.where(polar, 1.0 / alpha.clamp_min(1e-30), torch.ones_like(alpha))[:, None]
        mask = polar[:, None].to(E.dtype)

        def A(m: Tensor) -> Tensor:
            return mask * (inv_a * m - T(m))

        mu = alpha[:, None] * E
        res = mask * E - A(mu)
        z = alpha[:, None] * res
        p = z.clone()
        rz = (res * z).sum()
        tol = self.polar_eps * DEBYE
        for _ in range(self.max_iter):
            if float(rz) == 0.0:
                break
            Ap = A(p)
            step = rz / (p * Ap).sum()
            mu = mu + step * p
            res = res - step * Ap
            if float(torch.sqrt((step * p).pow(2).sum(-1).mean())) < tol:
                break
            z = alpha[:, None] * res
            rz_new = (res * z).sum()
            p = z + (rz_new / rz) * p
            rz = rz_new
        return mu * mask

    # ------------------------------------------------------------------ periodic water boxes
    def _periodic_ok(self) -> None:
        P = self.params
        ok = (P.scale("mpole", 2) == 0 and P.scale("mpole", 3) == 0 and P.scale("polar", 2) == 0
              and P.scale("polar", 3) == 0 and P.group_scale("direct", 1) == 0 and P.group_scale("mutual", 1) == 1
              and len(self.topology.pairs14) == 0 and len(self.topology.dihedrals) == 0)
        if not ok:
            raise NotImplementedError("periodic AMOEBA is built for boxes of small rigid-topology molecules "
                                      "(water): every intramolecular pair a 1-2 or 1-3 pair")

    def _electrostatics_periodic(self, data: AtomicGraph, x: Tensor, cell: Tensor):
        self._periodic_ok()
        rc = min(7.0, self.cutoff)
        setup = self.ewald or EwaldSetup(alpha=ewald_coefficient(rc), cutoff=rc, order=5,
                                         mesh=tuple(_mesh_size(float(torch.linalg.norm(c))) for c in cell.detach()))
        key = (setup.alpha, setup.cutoff, tuple(setup.mesh), setup.order)
        if getattr(self, "_pme_key", None) != key:
            self._pme = PolarizableMultipoles(setup, tol_debye=self.polar_eps, max_iter=self.max_iter,
                                              thole=float(self.pol_thole.max()), mutual_intra=True)
            self._pme_key = key
        pme = self._pme
        q, d, Q = self.moments(x)
        alpha = self.pol_alpha.to(x.dtype)
        mol = self.molecule_ids.to(x.device)
        pairs = pme.pairs(x.detach(), cell.detach(), mol)
        e_mp = pme.electrostatic(x, cell, pairs, q, d, Q)
        if self.polarization == "none":
            return e_mp, x.new_zeros(()), x.new_zeros(x.shape[0], 3)
        if self.polarization == "direct":
            F = pme.field(x, cell, pairs, q, d, Q, pol=alpha) / KE
            mu = alpha[:, None] * F
        else:
            mu, _, _ = pme.induce(x.detach(), cell.detach(), pairs, q.detach(), d.detach(), Q.detach(), alpha)
        u = pme.polarizable_energy(x, cell, pairs, q, d, Q, alpha, mu.detach())
        return e_mp, u - e_mp, mu

    def _vdw_periodic(self, data: AtomicGraph, x: Tensor) -> Tensor:
        n = x.shape[0]
        excl = torch.tensor(self.topology.exclusions, dtype=torch.long, device=x.device).reshape(-1, 2).t()
        cache = self.__dict__.setdefault("_excl_cache", {})
        src, dst, vec, r2, half, keep = half_edges(data, excl, n, cache)
        red = self.vdw_par[:, 2].to(x.dtype)
        par = self.vdw_parent
        bvec = x - x[par]
        if data.cell is not None:
            c = data.cell[0].to(x.dtype)
            frac = bvec @ torch.linalg.inv(c)
            bvec = (frac - torch.round(frac)) @ c                 # the bond across the boundary
        delta = (red[:, None] - 1.0) * bvec
        sv = vec + delta[dst] - delta[src]
        r = torch.linalg.norm(sv, dim=-1)
        R, eps = self._vdw_mix(src, dst, x.dtype)
        e = self._buffered_14_7(r.clamp_min(1e-6), R, eps, self.params.get("delta-halgren", 0.07),
                                self.params.get("gamma-halgren", 0.12))
        sw = quintic_switch(r, self.cutoff, 0.1 * self.cutoff)
        return (half * keep.to(x.dtype) * sw * e).sum()

    # ------------------------------------------------------------------ forward
    def forward(self, data: AtomicGraph) -> dict:
        N, B, n = self._check_batch(data)
        pos = data.pos
        x = pos.view(B, n, 3)
        val = self._valence(x)
        periodic = data.cell is not None and bool(torch.as_tensor(data.pbc).any())
        e_vdw, e_mp, e_pol, mus = [], [], [], []
        for b in range(B):
            xb = x[b]
            if periodic:
                if B != 1:
                    raise NotImplementedError("periodic AMOEBA evaluates one box per call")
                e_vdw.append(self._vdw_periodic(data, xb) * KCAL_TO_EV)
                em, ep, mu = self._electrostatics_periodic(data, xb, data.cell[b].to(xb.dtype))
            else:
                e_vdw.append(self._vdw_cluster(xb[None])[0] * KCAL_TO_EV)
                em, ep, mu = self._electrostatics_cluster(xb)
            e_mp.append(em)
            e_pol.append(ep)
            mus.append(mu)
        terms = {k: v * KCAL_TO_EV for k, v in val.items()}
        terms["e_vdw"] = torch.stack(e_vdw)
        terms["e_multipole"] = torch.stack(e_mp)
        terms["e_polar"] = torch.stack(e_pol)
        e_ref_node = self.atom_ref(data.atomic_numbers).squeeze(-1)
        terms["e_ref"] = scatter_sum(e_ref_node, data.batch, B)
        energy = sum(terms.values())
        # per-atom energies: the structure's interaction energy shared equally, plus the references
        per_atom = (energy - terms["e_ref"]) / float(n)
        node = per_atom.repeat_interleave(n) + e_ref_node
        out = {"node_energy": node, "energy": energy, "induced_dipoles": torch.cat(mus, 0),
               "node_features": node[:, None]}
        out.update(terms)
        return out

    def write_tinker_inputs(self, directory, positions, cell=None, name: str = "system"):
        """Tinker inputs of this system: ``<name>.xyz`` (coordinates, types, connectivity),
        ``<name>.key`` and the parameter file ``<name>.prm`` (for the built-in water model its
        Tinker text); returns the three paths."""
        from pathlib import Path

        from ..data.elements import SYMBOLS
        from .amoeba_params import write_tinker_key, write_tinker_xyz
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        syms = [SYMBOLS[int(z)] for z in self.top_z.tolist()]
        xyz = write_tinker_xyz(d / f"{name}.xyz", positions, self.top_type.tolist(), self.topology.bonds, syms,
                               cell=cell)
        prm = d / f"{name}.prm"
        if self.params.source_text:
            prm.write_text(self.params.source_text)
        else:
            raise ValueError("the parameter set has no Tinker text to write (read it from a .prm file)")
        key = write_tinker_key(d / f"{name}.key", prm.name, cell=cell, cutoff=self.cutoff, polar_eps=self.polar_eps)
        return xyz, key, prm

    @property
    def masses(self) -> Tensor:
        return torch.tensor([self.params.types[int(t)][3] for t in self.top_type.tolist()], dtype=torch.float64)

    @classmethod
    def from_config(cls, cfg) -> "Amoeba":
        e = dict(cfg.extra or {})
        top = e.get("topology")
        if top is None and "n_water" in e:
            return cls.water(int(e["n_water"]), e.get("ffield", "amoeba-water-2003"), cutoff=float(cfg.cutoff))
        from .topology import read_topology
        return cls(e.get("ffield", "amoeba-water-2003"), read_topology(top), cutoff=float(cfg.cutoff))


def ewald_coefficient(cutoff: float, tol: float = 1e-8) -> float:
    """Ewald ``alpha`` with ``erfc(alpha rc) / rc = tol`` (bisection; Tinker's default rule)."""
    lo, hi = 0.0, 10.0
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if math.erfc(mid * cutoff) / cutoff > tol:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def _mesh_size(length: float, density: float = 1.2) -> int:
    """Tinker's PME grid rule: at least ``density`` points per Angstrom, even, factors 2, 3 and 5."""
    k = max(16, int(math.ceil(length * density)))
    while True:
        if k % 2 == 0:
            m = k
            for f in (2, 3, 5):
                while m % f == 0:
                    m //= f
            if m == 1:
                return k
        k += 1
