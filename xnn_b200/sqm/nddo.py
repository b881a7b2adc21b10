"""NDDO semi-empirical Hamiltonians (MNDO family) on batched dense SCF: PM3.

The model (reference ``sqmnn/models/nddo.py:1-60``, ``methods.py:63-80``) is a
Hartree-Fock calculation with the neglect of diatomic differential overlap
over a minimal valence basis of Slater ``s`` and ``p`` orbitals:

    E = 1/2 sum P (H + F) + sum_{A<B} E_core(A, B)

* ``H``: one-center energies ``U`` plus the attraction of each atom's
  electrons to the other cores, ``-Z_B (mu nu | s_B s_B)``; resonance
  integrals ``(beta_mu + beta_nu) / 2 S_mu,nu`` from the exact Slater overlaps.
* ``F = H + G(P)``: one-center Coulomb and exchange from ``Gss``, ``Gsp``,
  ``Gpp``, ``Gp2``, ``Hsp``; two-center Coulomb and exchange from the multipole
  integrals of :mod:`.integrals`.
* PM3 core-core terms (Stewart, J. Comput. Chem. 10, 209 (1989)):
  ``Z_A Z_B gamma_AB (1 + exp(-a_A R) + exp(-a_B R))`` (``R exp(-a R)`` for the
  N or O atom of an N-H or O-H pair; ``1 + 2 x_AB exp(-a_AB R)`` where diatomic
  parameters exist) plus the Gaussians ``Z_A Z_B / R sum_k K exp(-L (R-M)^2)``
  of both atoms (``L (R-M)^2 <= 25``); the amide torsion barrier
  ``k sin^2(phi)`` of every H-N-C=O group.

``energy`` is the heat of formation in eV (``Delta H_f / 23.06``):
``E - sum_A E_isol(A)`` plus the atoms' experimental heats of formation.

GPU layout: a batch of molecules is one set of padded dense matrices
``(B, nb, nb)`` (padded orbitals are shifted far above the spectrum);
integrals of all atom pairs are formed at once; the SCF runs batched
(``torch.linalg.eigh`` per molecule in one call, Pulay DIIS per molecule,
convergence tested on the device and read back every few iterations). The
energy is stationary in the density, so forces (and parameter gradients of the
energy) follow by autograd from the integrals at the converged, detached
density. Restricted for closed shells; unrestricted for open shells or when
asked.
"""
from __future__ import annotations

from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..models.base import InteratomicPotential
from ..models.registry import register_model
from . import integrals as I
from .parameters import (ATOM_HEAT, ELEMENT_KEYS, GAUSSIAN_KEYS, NDDOParameters, load_parameters,
                         principal_quantum_number, valence_occupation)

_MAXZ = 54
_PAD_SHIFT = 1.0e4          # eV added to the diagonal of padded orbitals


def _pairs_within(batch: Tensor, ptr: Tensor) -> Tuple[Tensor, Tensor]:
    """All pairs ``i < j`` of atoms of the same structure (atoms sorted by structure)."""
    n = batch.shape[0]
    idx = torch.arange(n, device=batch.device)
    after = ptr[batch + 1] - idx - 1
    total = int(after.sum())
    src = torch.repeat_interleave(idx, after)
    start = torch.cumsum(after, 0) - after
    dst = src + 1 + (torch.arange(total, device=batch.device) - torch.repeat_interleave(start, after))
    return src, dst


class _Layout:
    """Orbital layout of a batch: per atom its 4 slots in the padded matrices (the sink index ``nb`` for the
    orbitals an atom lacks), the number of orbitals per structure and the pair lists."""

    def __init__(self, batch: Tensor, n_struct: int, norb_atom: Tensor):
        dev = batch.device
        counts = torch.zeros(n_struct, dtype=torch.long, device=dev).index_add_(0, batch, torch.ones_like(batch))
        self.ptr = torch.cat([counts.new_zeros(1), torch.cumsum(counts, 0)])
        orb_counts = torch.zeros(n_struct, dtype=torch.long, device=dev).index_add_(0, batch, norb_atom)
        self.nb = int(orb_counts.max()) if n_struct else 0
        first = torch.cumsum(norb_atom, 0) - norb_atom
        nonempty = counts > 0
        mol_first = torch.zeros(n_struct, dtype=torch.long, device=dev)
        mol_first[nonempty] = first[self.ptr[:-1][nonempty]]
        local = first - mol_first[batch]
        m = torch.arange(4, device=dev)
        self.ao = torch.where(m[None, :] < norb_atom[:, None], local[:, None] + m[None, :],
                              torch.full_like(local[:, None], self.nb))
        self.valid = torch.arange(self.nb, device=dev)[None, :] < orb_counts[:, None]     # (B, nb)
        self.batch = batch
        self.n_struct = n_struct
        self.pa, self.pb = _pairs_within(batch, self.ptr)

    def gather_atoms(self, M: Tensor) -> Tensor:
        """Atom blocks ``(..., n, 4, 4)`` of padded matrices ``(..., B, nb+1, nb+1)``."""
        a = self.ao
        return M[..., self.batch[:, None, None], a[:, :, None], a[:, None, :]]

    def gather_pairs(self, M: Tensor) -> Tensor:
        return M[..., self.batch[self.pa][:, None, None], self.ao[self.pa][:, :, None], self.ao[self.pb][:, None, :]]

    def assemble(self, atom_blocks: Tensor, pair_blocks: Tensor, lead: Tuple[int, ...] = ()) -> Tensor:
        """Padded matrices from atom blocks and the (A, B) pair blocks (the (B, A) blocks their transposes);
        the sink row and column stay zero."""
        dev, dt = atom_blocks.device, atom_blocks.dtype
        M = atom_blocks.new_zeros(lead + (self.n_struct, self.nb + 1, self.nb + 1))
        a = self.ao
        lead_idx = (Ellipsis,) if lead else ()
        M[lead_idx + (self.batch[:, None, None], a[:, :, None], a[:, None, :])] = atom_blocks
        bp = self.batch[self.pa][:, None, None]
        ra, rb = self.ao[self.pa], self.ao[self.pb]
        M[lead_idx + (bp, ra[:, :, None], rb[:, None, :])] = pair_blocks
        M[lead_idx + (bp, rb[:, :, None], ra[:, None, :])] = pair_blocks.transpose(-1, -2)
        keep = torch.ones(self.nb + 1, dtype=dt, device=dev)
        keep[self.nb] = 0.0
        return M * keep[:, None] * keep[None, :]


class NDDO(InteratomicPotential):
    """Shared NDDO machinery; subclasses define :meth:`core_core` and :meth:`corrections`.

    Parameters
    ----------
    parameters : str, Path or NDDOParameters
        A MOPAC ``EXTERNAL`` parameter file (or a named set found through ``XNN_B200_NDDO_DIR``).
    trainable : sequence of str
        Parameter names (``"BETAS"``, ``"USS"``, ``"ALP"``, ``"FN11"``...) held as trainable tables.
    unrestricted : bool
        UHF for closed shells too (open shells always run unrestricted).
    density_tol, energy_tol : float
        SCF convergence: largest change of a density element and of the electronic energy (eV).
    max_iter, diis_size : int
    """

    peptide_barrier = 0.0

    def __init__(self, parameters: Union[str, Path, NDDOParameters], trainable: Sequence[str] = (),
                 unrestricted: bool = False, density_tol: float = 1e-10, energy_tol: float = 1e-10,
                 max_iter: int = 300, diis_size: int = 8, check_every: int = 4):
        super().__init__()
        self.parameters_source = load_parameters(parameters)
        p = self.parameters_source
        self.unrestricted = unrestricted
        self.density_tol, self.energy_tol = density_tol, energy_tol
        self.max_iter, self.diis_size, self.check_every = max_iter, diis_size, check_every
        keys = ELEMENT_KEYS + GAUSSIAN_KEYS
        trainable = set(trainable)
        unknown = trainable - set(keys) - {"ALPB", "XFAC"}
        if unknown:
            raise ValueError(f"unknown trainable parameters {sorted(unknown)}")
        for key in keys:
            t = torch.zeros(_MAXZ + 1, dtype=torch.float64)
            for z in p.elements:
                if z <= _MAXZ:
                    t[z] = p.value(z, key)
            if key in trainable:
                setattr(self, "p_" + key, nn.Parameter(t))
            else:
                self.register_buffer("p_" + key, t)
        for key in ("ALPB", "XFAC"):
            t = torch.zeros(_MAXZ + 1, _MAXZ + 1, dtype=torch.float64)
            for (z1, z2), vals in p.pairs.items():
                if z1 <= _MAXZ:
                    t[z1, z2] = t[z2, z1] = vals.get(key, 0.0)
            if key in trainable:
                setattr(self, "p_" + key, nn.Parameter(t))
            else:
                self.register_buffer("p_" + key, t)
        self.register_buffer("atom_heat", torch.tensor([ATOM_HEAT.get(z, 0.0) for z in range(_MAXZ + 1)],
                                                       dtype=torch.float64))

    # ----------------------------------------------------------------------------------------------- hooks
    def core_core(self, za: Tensor, zb: Tensor, r: Tensor, gab: Tensor, tore_a: Tensor, tore_b: Tensor) -> Tensor:
        raise NotImplementedError

    def corrections(self, z: Tensor, pos: Tensor, batch: Tensor,
                    pairs: Optional[Tuple[Tensor, Tensor]] = None) -> Tensor:
        """Per-atom post-SCF corrections (kcal/mol); ``pairs`` are the atom pairs ``i < j`` of each structure."""
        return pos.new_zeros(z.shape[0])

    def parameter_set(self) -> NDDOParameters:
        """The current values as a parameter set (writable with :func:`~.parameters.save_parameters`)."""
        out = NDDOParameters(name=self.parameters_source.name)
        for z in self.parameters_source.elements:
            out.elements[z] = {k: float(getattr(self, "p_" + k)[z]) for k in ELEMENT_KEYS + GAUSSIAN_KEYS
                               if float(getattr(self, "p_" + k)[z]) != 0.0}
        for (z1, z2) in self.parameters_source.pairs:
            out.pairs[(z1, z2)] = {k: float(getattr(self, "p_" + k)[z1, z2]) for k in ("ALPB", "XFAC")}
        out.globals = dict(self.parameters_source.globals)
        return out

    # ----------------------------------------------------------------------------------------------- elements
    def _elements(self, uz: List[int], device, dtype) -> Dict[str, Tensor]:
        for z in uz:
            if z not in self.parameters_source.elements:
                raise ValueError(f"no parameters for element Z={z}")
            valence_occupation(z)
        zt = torch.tensor(uz, device=device)
        table = {k: getattr(self, "p_" + k).to(device=device, dtype=dtype)[zt] for k in ELEMENT_KEYS}
        has_p = table["ZP"] > 1e-20
        pqn = torch.tensor([principal_quantum_number(z) for z in uz], device=device)
        occ = torch.tensor([valence_occupation(z) for z in uz], device=device)
        q = I.element_quantities(zt, table, pqn, occ[:, 0], occ[:, 1], has_p)
        q.update(table=table, has_p=has_p, pqn=pqn, z=zt, tore=(occ[:, 0] + occ[:, 1]).to(dtype),
                 occ=occ.to(dtype), norb=torch.where(has_p, 4, 1))
        return q

    # ----------------------------------------------------------------------------------------------- integrals
    def _integrals(self, el: Dict[str, Tensor], sp: Tensor, pos: Tensor, lay: _Layout):
        """Core Hamiltonian atom and pair blocks, the two-center integrals (molecular frame) and the core-core
        energies of all pairs."""
        pa, pb = lay.pa, lay.pb
        sa, sb = sp[pa], sp[pb]
        vec = pos[pb] - pos[pa]
        r, frames = I.pair_frames(vec)
        rb = r / I.BOHR
        T = I.orbital_rotation(frames)
        dsep = I._separations(el["dd"], el["qq"])
        rho = I._slot_rho(el["rho"])
        tore = el["tore"]
        W = rb.new_zeros(rb.shape[0], 4, 4, 4, 4)
        Va = rb.new_zeros(rb.shape[0], 4, 4)
        Vb = rb.new_zeros(rb.shape[0], 4, 4)
        chunk = 8192
        for s0 in range(0, rb.shape[0], chunk):
            sl = slice(s0, s0 + chunk)
            a, b = sa[sl], sb[sl]
            W[sl] = I.rotate4(I.local_repulsion(rb[sl], dsep[a], rho[a], dsep[b], rho[b]), T[sl])
            Va[sl] = I.rotate2(I.local_core_attraction(rb[sl], dsep[a], rho[a], el["po9"][b], 1.0), T[sl])
            Vb[sl] = I.rotate2(I.local_core_attraction(rb[sl], dsep[b], rho[b], el["po9"][a], -1.0), T[sl])
        # overlaps by (n_A, n_B, p_A, p_B) group
        Sloc = rb.new_zeros(rb.shape[0], 4, 4)
        na, nbq = el["pqn"][sa], el["pqn"][sb]
        hpa, hpb = el["has_p"][sa], el["has_p"][sb]
        key = ((na * 8 + nbq) * 2 + hpa.long()) * 2 + hpb.long()
        for k in torch.unique(key).tolist():
            m = torch.nonzero(key == k).squeeze(1)
            kk = int(k)
            ppb, ppa = bool(kk & 1), bool((kk >> 1) & 1)
            n1, n2 = (kk >> 2) // 8, (kk >> 2) % 8
            tab = el["table"]
            Sloc = Sloc.index_put((m,), I.local_overlaps(n1, n2, tab["ZS"][sa[m]], tab["ZP"][sa[m]].clamp(min=0.3),
                                                         tab["ZS"][sb[m]], tab["ZP"][sb[m]].clamp(min=0.3),
                                                         rb[m], ppa, ppb))
        Smol = torch.einsum("nia,nab,njb->nij", T, Sloc, T)
        tab = el["table"]
        beta = torch.stack([tab["BETAS"], tab["BETAP"], tab["BETAP"], tab["BETAP"]], -1)
        H_pair = 0.5 * (beta[sa][:, :, None] + beta[sb][:, None, :]) * Smol
        # core Hamiltonian atom blocks: U plus the other cores' attraction
        U = torch.stack([tab["UPP"]] * 4, -1).clone()
        U[:, 0] = tab["USS"]
        H_atom = torch.diag_embed(U[sp])
        H_atom = H_atom.index_add(0, pa, -tore[sb][:, None, None] * Va).index_add(0, pb, -tore[sa][:, None, None] * Vb)
        gab = I.HARTREE / torch.sqrt(rb * rb + (el["po9"][sa] + el["po9"][sb]) ** 2)
        e_core = self.core_core(el["z"][sa], el["z"][sb], r, gab, tore[sa], tore[sb])
        return H_atom, H_pair, W, e_core

    # ----------------------------------------------------------------------------------------------- Fock
    @staticmethod
    def _fock_blocks(lay: _Layout, one: Tensor, W: Tensor, P: Tensor):
        """Two-electron atom and pair blocks ``G`` for spin densities ``P (S, B, nb+1, nb+1)`` (``S = 1``:
        restricted, ``P`` the density of one spin)."""
        S = P.shape[0]
        PA = lay.gather_atoms(P)                           # (S, n, 4, 4)
        PA_tot = PA.sum(0) * (2.0 if S == 1 else 1.0)
        PAB = lay.gather_pairs(P)                          # (S, p, 4, 4)
        G_atom = torch.einsum("nijkl,nkl->nij", one, PA_tot)[None] - torch.einsum("nikjl,snkl->snij", one, PA)
        J_a = torch.einsum("pijkl,pkl->pij", W, PA_tot[lay.pb])
        J_b = torch.einsum("pijkl,pij->pkl", W, PA_tot[lay.pa])
        G_atom = G_atom + (torch.zeros_like(PA_tot).index_add(0, lay.pa, J_a).index_add(0, lay.pb, J_b))[None]
        G_pair = -torch.einsum("pijkl,spjl->spik", W, PAB)
        return G_atom, G_pair

    def _fock(self, lay, H, one, W, P):
        G_atom, G_pair = self._fock_blocks(lay, one, W, P)
        return H[None] + lay.assemble(G_atom, G_pair, lead=(P.shape[0],))

    # ----------------------------------------------------------------------------------------------- SCF
    def _scf(self, lay: _Layout, H: Tensor, one: Tensor, W: Tensor, n_occ: Tensor, P0: Tensor) -> Tensor:
        """Converged spin densities (no autograd). ``n_occ (S, B)`` occupied orbitals per spin."""
        nb = lay.nb
        S, B = n_occ.shape
        pad = (~lay.valid).to(H.dtype) * _PAD_SHIFT
        cols = torch.arange(nb, device=H.device)
        occ_mask = (cols[None, None, :] < n_occ[:, :, None]).to(H.dtype)       # (S, B, nb)
        P = P0
        F_hist: List[Tensor] = []
        e_hist: List[Tensor] = []
        e_old = None
        converged = False
        for it in range(self.max_iter):
            F = self._fock(lay, H, one, W, P)
            Fv = F[..., :nb, :nb]
            Pv = P[..., :nb, :nb]
            e_el = 0.5 * ((Pv * (H[None, :, :nb, :nb] + Fv)).sum((-1, -2)) * (2.0 if S == 1 else 1.0)).sum(0)
            err = Fv @ Pv - Pv @ Fv
            F_hist.append(Fv)
            e_hist.append(err)
            if len(F_hist) > self.diis_size:
                F_hist.pop(0)
                e_hist.pop(0)
            m = len(F_hist)
            if m >= 2:
                E = torch.stack(e_hist, 0)                                        # (m, S, B, nb, nb)
                Bm = torch.einsum("isbxy,jsbxy->bij", E, E)
                A = Bm.new_zeros(B, m + 1, m + 1)
                A[:, :m, :m] = Bm / Bm.diagonal(dim1=-2, dim2=-1).amax(-1).clamp(min=1e-300)[:, None, None]
                A[:, :m, m] = -1.0
                A[:, m, :m] = -1.0
                rhs = Bm.new_zeros(B, m + 1)
                rhs[:, m] = -1.0
                A[:, :m, :m] += 1e-14 * torch.eye(m, dtype=A.dtype, device=A.device)
                c = torch.linalg.solve(A, rhs)[:, :m]                                # (B, m)
                Fx = torch.einsum("bi,isbxy->sbxy", c, torch.stack(F_hist, 0))
            else:
                Fx = Fv
            Fx = Fx + torch.diag_embed(pad)[None]
            eps, C = torch.linalg.eigh(Fx)
            if it < self.smear_iters:
                # Fermi smearing with a falling temperature steers the first iterations to the ground state
                kt = self.smear_kt * (1.0 - it / self.smear_iters)
                Co = C * _fermi(eps, n_occ, kt)[:, :, None, :]
                if it == self.smear_iters - 1:
                    F_hist.clear()
                    e_hist.clear()
            else:
                Co = C * occ_mask[:, :, None, :]
            Pn = Co @ C.transpose(-1, -2)
            Pn = torch.nn.functional.pad(Pn, (0, 1, 0, 1))
            dP = (Pn - P).abs().amax()
            dE = (e_el - e_old).abs().amax() if e_old is not None else torch.full((), float("inf"), device=H.device,
                                                                                dtype=H.dtype)
            P, e_old = Pn, e_el
            if (it + 1) % self.check_every == 0 or it == self.max_iter - 1:
                flags = torch.stack([dP <= self.density_tol, dE <= self.energy_tol]).tolist()
                if all(flags):
                    converged = True
                    break
        if not converged:
            raise RuntimeError(f"NDDO SCF did not converge in {self.max_iter} iterations")
        return P

    smear_iters = 16
    smear_kt = 1.0

    def _initial_density(self, lay: _Layout, el, sp: Tensor, n_e: Tensor, S: int, n_spin: Tensor) -> Tensor:
        occ = el["occ"][sp]                                                   # (n, 2)
        shells = torch.stack([occ[:, 0], occ[:, 1] / 3.0, occ[:, 1] / 3.0, occ[:, 1] / 3.0], -1)
        shells = shells * (lay.ao < lay.nb).to(shells.dtype)
        tot = torch.zeros(lay.n_struct, dtype=shells.dtype, device=shells.device).index_add(0, lay.batch,
                                                                                              shells.sum(-1))
        scale = n_e.to(shells.dtype) / tot.clamp(min=1e-12)
        diag = shells * scale[lay.batch][:, None]
        blocks = torch.diag_embed(diag)
        P = lay.assemble(blocks, blocks.new_zeros(lay.pa.shape[0], 4, 4))
        frac = n_spin.to(P.dtype) / n_e.clamp(min=1).to(P.dtype)                # (S, B)
        return P[None] * frac[:, :, None, None]

    # ----------------------------------------------------------------------------------------------- forward
    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        z = data.atomic_numbers.long()
        pos = data.pos
        dt = torch.float64
        pos64 = pos.to(dt)
        batch = data.batch if data.batch is not None else torch.zeros_like(z)
        n_struct = data.num_graphs
        uz = sorted(set(z.tolist()))
        el = self._elements(uz, pos.device, dt)
        lookup = torch.zeros(_MAXZ + 1, dtype=torch.long, device=z.device)
        lookup[torch.tensor(uz, device=z.device)] = torch.arange(len(uz), device=z.device)
        sp = lookup[z]
        lay = _Layout(batch, n_struct, el["norb"][sp])
        charge = (data.total_charge.to(dt).reshape(-1) if data.total_charge is not None
                  else torch.zeros(n_struct, dtype=dt, device=pos.device))
        n_e = (torch.zeros(n_struct, dtype=dt, device=pos.device).index_add(0, batch, el["tore"][sp]) - charge)
        n_e = torch.round(n_e).long()
        mult = 1 + n_e % 2
        if data.spin_multiplicity is not None:
            # a multiplicity of 0 (a structure batched without one) means the lowest for its electron count
            given = torch.round(data.spin_multiplicity.to(dt).reshape(-1)).long()
            mult = torch.where(given > 0, given, mult)
        if bool(((n_e + mult - 1) % 2 != 0).any()):
            raise ValueError("spin multiplicity inconsistent with the electron count")
        n_alpha, n_beta = (n_e + mult - 1) // 2, (n_e - mult + 1) // 2
        uhf = self.unrestricted or bool((mult != 1).any())
        n_occ = torch.stack([n_alpha, n_beta]) if uhf else n_alpha[None]

        H_atom, H_pair, W, e_core = self._integrals(el, sp, pos64, lay)
        one = el["one_center"][sp]
        H = lay.assemble(H_atom, H_pair)
        with torch.no_grad():
            P0 = self._initial_density(lay, el, sp, n_e, n_occ.shape[0], n_occ)
            P = self._scf(lay, H.detach(), one.detach(), W.detach(), n_occ, P0)

        # energies at the converged density (stationary: autograd gives forces and parameter gradients)
        S = P.shape[0]
        w = 2.0 if S == 1 else 1.0
        G_atom, G_pair = self._fock_blocks(lay, one, W, P)
        PA = lay.gather_atoms(P)
        PAB = lay.gather_pairs(P)
        # per-atom electronic energy: the atom blocks and half of each pair block to each atom
        e_atom = w * ((PA * (H_atom[None] + 0.5 * G_atom)).sum((-1, -2))).sum(0)
        e_pair = w * 2.0 * ((PAB * (H_pair[None] + 0.5 * G_pair)).sum((-1, -2))).sum(0)
        e_atom = e_atom.index_add(0, lay.pa, 0.5 * (e_pair + e_core)).index_add(0, lay.pb, 0.5 * (e_pair + e_core))
        corr = self.corrections(z, pos64, batch, (lay.pa, lay.pb))
        node_kcal = (e_atom - el["eisol"][sp]) * I.EV_TO_KCAL + self.atom_heat.to(pos.device)[z] + corr
        hof = torch.zeros(n_struct, dtype=dt, device=pos.device).index_add(0, batch, node_kcal)
        zeros = torch.zeros(n_struct, dtype=dt, device=pos.device)
        e_el = zeros.index_add(0, batch, w * ((PA * (H_atom[None] + 0.5 * G_atom)).sum((-1, -2))).sum(0))
        e_el = e_el.index_add(0, batch[lay.pa], e_pair)
        e_nuc = zeros.index_add(0, batch[lay.pa], e_core)
        P_tot = PA.sum(0) * w
        charges = el["tore"][sp] - P_tot.diagonal(dim1=-2, dim2=-1).sum(-1)
        # dipole: point charges plus the sp hybridization dipoles (about the centre of mass of ions)
        hyb = -2.0 * I.BOHR * el["dd"][sp][:, None] * P_tot[:, 0, 1:]
        dip_atom = charges[:, None] * pos64 + hyb
        mass = torch.tensor([_MASS.get(v, 0.0) for v in range(_MAXZ + 1)], dtype=dt, device=pos.device)[z]
        msum = zeros.index_add(0, batch, mass)
        com = torch.zeros(n_struct, 3, dtype=dt, device=pos.device).index_add(0, batch, mass[:, None] * pos64)
        com = com / msum[:, None] * (charge.abs() > 0.5).to(dt)[:, None]
        dip_atom = dip_atom - charges[:, None] * com[batch]
        dipole = torch.zeros(n_struct, 3, dtype=dt, device=pos.device).index_add(0, batch, dip_atom)
        return {
            "node_energy": (node_kcal / I.EV_TO_KCAL).to(pos.dtype),
            "energy": (hof / I.EV_TO_KCAL).to(pos.dtype),
            "heat_of_formation": hof,
            "total_energy": e_el + e_nuc,
            "electronic_energy": e_el,
            "core_core_energy": e_nuc,
            "charges": charges,
            "dipole": dipole,
            "density": P.detach(),
        }

    @classmethod
    def from_config(cls, cfg) -> "NDDO":
        extra = dict(getattr(cfg, "extra", {}) or {})
        return cls(extra.pop("parameters"), **extra)


def _fermi(eps: Tensor, n_occ: Tensor, kt: float) -> Tensor:
    """Occupations ``1 / (1 + exp((eps - mu) / kt))`` with ``mu`` per spin and structure set by bisection so
    that they sum to ``n_occ``."""
    lo = eps.amin(-1) - 50.0 * kt - 1.0
    hi = torch.minimum(eps.amax(-1), eps.amin(-1) + 1.0e3) + 50.0 * kt + 1.0
    target = n_occ.to(eps.dtype)
    for _ in range(100):
        mu = 0.5 * (lo + hi)
        f = torch.sigmoid((mu[..., None] - eps) / kt).sum(-1)
        lo = torch.where(f < target, mu, lo)
        hi = torch.where(f < target, hi, mu)
    return torch.sigmoid(((0.5 * (lo + hi))[..., None] - eps) / kt)


# average atomic masses (u) for the centre of mass of ions
_MASS = {1: 1.00790, 3: 6.94, 4: 9.01218, 5: 10.81, 6: 12.011, 7: 14.0067, 8: 15.9994, 9: 18.9984, 11: 22.98977,
         12: 24.305, 13: 26.98154, 14: 28.0855, 15: 30.97376, 16: 32.06, 17: 35.453, 19: 39.0983, 20: 40.08,
         31: 69.735, 32: 72.59, 33: 74.9216, 34: 78.96, 35: 79.904, 37: 85.4678, 38: 87.62, 49: 114.82,
         50: 118.69, 51: 121.75, 52: 127.6, 53: 126.9045}


def _sin2_dihedral(p: Tensor, i: int, j: int, k: int, l: int) -> Tensor:
    b1, b2, b3 = p[j] - p[i], p[k] - p[j], p[l] - p[k]
    n1, n2 = torch.linalg.cross(b1, b2), torch.linalg.cross(b2, b3)
    c = (n1 * n2).sum() / (n1.norm() * n2.norm())
    return 1.0 - c * c


def amide_torsions(z: Tensor, pos: Tensor, barrier: float, batch: Optional[Tensor] = None,
                   pairs: Optional[Tuple[Tensor, Tensor]] = None) -> Tensor:
    """Per-atom amide torsion barrier (kcal/mol) on the nitrogen of each H-N-C=O group.

    A carbon with an oxygen within 1.3 A, a nitrogen within 1.6 A that has a hydrogen within 1.3 A and a
    further neighbour X within 1.7 A (neither the carbon nor that hydrogen) adds ``barrier`` times
    ``sin^2`` of the torsions O=C-N-X and O=C-N-H; each nitrogen counts once and, per carbon, the first
    match in atom order is taken (reference ``sqmnn/models/corrections.py:368-414``). The search runs on
    the host over the neighbour lists within 1.7 A of the atom pairs of each structure (``pairs``, all
    pairs ``i < j`` of a structure; built from ``batch`` when not given)."""
    out = pos.new_zeros(z.shape[0])
    if barrier == 0.0 or z.shape[0] < 4:
        return out
    if pairs is None:
        b = batch if batch is not None else torch.zeros_like(z)
        counts = torch.zeros(int(b.max()) + 1, dtype=torch.long, device=z.device).index_add_(0, b, torch.ones_like(b))
        pairs = _pairs_within(b, torch.cat([counts.new_zeros(1), torch.cumsum(counts, 0)]))
    pa, pb = pairs
    r = (pos.detach()[pb] - pos.detach()[pa]).norm(dim=-1)
    near = r <= 1.7
    zl = z.tolist()
    ia, ib, rr = pa[near].tolist(), pb[near].tolist(), r[near].tolist()
    nbrs: Dict[int, List[Tuple[int, float]]] = {}
    for a, b, d in zip(ia, ib, rr):
        nbrs.setdefault(a, []).append((b, d))
        nbrs.setdefault(b, []).append((a, d))
    for v in nbrs.values():
        v.sort()
    used = set()
    for c in sorted(a for a in nbrs if zl[a] == 6):
        hit = None
        for o in (a for a, d in nbrs[c] if zl[a] == 8 and d <= 1.3):
            for n in (a for a, d in nbrs[c] if zl[a] == 7 and d <= 1.6):
                for h in (a for a, d in nbrs.get(n, []) if zl[a] == 1 and d <= 1.3):
                    xs = [a for a, d in nbrs[n] if a not in (h, c)]
                    if xs and n not in used:
                        hit = (o, n, h, xs[0])
                        break
                if hit:
                    break
            if hit:
                break
        if hit:
            o, n, h, x = hit
            used.add(n)
            e = barrier * (_sin2_dihedral(pos, o, c, n, x) + _sin2_dihedral(pos, o, c, n, h))
            out = out.index_add(0, torch.tensor([n], device=pos.device), e.reshape(1))
    return out


@register_model("pm3")
class PM3(NDDO):
    """PM3 (Stewart 1989) on the NDDO machinery of this module."""

    peptide_barrier = 7.1853

    def core_core(self, za, zb, r, gab, tore_a, tore_b):
        zz = tore_a * tore_b
        enuc = zz * gab
        x = self.p_XFAC.to(r.device)[za, zb]
        a = self.p_ALPB.to(r.device)[za, zb]
        a = torch.where(a < 1e-6, torch.full_like(a, 1.2), a)
        diatomic = x.abs() > 1e-5
        alp = self.p_ALP.to(r.device)
        ea, eb = torch.exp(-alp[za] * r), torch.exp(-alp[zb] * r)
        nh = ((za == 1) & ((zb == 7) | (zb == 8))) | ((zb == 1) & ((za == 7) | (za == 8)))
        fa = torch.where(nh & (za != 1), r * ea, ea)
        fb = torch.where(nh & (zb != 1), r * eb, eb)
        e = torch.where(diatomic, enuc * (1.0 + 2.0 * x * torch.exp(-a * r)), (enuc * (fa + fb)).abs() + enuc)
        # Gaussians of both atoms (pairs without diatomic parameters)
        gauss = torch.zeros_like(r)
        for k in range(1, 5):
            for zt in (za, zb):
                K = getattr(self, f"p_FN1{k}").to(r.device)[zt]
                L = getattr(self, f"p_FN2{k}").to(r.device)[zt]
                M = getattr(self, f"p_FN3{k}").to(r.device)[zt]
                ax = L * (r - M) ** 2
                ok = (ax <= 25.0) & (K.abs() > 0.0) & ~(x > 1e-4)
                gauss = gauss + torch.where(ok, zz / r * K * torch.exp(-torch.where(ok, ax, torch.zeros_like(ax))),
                                            torch.zeros_like(r))
        return e + gauss

    def corrections(self, z, pos, batch, pairs=None):
        return amide_torsions(z, pos, self.peptide_barrier, batch, pairs)
