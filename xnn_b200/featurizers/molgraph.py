"""Two-dimensional molecular graphs for graph-parameterised force fields (the EGT trunk of ByteFF):
integer atom features (element, degree, formal charge, ring degree, smallest ring of at most
``MAX_RING_SIZE`` atoms), bond features (in ring, order), the bonds, angles, proper torsions and
impropers (carbon / nitrogen centres with three neighbours, centre first) with the directed edges
along each term, pairs one to four bonds apart, torsions through linear centres, and the classes of
topologically equivalent atoms and bonds.

Built here from an explicit bond list with bond orders and formal charges (RDKit, which perceives
them from coordinates and standardises resonance structures in the reference, is not part of this
build). Equivalence classes come from colour refinement (1-WL) of the graph with single bonds and no
charges, which separates every atom pair that any graph invariant separates on molecular graphs of
this size in practice. Field layout and conventions follow the reference
(``src/xnn/gnn/featurizers/molgraph.py``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

MAX_RING_SIZE = 8
BOND_ORDERS = (1.0, 2.0, 3.0, 1.5)


@dataclass
class MolecularGraph:
    atomic_numbers: np.ndarray
    formal_charges: np.ndarray
    degree: np.ndarray
    ring_degree: np.ndarray
    min_ring: np.ndarray
    bonds: np.ndarray
    bond_in_ring: np.ndarray
    bond_order: np.ndarray
    angles: np.ndarray
    propers: np.ndarray
    impropers: np.ndarray
    angle_edges: np.ndarray
    proper_edges: np.ndarray
    improper_edges: np.ndarray
    proper_linear: np.ndarray
    hypervalent: np.ndarray
    atom_class: np.ndarray
    edge_class: np.ndarray
    pairs12: np.ndarray
    pairs13: np.ndarray
    pairs14: np.ndarray
    pairs15: np.ndarray
    smiles: str = field(default="")

    @property
    def n_atoms(self) -> int:
        return int(self.atomic_numbers.shape[0])

    @property
    def total_charge(self) -> int:
        return int(self.formal_charges.sum())

    def node_features(self) -> np.ndarray:
        """``(N, 5)``: element, degree, formal charge, ring degree, smallest ring."""
        return np.stack([self.atomic_numbers, self.degree, self.formal_charges, self.ring_degree, self.min_ring], 1)

    def edge_features(self) -> np.ndarray:
        """``(2M, 2)`` per directed bond (both directions consecutive): in ring, order index."""
        return np.repeat(np.stack([self.bond_in_ring, self.bond_order], 1), 2, axis=0)

    def edge_index(self) -> np.ndarray:
        """``(2, 2M)`` directed bonds ``(i -> j), (j -> i)`` per bond."""
        return np.stack([self.bonds, self.bonds[:, ::-1]], 1).reshape(-1, 2).T.copy()


def _shells(adj, n: int, limit: int):
    out = []
    for s in range(n):
        seen, front = {s: 0}, [s]
        for d in range(1, limit + 1):
            nxt = []
            for a in front:
                for b in adj[a]:
                    if b not in seen:
                        seen[b] = d
                        nxt.append(b)
            front = nxt
        out.append(seen)
    return out


def _cycle_through(adj, a: int, b: int, limit: int) -> int:
    """Size of the smallest ring of at most ``limit`` atoms through bond ``a-b`` (0 if none)."""
    seen, front = {a}, [a]
    for d in range(1, limit):
        nxt = []
        for x in front:
            for y in adj[x]:
                if x == a and y == b:
                    continue
                if y == b:
                    return d + 1
                if y not in seen:
                    seen.add(y)
                    nxt.append(y)
        front = nxt
    return 0


def _canonical(t: tuple) -> tuple:
    for i in range(len(t) // 2):
        if t[i] != t[-i - 1]:
            return t if t[i] < t[-i - 1] else t[::-1]
    return t


def _refine(z: Sequence[int], adj) -> list:
    """Colour refinement of the element-labelled graph to a fixed point; class ids by first atom."""
    col = [int(v) for v in z]
    for _ in range(len(z)):
        sig = [(col[i], tuple(sorted(col[j] for j in adj[i]))) for i in range(len(z))]
        ids = {s: k for k, s in enumerate(sorted(set(sig)))}
        new = [ids[s] for s in sig]
        if len(set(new)) == len(set(col)):
            col = new
            break
        col = new
    return col


def molecular_graph_from_bonds(atomic_numbers: Sequence[int], bonds: Sequence[Sequence[int]],
                               bond_orders: Optional[Sequence[float]] = None,
                               formal_charges: Optional[Sequence[int]] = None) -> MolecularGraph:
    """A :class:`MolecularGraph` of one molecule (explicit hydrogens) from its bonds, bond orders
    (1, 1.5, 2, 3; single by default) and formal charges (zero by default)."""
    z = np.asarray(atomic_numbers, dtype=np.int64)
    n = len(z)
    fc = np.zeros(n, dtype=np.int64) if formal_charges is None else np.asarray(formal_charges, dtype=np.int64)
    orders = [1.0] * len(bonds) if bond_orders is None else [float(o) for o in bond_orders]
    adj = [[] for _ in range(n)]
    order_of = {}
    for (i, j), o in zip(bonds, orders):
        i, j = sorted((int(i), int(j)))
        if o not in BOND_ORDERS:
            raise ValueError(f"bond {i}-{j} has unsupported order {o}")
        order_of[(i, j)] = BOND_ORDERS.index(o)
        adj[i].append(j)
        adj[j].append(i)
    adj = [sorted(a) for a in adj]
    blist = sorted(order_of)
    edge = {}
    for k, (i, j) in enumerate(blist):
        edge[(i, j)], edge[(j, i)] = 2 * k, 2 * k + 1
    cycle = {bd: _cycle_through(adj, bd[0], bd[1], MAX_RING_SIZE) for bd in blist}
    ring_degree, min_ring = np.zeros(n, dtype=np.int64), np.zeros(n, dtype=np.int64)
    for (i, j), size in cycle.items():
        if size:
            for a in (i, j):
                ring_degree[a] += 1
                min_ring[a] = size if min_ring[a] == 0 else min(min_ring[a], size)
    angles = sorted({(a, c, b) if a < b else (b, c, a) for c in range(n) for x, a in enumerate(adj[c])
                     for b in adj[c][x + 1:]})
    propers = sorted({_canonical((a, b, c, d)) for b, c in blist for a in adj[b] for d in adj[c]
                      if a != c and d != b and a != d})
    impropers = sorted((c, *adj[c]) for c in range(n) if z[c] in (6, 7) and len(adj[c]) == 3)
    hcount = [sum(1 for j in adj[i] if z[j] == 1) for i in range(n)]
    ring5or6 = [any(cycle.get(tuple(sorted((i, j))), 0) in (5, 6) for j in adj[i]) for i in range(n)]

    def linear(i, ends):
        if z[i] == 6 and len(adj[i]) == 2:
            return not ring5or6[i]
        if z[i] == 7 and len(adj[i]) == 2 and fc[i] == 1:
            return not any(z[j] == 7 and hcount[j] == 1 for j in ends)
        return False
    proper_linear = np.array([linear(p[1], (p[0], p[2])) or linear(p[2], (p[3], p[1])) for p in propers], dtype=bool)
    rank = _refine(z, adj)
    first: dict = {}
    atom_class = np.array([first.setdefault(r, i) for i, r in enumerate(rank)], dtype=np.int64)
    first = {}
    directed = [e for i, j in blist for e in ((i, j), (j, i))]
    edge_class = np.array([first.setdefault(tuple(sorted((rank[i], rank[j]))), k) for k, (i, j) in enumerate(directed)],
                          dtype=np.int64)
    dist = _shells(adj, n, 4)
    shells = {d: set() for d in (1, 2, 3, 4)}
    for i in range(n):
        for j, d in dist[i].items():
            if i < j and d in shells:
                shells[d].add((i, j))

    def arr(rows, width):
        return np.asarray(rows, dtype=np.int64).reshape(-1, width)
    return MolecularGraph(
        atomic_numbers=z, formal_charges=fc, degree=np.array([len(a) for a in adj], dtype=np.int64),
        ring_degree=ring_degree, min_ring=min_ring, bonds=arr(blist, 2),
        bond_in_ring=np.array([cycle[bd] > 0 for bd in blist], dtype=np.int64),
        bond_order=np.array([order_of[bd] for bd in blist], dtype=np.int64),
        angles=arr(angles, 3), propers=arr(propers, 4), impropers=arr(impropers, 4),
        angle_edges=arr([(edge[(a, b)], edge[(b, c)]) for a, b, c in angles], 2),
        proper_edges=arr([(edge[(a, b)], edge[(b, c)], edge[(c, d)]) for a, b, c, d in propers], 3),
        improper_edges=arr([(edge[(c, x)], edge[(c, y)], edge[(c, w)]) for c, x, y, w in impropers], 3),
        proper_linear=proper_linear,
        hypervalent=np.array([z[i] in (15, 16) and len(adj[i]) >= 5 for i in range(n)], dtype=bool),
        atom_class=atom_class, edge_class=edge_class,
        pairs12=arr(sorted(shells[1]), 2), pairs13=arr(sorted(shells[2]), 2), pairs14=arr(sorted(shells[3]), 2),
        pairs15=arr(sorted(shells[4]), 2))
