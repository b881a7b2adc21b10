"""Symmetry search of sGDML (Chmiela et al., Nat. Commun. 9, 3887, 2018): pairwise matching of
training geometries through the eigenvectors of their distance matrices (an assignment problem
per pair, same-element constraint), synchronisation along a minimum spanning tree of the matching
costs, and closure of the permutations to a group (a subgroup of the longest cycles when the
closure exceeds ``max_size``). The steps are those of the published method, as in the reference
(``src/xnn/krnn/common/permutations.py``)."""
from __future__ import annotations

from typing import Optional

import numpy as np

MAX_PERMUTATIONS = 100


def _distances(r: np.ndarray, cell: Optional[np.ndarray]) -> np.ndarray:
    d = r[:, None, :] - r[None, :, :]
    if cell is not None:
        d = d - np.rint(d @ np.linalg.inv(cell)) @ cell
    return np.sqrt((d * d).sum(-1))


def match_pairs(positions: np.ndarray, atomic_numbers: np.ndarray, cell: Optional[np.ndarray] = None):
    from scipy.optimize import linear_sum_assignment
    m, n = positions.shape[:2]
    z = np.asarray(atomic_numbers)
    other = (z[:, None] != z[None, :]).astype(float)
    adj = np.stack([_distances(positions[k], cell) for k in range(m)])
    w, v = np.linalg.eigh(adj)
    vec = np.abs(v[:, :, ::-1])                      # eigenvectors by descending eigenvalue
    flat = adj.reshape(m, -1)
    perms, cost = {}, np.zeros((m, m))
    for i in range(m - 1):
        for j in range(i + 1, m):
            c = -vec[i] @ vec[j].T
            c = c + other * np.abs(c).max()
            p = linear_sum_assignment(c)[1]
            before = np.linalg.norm(flat[i] - flat[j])
            after = np.linalg.norm(adj[i][np.ix_(p, p)].reshape(-1) - flat[j])
            cost[i, j] = min(after, before)
            if after < before and not np.isclose(before, after):
                perms[i, j] = p
    cost = cost + cost.T
    np.fill_diagonal(cost, np.inf)
    return perms, cost


def synchronize(perms: dict, cost: np.ndarray, n_atoms: int) -> np.ndarray:
    from scipy.sparse import csr_matrix
    from scipy.sparse.csgraph import minimum_spanning_tree
    tree = minimum_spanning_tree(csr_matrix(np.where(np.isfinite(cost), cost, 0.0)))
    out = [np.arange(n_atoms)]
    for i, j in zip(*tree.nonzero()):
        p = perms.get((int(min(i, j)), int(max(i, j))))
        if p is not None:
            out.append(p)
    return np.unique(np.vstack(out), axis=0)


def close_group(perms: np.ndarray, max_size: int = MAX_PERMUTATIONS) -> Optional[np.ndarray]:
    perms = np.asarray(perms)
    grew = True
    while grew:
        grew = False
        for i in range(perms.shape[0]):
            for j in range(perms.shape[0]):
                new = perms[i, perms[j]]
                if not (new == perms).all(1).any():
                    perms = np.vstack((perms, new))
                    grew = True
                    if perms.shape[0] >= max_size:
                        return None
    return perms


def _cycles(perm) -> list:
    left = {i: int(perm[i]) for i in range(len(perm))}
    out = []
    while left:
        k = next(iter(left))
        cyc = []
        while k in left:
            cyc.append(k)
            k = left.pop(k)
        out.append(cyc)
    return out


def largest_cycle_subgroup(perms: np.ndarray) -> np.ndarray:
    long = [c for p in perms for c in _cycles(p) if len(c) > 1]
    shadowed = lambda c: any(len(c) < len(o) and not set(c).isdisjoint(o) for o in long)  # noqa: E731
    return perms[[k for k, p in enumerate(perms) if not any(shadowed(c) for c in _cycles(p) if len(c) > 1)]]


def find_permutations(positions, atomic_numbers, cell=None, max_size: int = MAX_PERMUTATIONS) -> np.ndarray:
    r = np.asarray(positions, dtype=float)
    cell = None if cell is None else np.asarray(cell, dtype=float)
    perms, cost = match_pairs(r, np.asarray(atomic_numbers), cell)
    synced = synchronize(perms, cost, r.shape[1])
    group = close_group(synced, max_size)
    if group is None:
        group = close_group(largest_cycle_subgroup(synced), max_size)
    return np.arange(r.shape[1])[None] if group is None else group
