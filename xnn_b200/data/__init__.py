"""Core data: the :class:`AtomicGraph`, neighbour lists, datasets, batching and synthetic data."""
from .atomic_graph import AtomicGraph
from .dataset import AtomicDataset, collate, structure_to_graph
from .neighborlist import build_neighbor_list, nearest_edges, unique_pairs

__all__ = ["AtomicDataset", "AtomicGraph", "build_neighbor_list", "collate", "nearest_edges",
           "structure_to_graph", "unique_pairs"]
