"""In-memory graph containers.

Same structure as DGF's boundary types (dgf/src/data/in_memory_graph.py:24-69)
because the sampler's callers construct and consume them: a graph is a dict of
node sets (num_nodes + per-node feature arrays) and a dict of edge sets (an
int [2, num_edges] adjacency, row 0 = source index, row 1 = target index, plus
per-edge feature arrays).
"""

from __future__ import annotations

import dataclasses
from typing import Dict, Optional

import numpy as np

Features = Dict[str, np.ndarray]


@dataclasses.dataclass(frozen=True)
class InMemoryNodeSet:
    """A node set: node count and per-node features ([num_nodes, ...])."""

    num_nodes: Optional[int]
    features: Features = dataclasses.field(default_factory=dict)


@dataclasses.dataclass(frozen=True)
class InMemoryEdgeSet:
    """An edge set: [2, num_edges] adjacency and per-edge features."""

    adjacency: np.ndarray
    features: Features = dataclasses.field(default_factory=dict)

    def num_edges(self) -> int:
        return self.adjacency.shape[1]


@dataclasses.dataclass(frozen=True)
class InMemoryGraph:
    """A heterogeneous graph held in host memory."""

    node_sets: Dict[str, InMemoryNodeSet]
    edge_sets: Dict[str, InMemoryEdgeSet]
    timestamp: Optional[int] = None
