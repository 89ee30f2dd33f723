"""Padding of merged batches: the reference's dataclasses
(dgf/src/data/padding.py), kept field for field because callers build them."""

import dataclasses
from typing import Dict


@dataclasses.dataclass
class NodeSetPadding:
    num_nodes: int


@dataclasses.dataclass
class EdgeSetPadding:
    num_edges: int


@dataclasses.dataclass
class Padding:
    """Fixed node / edge counts per set for a padded merged graph."""

    node_sets: Dict[str, NodeSetPadding]
    edge_sets: Dict[str, EdgeSetPadding]
