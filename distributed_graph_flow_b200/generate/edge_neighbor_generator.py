"""Positive and negative neighbours for link prediction.

Same classes, arguments and results as dgf/src/generate/
edge_neighbor_generator.py:30-260: ``RandomNegativeSampler`` (uniform target
nodes), ``RandomWalkNegativeSampler`` (the sampler's
``RandomWalkNegativeSampling``, run on the GPU by
``dgfx_random_walk_negatives``), the two generator configs and
``EdgeNeighborGenerator``. The configs are plain dataclasses (the reference
also registers them for JSON round trips).
"""

from __future__ import annotations

import abc
import dataclasses
from typing import Optional, Union

import numpy as np

from distributed_graph_flow_b200.data import in_memory_graph as in_memory_graph_lib
from distributed_graph_flow_b200.data import schema as schema_lib
from distributed_graph_flow_b200.sampling import in_memory_sampler as in_memory_sampler_lib


class AbstractNegativeNeighborSampler(abc.ABC):
    """Samples negative target nodes for a batch of seed (positive) edges."""

    @abc.abstractmethod
    def sample(self, seed_edge_idxs: np.ndarray) -> np.ndarray:
        """[len(seed_edge_idxs), num_negative_neighbors] negative target node ids."""


class RandomNegativeSampler(AbstractNegativeNeighborSampler):
    """Uniform random nodes of the target edge set's target node set
    (edge_neighbor_generator.py:45-90), drawn with numpy's global generator."""

    def __init__(self, graph: in_memory_graph_lib.InMemoryGraph, schema: schema_lib.GraphSchema, target_edgeset: str,
                 num_negative_neighbors: int):
        self._schema = schema
        self._num_negative_neighbors = num_negative_neighbors
        self._num_nodes_in_target_nodeset = graph.node_sets[schema.edge_sets[target_edgeset].target].num_nodes

    def sample(self, seed_edge_idxs: np.ndarray) -> np.ndarray:
        return np.random.randint(0, self._num_nodes_in_target_nodeset,
                                 size=(len(seed_edge_idxs), self._num_negative_neighbors))


class RandomWalkNegativeSampler(AbstractNegativeNeighborSampler):
    """Negatives from random walks over ``sampler``'s plan
    (edge_neighbor_generator.py:93-132): the walks start at each seed edge's
    source node; see ``Sampler.RandomWalkNegativeSampling``."""

    def __init__(self, graph: in_memory_graph_lib.InMemoryGraph, schema: schema_lib.GraphSchema, target_edgeset: str,
                 num_negative_neighbors: int, sampler: in_memory_sampler_lib.Sampler, num_walks: int):
        self._graph = graph
        self._target_edgeset = target_edgeset
        self._schema = schema
        self._num_negative_neighbors = num_negative_neighbors
        self._num_nodes_in_target_nodeset = graph.node_sets[schema.edge_sets[target_edgeset].target].num_nodes
        self._sampler = sampler
        self._num_walks = num_walks
        self._target_edgeset_idx = self._sampler._cc_sampler.EdgesetNameToEdgesetIdx(target_edgeset)

    def _sample_from_seed_node_idxs(self, seed_node_idxs: np.ndarray) -> np.ndarray:
        return self._sampler._cc_sampler.RandomWalkNegativeSampling(
            seed_node_idxs=seed_node_idxs,
            target_edgeset_idx=self._target_edgeset_idx,
            num_walks=self._num_walks,
            num_negatives_per_seed=self._num_negative_neighbors,
        )

    def sample_device(self, seed_node_idxs, stream=None):
        """Device variant: int64 CUDA seed node ids in, int64 CUDA
        [num_seeds, num_negative_neighbors] out, asynchronous on ``stream``
        (errors are latched; ``self._sampler._cc_sampler.check_random_walk_negatives()``)."""
        return self._sampler._cc_sampler.random_walk_negatives(
            seed_node_idxs, self._target_edgeset_idx, self._num_walks, self._num_negative_neighbors, stream=stream,
            check=False)

    def sample(self, seed_edge_idxs: np.ndarray) -> np.ndarray:
        target_edgeset_data = self._graph.edge_sets[self._target_edgeset]
        seed_node_idxs = np.asarray(target_edgeset_data.adjacency)[0][seed_edge_idxs]
        return self._sample_from_seed_node_idxs(seed_node_idxs)


@dataclasses.dataclass
class EdgeNeighborIdxs:
    """Positive source / target node ids ([B]) and negative targets ([B, K])."""

    pos_src_node_idxs: np.ndarray
    pos_trg_node_idxs: np.ndarray
    neg_trg_node_idxs: np.ndarray


@dataclasses.dataclass
class RandomEdgeNeighborGeneratorConfig:
    pass


@dataclasses.dataclass
class RandomWalkEdgeNeighborGeneratorConfig:
    num_walks_per_negative: int = 10


EdgeNeighborGeneratorConfig = Union[RandomEdgeNeighborGeneratorConfig, RandomWalkEdgeNeighborGeneratorConfig]


class EdgeNeighborGenerator:
    """Positive pairs from seed edges plus negative targets
    (edge_neighbor_generator.py:178-260). The random-walk config runs
    num_walks_per_negative * num_negative_neighbors walks per seed."""

    def __init__(self, graph: in_memory_graph_lib.InMemoryGraph, schema: schema_lib.GraphSchema, target_edgeset: str,
                 num_negative_neighbors: int, *, sampler: Optional[in_memory_sampler_lib.Sampler] = None,
                 config: EdgeNeighborGeneratorConfig = RandomEdgeNeighborGeneratorConfig()):
        if isinstance(config, RandomEdgeNeighborGeneratorConfig):
            self._negative_node_sampler = RandomNegativeSampler(graph, schema, target_edgeset, num_negative_neighbors)
        elif isinstance(config, RandomWalkEdgeNeighborGeneratorConfig):
            if sampler is None:
                raise ValueError("A sampler must be provided when using the 'random-walk' method.")
            self._negative_node_sampler = RandomWalkNegativeSampler(
                graph, schema, target_edgeset, num_negative_neighbors, sampler,
                config.num_walks_per_negative * num_negative_neighbors)
        else:
            raise ValueError(f"Unknown negative sampling config: {type(config)}")
        self._target_edgeset_data = graph.edge_sets[target_edgeset]

    def generate(self, seed_edge_idxs: np.ndarray) -> EdgeNeighborIdxs:
        adjacency = np.asarray(self._target_edgeset_data.adjacency)
        return EdgeNeighborIdxs(
            pos_src_node_idxs=adjacency[0][seed_edge_idxs],
            pos_trg_node_idxs=adjacency[1][seed_edge_idxs],
            neg_trg_node_idxs=self._negative_node_sampler.sample(seed_edge_idxs),
        )
