"""Graph data model (boundary types of the sampler)."""

from distributed_graph_flow_b200.data.in_memory_graph import InMemoryEdgeSet, InMemoryGraph, InMemoryNodeSet
from distributed_graph_flow_b200.data.schema import (
    EdgeSchema,
    FeatureFormat,
    FeatureSchema,
    FeatureSemantic,
    GraphSchema,
    NodeSchema,
)
