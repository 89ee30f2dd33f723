"""Sampling configurations.

The dataclasses keep the names and fields of DGF's sampling API
(dgf/src/sampling/config.py:38-123) so existing plans work unchanged:
``SimpleSamplingConfig`` (one hop width for every hop), ``SamplingPlan`` (an
explicit tree of ``PlanNode`` / ``PlanEdge`` with a hop width per edge) and
``simple_sampling_config_to_sampling_plan`` (config.py:125-180).
"""

from __future__ import annotations

import collections
import dataclasses
from typing import Dict, List

from distributed_graph_flow_b200.data import schema as schema_lib
from distributed_graph_flow_b200.util import temporal as temporal_util


@dataclasses.dataclass
class SimpleSamplingConfig:
    """Breadth-style neighbourhood sampling from ``seed_nodeset``.

    Every hop follows every edge set touching the current node set (both
    directions when ``reverse``), taking up to ``hop_width`` neighbours per
    edge set. ``with_replacement`` turns the sample into a tree (repeated
    visits become new nodes); ``temporal_sampling`` enables the per-edge
    timestamp cutoff with timestamps inferred from the schema.
    """

    seed_nodeset: str
    num_hops: int = 3
    hop_width: int = 5
    reverse: bool = True
    with_replacement: bool = False
    temporal_sampling: bool = False


@dataclasses.dataclass
class PlanNode:
    nodeset: str
    children: List["PlanEdge"] = dataclasses.field(default_factory=list)


@dataclasses.dataclass
class PlanEdge:
    """One sampling step: up to ``hop_width`` neighbours over ``edgeset``."""

    edgeset: str
    reversed: bool
    node: PlanNode
    hop_width: int


@dataclasses.dataclass
class SamplingPlan:
    root: PlanNode
    with_replacement: bool = False
    temporal_sampling: bool = False
    edgeset_timestamp_features: Dict[str, str] = dataclasses.field(default_factory=dict)


def simple_sampling_config_to_sampling_plan(
    src: SimpleSamplingConfig, schema: schema_lib.GraphSchema
) -> SamplingPlan:
    """Expands a SimpleSamplingConfig into an explicit plan.

    Edge sets are visited in sorted-name order; with ``reverse`` every edge
    set is also walked backwards from its target node set.
    """
    if src.seed_nodeset not in schema.node_sets:
        raise ValueError(
            f"Seed nodeset '{src.seed_nodeset}' not found in the graph schema. The"
            f" available nodesets are: {list(schema.node_sets.keys())}"
        )
    links = collections.defaultdict(list)
    for name, es in sorted(schema.edge_sets.items()):
        links[es.source].append((name, es.target, False))
        if src.reverse:
            links[es.target].append((name, es.source, True))

    def build(nodeset: str, depth: int) -> PlanNode:
        children = []
        if depth < src.num_hops:
            for edgeset, other, rev in links.get(nodeset, []):
                children.append(
                    PlanEdge(edgeset=edgeset, reversed=rev, node=build(other, depth + 1), hop_width=src.hop_width)
                )
        return PlanNode(nodeset, children)

    ts_features = temporal_util.edgeset_timestamp_features(schema) if src.temporal_sampling else {}
    return SamplingPlan(
        root=build(src.seed_nodeset, 0),
        with_replacement=src.with_replacement,
        temporal_sampling=src.temporal_sampling,
        edgeset_timestamp_features=ts_features,
    )


def explicit_plan(
    seed_nodeset: str, edgeset: str, hop_widths: List[int], reversed_edges: bool = False
) -> SamplingPlan:
    """Homogeneous chain plan with one hop width per hop (e.g. [10, 5]).

    The per-hop fanouts used by GraphSAGE-style samplers; equivalent to an
    explicit SamplingPlan of nested PlanEdges over one edge set.
    """
    node = PlanNode(seed_nodeset)
    for hw in reversed(hop_widths):
        node = PlanNode(seed_nodeset, [PlanEdge(edgeset=edgeset, reversed=reversed_edges, node=node, hop_width=hw)])
    return SamplingPlan(root=node)
