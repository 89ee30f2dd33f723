"""Plan construction and the plan/index string formats (CPU only)."""

import numpy as np

from golden import reference_cases as rc
from helpers import temporal_graph, toy_graph

from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext
from distributed_graph_flow_b200.sampling import config as cfg
from distributed_graph_flow_b200.util import temporal as temporal_util


def test_simple_config_plan_string_matches_reference():
    graph, schema = toy_graph()
    plan = cfg.simple_sampling_config_to_sampling_plan(cfg.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2), schema)
    text = ext._plan_to_string(plan, schema.nodeset_index(), schema.edgeset_index())
    # The plan part of the reference's Sampler.__str__ golden.
    start = rc.TOY_SAMPLER_STR.index("SamplingPlan(")
    end = rc.TOY_SAMPLER_STR.index(",\n  nodeset_index")
    assert text == rc.TOY_SAMPLER_STR[start:end]


def test_plan_flattening():
    graph, schema = toy_graph()
    plan = cfg.simple_sampling_config_to_sampling_plan(cfg.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2), schema)
    pa = ext._PlanArrays(plan, schema.nodeset_index(), schema.edgeset_index())
    assert len(pa.node_nodeset) == 1 + 3 + 9
    assert pa.node_num_edges[0] == 3
    assert pa.edge_edgeset[:3] == [0, 0, 1]
    assert pa.edge_reversed[:3] == [0, 1, 0]
    for i, (f, n) in enumerate(zip(pa.node_first_edge, pa.node_num_edges)):
        for j in range(f, f + n):
            assert pa.edge_child[j] > i


def test_temporal_features_inferred():
    graph, schema = temporal_graph()
    assert temporal_util.edgeset_timestamp_features(schema) == {"e1": "timestamp"}
    plan = cfg.simple_sampling_config_to_sampling_plan(
        cfg.SimpleSamplingConfig(seed_nodeset="n1", num_hops=2, hop_width=2, reverse=False, temporal_sampling=True),
        schema,
    )
    assert plan.edgeset_timestamp_features == {"e1": "timestamp"}
    assert [c.edgeset for c in plan.root.children] == ["e1", "e2"]


def test_explicit_plan():
    plan = cfg.explicit_plan("n", "e", [10, 5])
    assert plan.root.children[0].hop_width == 10
    assert plan.root.children[0].node.children[0].hop_width == 5
    assert plan.root.children[0].node.children[0].node.children == []


def test_unknown_seed_nodeset():
    graph, schema = toy_graph()
    try:
        cfg.simple_sampling_config_to_sampling_plan(cfg.SimpleSamplingConfig(seed_nodeset="zz"), schema)
    except ValueError as e:
        assert "Seed nodeset 'zz' not found" in str(e)
    else:
        raise AssertionError("expected ValueError")
